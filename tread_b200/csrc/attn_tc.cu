// Recompute attention on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), sm_100a.
//
// Same contract as the CUDA-core path in attn_rows.cu (tread/blend.py:76,110 and the query
// forward of tread/engine.py:131-132): row r of head h attends to every cache key at a
// position <= pos[r] of KV head h / (Hq/Hkv). This path covers bf16/fp16 with head_dim 128.
//
// One CTA (128 threads = one warpgroup) owns a tile of 128 consecutive rows of one query head:
//   - TMA (128-byte swizzle) brings the Q tile once and a 128-key K tile and V tile per step
//     into shared memory, straight from the [R, Hq, D] queries and the [Hkv, T, D] cache;
//   - thread 0 issues S = Q K^T (M=128, N=128, K=128: 8 x tcgen05.mma kind::f16) into TMEM
//     columns [0,128) and commits to an mbarrier;
//   - each thread owns one row (= one TMEM lane): it reads its S row with tcgen05.ld, masks keys
//     past its position, and keeps an online softmax in the exp2 domain. The output accumulator
//     O lives in TMEM columns [128,256); it is rescaled (tcgen05.ld/st) only when the running
//     max grows by more than 8 (log2 units) — a stale max is exact because the final 1/l uses
//     the same max;
//   - P (bf16) is written to shared memory in the canonical K-major 128B-swizzled layout and
//     thread 0 issues O += P V (V as an MN-major B operand) into TMEM;
//   - at the end each thread reads its O row, divides by l and stores it.
// Every mbarrier wait is bounded; on timeout the CTA records bit 2 in *err, frees its TMEM and
// returns.
#include <cuda.h>

#include <mutex>
#include <type_traits>

#include "common.cuh"

namespace tread {

int attn_rows_simt(const void* q, const void* K, const void* V, long long c_sh, long long T_cache, const int64_t* pos,
                   int R, int Hq, int Hkv, int D, float sm_scale, void* out, int dtype, unsigned* err,
                   cudaStream_t st);

namespace {

constexpr int kRows = 128;   // query rows per CTA (MMA M)
constexpr int kKeys = 128;   // keys per step (MMA N of Q K^T, K of P V)
constexpr int kD = 128;      // head_dim (MMA K of Q K^T, N of P V)
constexpr int kBlock = 16384;  // one 128 x 64 bf16 swizzled block
constexpr int kSmem = 8 * kBlock + 1024 + 128;
constexpr unsigned long long kWaitNs = 1000000000ull;  // 1 s: legitimate waits here take microseconds

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(phase)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait: false if the phase did not complete within kWaitNs of wall time.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t phase) {
  if (mbar_try_wait(bar, phase)) return true;
  const unsigned long long t0 = global_ns();
  while (!mbar_try_wait(bar, phase))
    if (global_ns() - t0 > kWaitNs) return false;
  return true;
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// Shared-memory matrix descriptor, 128-byte swizzle (tcgen05 format: version 1 at bit 46,
// layout type 2 at bits 61-63), byte offsets encoded >> 4.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive fp32 TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
      "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
      "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])),
      "r"(__float_as_uint(v[17])), "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])),
      "r"(__float_as_uint(v[20])), "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])),
      "r"(__float_as_uint(v[23])), "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])),
      "r"(__float_as_uint(v[26])), "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])),
      "r"(__float_as_uint(v[29])), "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Instruction descriptor, kind::f16: fp32 accumulate (bit 4), A/B format (bits 7-9, 10-12:
// 0 = f16, 1 = bf16), B major (bit 16: 0 = K, 1 = MN), N >> 3 (bits 17-22), M >> 4 (bits 24-28).
__host__ __device__ constexpr uint32_t idesc_f16(uint32_t fmt, uint32_t b_mn_major, uint32_t M, uint32_t N) {
  return (1u << 4) | (fmt << 7) | (fmt << 10) | (b_mn_major << 16) | ((N >> 3) << 17) | ((M >> 4) << 24);
}

template <typename T>
__global__ void __launch_bounds__(128, 1)
    attn_rows_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v, const int64_t* __restrict__ pos, int R, int Hq,
                        int G, long long T_cache, float scale_log2, T* __restrict__ out, unsigned* err) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sQ = smem;               // 2 blocks: d 0-63, d 64-127
  unsigned char* sK = smem + 2 * kBlock;  // 2 blocks
  unsigned char* sV = smem + 4 * kBlock;  // 2 blocks
  unsigned char* sP = smem + 6 * kBlock;  // 2 blocks: keys 0-63, 64-127
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 8 * kBlock);  // [0] Q, [1] K/V, [2] MMA
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + 4);
  int* s_flag = reinterpret_cast<int*>(bars + 5);

  const int tid = threadIdx.x, warp = tid >> 5;
  const int h = blockIdx.y, g = h / G;
  const int r0 = blockIdx.x * kRows;
  const int row = r0 + tid;
  const bool live = row < R;
  long long p = live ? pos[row] : 0;
  if (p < 0 || p >= T_cache) {
    if (live && err) atomicOr(err, 2u);
    p = 0;
  }
  const int maxpos = __reduce_max_sync(0xffffffffu, (unsigned)p);
  __shared__ int s_wmax[4];
  if ((tid & 31) == 0) s_wmax[warp] = maxpos;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(s_tmem)),
                 "r"(256)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    mbar_init(&bars[2], 1);
    *s_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  const uint32_t tS = tmem, tO = tmem + 128;
  const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
  const int nsteps = max(max(s_wmax[0], s_wmax[1]), max(s_wmax[2], s_wmax[3])) / kKeys + 1;

  constexpr uint32_t fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
  constexpr uint32_t idesc_qk = idesc_f16(fmt, 0, kRows, kKeys);
  constexpr uint32_t idesc_pv = idesc_f16(fmt, 1, kRows, kD);
  const uint32_t aQ = smem_u32(sQ), aK = smem_u32(sK), aV = smem_u32(sV), aP = smem_u32(sP);

  if (tid == 0) {
    mbar_expect_tx(&bars[0], 2 * kBlock);
    tma_load_3d(sQ, &tm_q, &bars[0], 0, h, r0);
    tma_load_3d(sQ + kBlock, &tm_q, &bars[0], 64, h, r0);
  }

  float m = -INFINITY, l = 0.f;
  bool ok = true;
  uint32_t mma_phase = 0;
#pragma unroll 1
  for (int j = 0; j < nsteps && ok; ++j) {
    if (tid == 0) {
      mbar_expect_tx(&bars[1], 4 * kBlock);
      tma_load_3d(sK, &tm_k, &bars[1], 0, j * kKeys, g);
      tma_load_3d(sK + kBlock, &tm_k, &bars[1], 64, j * kKeys, g);
      tma_load_3d(sV, &tm_v, &bars[1], 0, j * kKeys, g);
      tma_load_3d(sV + kBlock, &tm_v, &bars[1], 64, j * kKeys, g);
    }
    bool w = true;
    if (j == 0) w = mbar_wait(&bars[0], 0);
    w = w && mbar_wait(&bars[1], j & 1);
    if (!__syncthreads_and(w)) {
      ok = false;
      break;
    }
    // S = Q K^T
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int k = 0; k < kD / 16; ++k) {
        const uint32_t off = (k >> 2) * kBlock + (k & 3) * 32;
        mma_f16(tS, sw128_desc(aQ + off, 16, 1024), sw128_desc(aK + off, 16, 1024), idesc_qk, k > 0);
      }
      mma_commit(&bars[2]);
    }
    if (!__syncthreads_and(mbar_wait(&bars[2], mma_phase))) {
      ok = false;
      break;
    }
    mma_phase ^= 1;
    tc_fence_after();

    // online softmax over this row's 128 scores (exp2 domain)
    const int key0 = j * kKeys;
    float tmax = -INFINITY;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      float v[32];
      tmem_ld32(tS + lane_off + c * 32, v);
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (key0 + c * 32 + i <= p) tmax = fmaxf(tmax, v[i] * scale_log2);
    }
    const float m_new = fmaxf(m, tmax);
    const bool rescale = j > 0 && m_new > m + 8.f;
    float alpha = 1.f;
    if (j == 0 || rescale) {
      alpha = exp2f(m - m_new);  // 0 for the first step
      l *= alpha;
      m = m_new;
    }
    // tcgen05.ld / tcgen05.st are warp-collective (.sync.aligned): the O rows of a warp are
    // rescaled together whenever any lane needs it, the other lanes multiplying by 1.
    if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float v[32];
        tmem_ld32(tO + lane_off + c * 32, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] *= alpha;
        tmem_st32(tO + lane_off + c * 32, v);
      }
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
    }
    // P row -> shared memory, K-major 128B-swizzled: 16-byte chunk q of an 8-row atom row goes to q ^ (row % 8)
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      float v[32];
      tmem_ld32(tS + lane_off + c * 32, v);
      uint32_t pk[16];
#pragma unroll
      for (int i = 0; i < 32; i += 2) {
        const float p0 = (key0 + c * 32 + i <= p) ? exp2f(v[i] * scale_log2 - m) : 0.f;
        const float p1 = (key0 + c * 32 + i + 1 <= p) ? exp2f(v[i + 1] * scale_log2 - m) : 0.f;
        l += p0 + p1;
        pk[i / 2] = pack2<T>(p0, p1);
      }
      unsigned char* blk = sP + (c >> 1) * kBlock + (tid >> 3) * 1024 + (tid & 7) * 128;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int chunk = (c & 1) * 4 + q;
        *reinterpret_cast<uint4*>(blk + ((chunk ^ (tid & 7)) << 4)) =
            make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
      }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc_fence_before();
    __syncthreads();
    // O += P V
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int k = 0; k < kKeys / 16; ++k) {
        const uint32_t offp = (k >> 2) * kBlock + (k & 3) * 32;
        const uint32_t offv = k * 16 * 128;  // 16 keys x 128 B per K step
        mma_f16(tO, sw128_desc(aP + offp, 16, 1024), sw128_desc(aV + offv, kBlock, 1024), idesc_pv,
                (j > 0 || k > 0) ? 1u : 0u);
      }
      mma_commit(&bars[2]);
    }
    if (!__syncthreads_and(mbar_wait(&bars[2], mma_phase))) {
      ok = false;
      break;
    }
    mma_phase ^= 1;
    tc_fence_after();
  }

  if (ok) {
    const float inv = 1.f / l;
    T* orow = out + ((long long)row * Hq + h) * kD;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      float v[32];
      tmem_ld32(tO + lane_off + c * 32, v);
      if (live) {
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          uint4 o = make_uint4(pack2<T>(v[i] * inv, v[i + 1] * inv), pack2<T>(v[i + 2] * inv, v[i + 3] * inv),
                               pack2<T>(v[i + 4] * inv, v[i + 5] * inv), pack2<T>(v[i + 6] * inv, v[i + 7] * inv));
          *reinterpret_cast<uint4*>(orow + c * 32 + i) = o;
        }
      }
    }
  } else if (tid == 0) {
    if (err) atomicOr(err, 4u);
    // let any TMA still in flight into our shared memory land before the CTA exits
    mbar_wait(&bars[1], 0);
    mbar_wait(&bars[1], 1);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(256) : "memory");
  }
}

// ---- host side: tensor maps -----------------------------------------------------------------

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 3-D bf16/fp16 map over (d, y, z) with element strides (1, sy, sz), box (64, by, bz), 128B swizzle.
bool make_map(CUtensorMap* m, const void* base, CUtensorMapDataType dt, uint64_t nd, uint64_t ny, uint64_t nz,
              uint64_t sy, uint64_t sz, uint32_t by, uint32_t bz) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[3] = {nd, ny, nz};
  const cuuint64_t strides[2] = {sy * 2, sz * 2};
  const cuuint32_t box[3] = {64, by, bz};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(m, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename T>
int launch_tc(const void* q, const void* K, const void* V, long long c_sh, long long T_cache, const int64_t* pos,
              int R, int Hq, int Hkv, float sm_scale, void* out, unsigned* err, cudaStream_t st) {
  const CUtensorMapDataType dt =
      std::is_same<T, __nv_bfloat16>::value ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap mq, mk, mv;
  if (!make_map(&mq, q, dt, kD, Hq, R, kD, (uint64_t)Hq * kD, 1, kRows) ||
      !make_map(&mk, K, dt, kD, T_cache, Hkv, kD, c_sh, kKeys, 1) ||
      !make_map(&mv, V, dt, kD, T_cache, Hkv, kD, c_sh, kKeys, 1)) {
    set_error("attn_rows: cuTensorMapEncodeTiled failed");
    return TREAD_ERR_CUDA;
  }
  static std::once_flag attr_once;
  static cudaError_t attr_rc = cudaSuccess;
  std::call_once(attr_once, [] {
    attr_rc = cudaFuncSetAttribute(attn_rows_tc_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   kSmem);
    if (attr_rc == cudaSuccess)
      attr_rc = cudaFuncSetAttribute(attn_rows_tc_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
  });
  TREAD_CHECK_CUDA(attr_rc);
  const float log2e = 1.4426950408889634f;
  dim3 grid((R + kRows - 1) / kRows, Hq);
  attn_rows_tc_kernel<T><<<grid, 128, kSmem, st>>>(mq, mk, mv, pos, R, Hq, Hq / Hkv, T_cache, sm_scale * log2e,
                                                   static_cast<T*>(out), err);
  TREAD_CHECK_LAUNCH("attn_rows_tc_kernel");
  return TREAD_OK;
}

}  // namespace

// Tensor-core path for bf16/fp16 with head_dim 128; everything else runs on CUDA cores.
int attn_rows_dispatch(const void* q, const void* K, const void* V, long long c_sh, long long T_cache,
                       const int64_t* pos, int R, int Hq, int Hkv, int D, float sm_scale, void* out, int dtype,
                       unsigned* err, cudaStream_t st, int force_simt) {
  const bool tc_ok = D == kD && (dtype == TREAD_BF16 || dtype == TREAD_F16) && !force_simt &&
                     (reinterpret_cast<uintptr_t>(q) % 16 == 0) && (reinterpret_cast<uintptr_t>(K) % 16 == 0) &&
                     (reinterpret_cast<uintptr_t>(V) % 16 == 0) && (c_sh * 2) % 16 == 0 && R <= 0x7fffffff - kRows;
  if (!tc_ok) return attn_rows_simt(q, K, V, c_sh, T_cache, pos, R, Hq, Hkv, D, sm_scale, out, dtype, err, st);
  if (dtype == TREAD_BF16) return launch_tc<__nv_bfloat16>(q, K, V, c_sh, T_cache, pos, R, Hq, Hkv, sm_scale, out, err, st);
  return launch_tc<__half>(q, K, V, c_sh, T_cache, pos, R, Hq, Hkv, sm_scale, out, err, st);
}

}  // namespace tread
