// Recompute attention on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), sm_100a.
//
// Same contract as the CUDA-core path in attn_rows.cu (tread/blend.py:76,110 and the query
// forward of tread/engine.py:131-132): row r of head h attends to every cache key at a
// position <= pos[r] of KV head h / (Hq/Hkv). This path covers bf16/fp16 with head_dim 128.
//
// One CTA owns a tile of 128 consecutive rows of one query head; the heaviest tiles (latest
// positions, longest key ranges) are scheduled first. Roles and pipeline:
//   - loader (lane 0 of warp 9): TMA (128-byte swizzle) loads the Q tile once and 128-key K and V
//     tiles into separate 2-stage rings (two steps ahead of the MMAs that read them) straight
//     from the [R, Hq, D] queries and the [Hkv, T, D] cache, refilling a stage when the MMA that
//     read it commits to that stage's "free" barrier;
//   - MMA issuer (lane 0 of warp 8): issues S_j = Q K_j^T (8 x tcgen05.mma kind::f16,
//     M=N=K=128, operands in shared memory) into one of two TMEM S buffers, so the MMA of step
//     j+1 runs while the rows are still in the softmax of step j, and PV_j as two K=64 halves,
//     O_h += P_j[:, half h] V_j[half h, :], with P read from TMEM;
//   - softmax (warps 0-7; a row = a TMEM lane, its 128 key columns split into two halves, one
//     per warp): reads its half of S once with tcgen05.ld, masks keys past the row's position
//     (only on tiles that reach it), keeps the half's own running max and sum in the exp2 domain
//     (ex2.approx on the MUFU pipe, which stays below saturation), rescales the half's O
//     in TMEM only when its max grows by more than 8 (a stale max is exact since 1/l uses the
//     same max; a warp rescales together because tcgen05.ld/st are warp-collective), and writes
//     P (bf16/fp16 pairs) with tcgen05.st over the S columns it has just read. The halves never
//     wait for each other: they are merged once, in the epilogue, by their maxima;
//   - mbarriers hand off K/V stages, S buffers, P and PV completion between the roles; QK(j+2)
//     reuses S buffer j%2 after PV(j) has read the P in it.
// TMEM: two 128-column S buffers + one 128-column O accumulator per key half (512 allocated; one
// CTA per SM by its shared memory). Every wait is bounded in wall time and aborts the whole CTA
// through a shared flag; an aborted CTA records bit 2 in *err, lets issued copies and MMAs land,
// frees its TMEM and returns.
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
constexpr int kSmem = 10 * kBlock + 1024 + 256;
constexpr unsigned long long kWaitNs = 1000000000ull;  // 1 s: legitimate waits here take microseconds
constexpr unsigned long long kAbortWaitNs = 20000000ull;  // 20 ms per barrier phase on the abort path
// TMEM columns: S buffers 0-127 and 128-255 (fp32; each column half also holds that half's P,
// bf16/fp16 pairs, once read), O accumulators of key halves 0 and 1 at 256-383 and 384-511.
constexpr uint32_t kTmemO = 256;

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
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t phase, unsigned long long limit_ns) {
  if (mbar_try_wait(bar, phase)) return true;
  const unsigned long long t0 = global_ns();
  while (!mbar_try_wait(bar, phase))
    if (global_ns() - t0 > limit_ns) return false;
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

// Same with A (M x K, 16-bit elements packed two per 32-bit column, row = TMEM lane) in TMEM.
__device__ __forceinline__ void mma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t b, uint32_t idesc,
                                           uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(b), "r"(idesc), "r"(acc)
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

// Same, without the wait: several loads can be in flight before one tcgen05.wait::ld.
__device__ __forceinline__ void tmem_ld32_async(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
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

__device__ __forceinline__ void tmem_st32u(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
      "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
      "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
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

// Roles: warps 0-7 run the softmax: warp w covers TMEM lanes (rows) 32*(w%4).. and S/O columns
// 64*(w/4).. of its row quadrant, so every row is shared by two warps that exchange their partial
// max through shared memory; lane 0 of warp 8 issues every tcgen05.mma; lane 0 of warp 9 issues
// every TMA load, waiting only on the "stage free" barriers the MMAs commit, so loads never hold
// up MMA issue.
constexpr int kWarpsPerQuad = 2;
constexpr int kSoftWarps = 4 * kWarpsPerQuad;
constexpr int kColsPerWarp = kKeys / kWarpsPerQuad;  // 64
constexpr int kMmaWarp = kSoftWarps, kLoadWarp = kSoftWarps + 1;
constexpr int kThreadsTC = (kSoftWarps + 2) * 32;

struct Waiter {
  volatile int* abort;
  // Bounded wait on an mbarrier phase; false if the CTA aborted or kWaitNs passed (then it aborts).
  __device__ __forceinline__ bool operator()(uint64_t* bar, uint32_t parity) const {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = global_ns();
    while (!mbar_try_wait(bar, parity)) {
      if (*abort) return false;
      if (global_ns() - t0 > kWaitNs) {
        *abort = 1;
        return false;
      }
    }
    return true;
  }
};

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Barrier over the softmax warps that share a row quadrant (named barrier 1 + quadrant).
__device__ __forceinline__ void quad_sync(int quadrant) {
  asm volatile("bar.sync %0, %1;" ::"r"(1 + quadrant), "r"(kWarpsPerQuad * 32) : "memory");
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed two-wide fp32 arithmetic of sm_100 (one issue slot for two lanes' worth of work): the
// softmax is issue-bound, so halving its FMAs and adds shortens each step.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}

__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

template <typename T>
__global__ void __launch_bounds__(kThreadsTC, 1)
    attn_rows_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v, const int64_t* __restrict__ pos, int R, int Hq,
                        int G, long long T_cache, float scale_log2, T* __restrict__ out, unsigned* err) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sQ = smem;               // 2 blocks: d 0-63, d 64-127
  unsigned char* sK = smem + 2 * kBlock;  // 2 stages x 2 blocks
  unsigned char* sV = smem + 6 * kBlock;  // 2 stages x 2 blocks
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 10 * kBlock);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;   // [2] K stage loaded
  uint64_t* v_full = bars + 3;   // [2] V stage loaded
  uint64_t* s_full = bars + 5;   // [2] S buffer written by QK
  // bars 7-8: unused
  uint64_t* p_full = bars + 9;   // [2] P of S buffer b written by the softmax
  uint64_t* pv_done = bars + 11; // [2] PV of S buffer b's P complete (buffer reusable, O stable)
  uint64_t* k_free = bars + 13;  // [2] K stage read by its QK
  uint64_t* v_free = bars + 15;  // [2] V stage read by its PV
  constexpr int kNumBars = 17;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + kNumBars);
  int* s_abort = reinterpret_cast<int*>(bars + kNumBars + 1);
  __shared__ int s_wmax[4];
  __shared__ float s_part[2][kWarpsPerQuad][kRows];  // [step parity][column part][row]: max / final sum

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quad = warp & 3, part = warp >> 2;
  const int h = blockIdx.x, g = h / G;
  const int tile = gridDim.y - 1 - blockIdx.y;  // latest rows (longest key ranges) start first
  const int r0 = tile * kRows;
  const int trow = quad * 32 + lane;  // row within the tile (= TMEM lane)
  const int row = r0 + trow;
  const bool soft = warp < kSoftWarps;
  const bool live = soft && row < R;
  long long p = live ? pos[row] : 0;
  if (p < 0 || p >= T_cache) {
    if (live && part == 0 && err) atomicOr(err, 2u);
    p = 0;
  }
  if (warp < 4) {
    const int wm = __reduce_max_sync(0xffffffffu, (unsigned)p);
    if (lane == 0) s_wmax[warp] = wm;
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(s_tmem)),
                 "r"(512)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    mbar_init(q_full, 1);
    mbar_init(&k_full[0], 1);
    mbar_init(&k_full[1], 1);
    mbar_init(&v_full[0], 1);
    mbar_init(&v_full[1], 1);
    mbar_init(&s_full[0], 1);
    mbar_init(&s_full[1], 1);
    mbar_init(&p_full[0], kSoftWarps * 32);
    mbar_init(&p_full[1], kSoftWarps * 32);
    mbar_init(&pv_done[0], 1);
    mbar_init(&pv_done[1], 1);
    mbar_init(&k_free[0], 1);
    mbar_init(&k_free[1], 1);
    mbar_init(&v_free[0], 1);
    mbar_init(&v_free[1], 1);
    *s_abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  const int nsteps = max(max(s_wmax[0], s_wmax[1]), max(s_wmax[2], s_wmax[3])) / kKeys + 1;
  // padding rows past R (output discarded) see every key, so they never take the masking path
  if (soft && row >= R) p = (long long)nsteps * kKeys - 1;
  const Waiter wait{s_abort};

  if (warp == kLoadWarp) {
    // ------------------------------------------------------------------ TMA loader (one lane)
    // K and V have separate 2-stage rings; K(j+2) goes into its stage once QK(j) has read it and
    // V(j+2) once PV(j) has, so copies run two steps ahead of the MMAs.
    if (lane == 0) {
      auto load_k = [&](int j) {
        const int s = j & 1;
        mbar_expect_tx(&k_full[s], 2 * kBlock);
        tma_load_3d(sK + s * 2 * kBlock, &tm_k, &k_full[s], 0, j * kKeys, g);
        tma_load_3d(sK + s * 2 * kBlock + kBlock, &tm_k, &k_full[s], 64, j * kKeys, g);
      };
      auto load_v = [&](int j) {
        const int s = j & 1;
        mbar_expect_tx(&v_full[s], 2 * kBlock);
        tma_load_3d(sV + s * 2 * kBlock, &tm_v, &v_full[s], 0, j * kKeys, g);
        tma_load_3d(sV + s * 2 * kBlock + kBlock, &tm_v, &v_full[s], 64, j * kKeys, g);
      };
      mbar_expect_tx(q_full, 2 * kBlock);
      tma_load_3d(sQ, &tm_q, q_full, 0, h, r0);
      tma_load_3d(sQ + kBlock, &tm_q, q_full, 64, h, r0);
      for (int j = 0; j < nsteps && j < 2; ++j) {
        load_k(j);
        load_v(j);
      }
      for (int j = 0; j + 2 < nsteps; ++j) {
        const int s = j & 1;
        if (!wait(&k_free[s], (j >> 1) & 1)) break;
        load_k(j + 2);
        if (!wait(&v_free[s], (j >> 1) & 1)) break;
        load_v(j + 2);
      }
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------------ MMA issuer (one lane)
    if (lane == 0) {
      constexpr uint32_t fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
      constexpr uint32_t idesc_qk = idesc_f16(fmt, 0, kRows, kKeys);
      constexpr uint32_t idesc_pv = idesc_f16(fmt, 1, kRows, kD);
      const uint32_t aQ = smem_u32(sQ), aK = smem_u32(sK), aV = smem_u32(sV);
      // PV(j): O_h += P_j[:, keys of half h] V_j[keys of half h, :] for h = 0, 1; P of half h sits
      // in S buffer j%2 at columns 64*h .. 64*h+31 (packed pairs)
      auto issue_pv = [&](int j) {
        const int b = j & 1;
        const uint32_t vbase = aV + b * 2 * kBlock;
#pragma unroll
        for (int k = 0; k < kKeys / 16; ++k)
          mma_f16_ts(tmem + kTmemO + (k >> 2) * 128, tmem + b * kKeys + (k >> 2) * 64 + (k & 3) * 8,
                     sw128_desc(vbase + k * 16 * 128, kBlock, 1024), idesc_pv, (j > 0 || (k & 3) > 0) ? 1u : 0u);
        mma_commit(&pv_done[b]);
        mma_commit(&v_free[b]);
      };
      bool ok = true;
      for (int j = 0; j < nsteps && ok; ++j) {
        const int s = j & 1;
        // S buffer s holds P(j-2) until PV(j-2) has read it
        ok = wait(&k_full[s], (j >> 1) & 1) && (j > 0 || wait(q_full, 0)) &&
             (j < 2 || wait(&pv_done[s], ((j - 2) >> 1) & 1));
        if (!ok) break;
        tc_fence_after();
        const uint32_t kbase = aK + s * 2 * kBlock;
#pragma unroll
        for (int k = 0; k < kD / 16; ++k) {
          const uint32_t off = (k >> 2) * kBlock + (k & 3) * 32;
          mma_f16(tmem + s * kKeys, sw128_desc(aQ + off, 16, 1024), sw128_desc(kbase + off, 16, 1024), idesc_qk,
                  k > 0);
        }
        mma_commit(&s_full[s]);
        mma_commit(&k_free[s]);
        if (j >= 1) {
          const int b = (j - 1) & 1;
          ok = wait(&p_full[b], ((j - 1) >> 1) & 1) && wait(&v_full[b], ((j - 1) >> 1) & 1);
          if (!ok) break;
          tc_fence_after();
          issue_pv(j - 1);
        }
      }
      const int b = (nsteps - 1) & 1;
      if (ok && wait(&p_full[b], ((nsteps - 1) >> 1) & 1) && wait(&v_full[b], ((nsteps - 1) >> 1) & 1)) {
        tc_fence_after();
        issue_pv(nsteps - 1);
      }
    }
  } else {
    // ------------------------------------------------------------------ softmax
    // Each key half keeps its own running max, sum and O accumulator, so the two warps of a lane
    // quadrant never wait for each other; the halves are merged once, in the epilogue.
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t col = part * kColsPerWarp;
    const uint32_t tOh = tmem + kTmemO + part * 128;  // this half's O accumulator
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nsteps; ++j) {
      const int s = j & 1;
      ok = __all_sync(0xffffffffu, wait(&s_full[s], (j >> 1) & 1));
      if (!ok) break;
      tc_fence_after();
      float v[kColsPerWarp];
      {
        uint32_t r[kColsPerWarp / 32][32];
#pragma unroll
        for (int c = 0; c < kColsPerWarp / 32; ++c)
          tmem_ld32_async(tmem + s * kKeys + col + c * 32 + lane_off, r[c]);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
        for (int c = 0; c < kColsPerWarp / 32; ++c)
#pragma unroll
          for (int i = 0; i < 32; ++i) v[c * 32 + i] = __uint_as_float(r[c][i]);
      }
      const long long key0 = (long long)j * kKeys + col;
      if (__any_sync(0xffffffffu, key0 + kColsPerWarp - 1 > p)) {
        // keys i > lim of this half are past the row's position (one 32-bit compare each)
        const int lim = (int)max(-1LL, min((long long)kColsPerWarp, p - key0));
#pragma unroll
        for (int i = 0; i < kColsPerWarp; ++i)
          if (i > lim) v[i] = -INFINITY;
      }
      float m4[4] = {v[0], v[1], v[2], v[3]};  // four independent 3-input max chains
#pragma unroll
      for (int i = 4; i < kColsPerWarp; i += 2) m4[(i >> 1) & 3] = fmax3(m4[(i >> 1) & 3], v[i], v[i + 1]);
      const float tmax = fmax3(m4[0], m4[1], fmaxf(m4[2], m4[3]));
      const float m_new = fmaxf(m, tmax * scale_log2);  // -inf while every key of this half is masked
      const bool rescale = j > 0 && m_new > m + 8.f;
      float alpha = 1.f;
      if (j == 0 || rescale) {
        alpha = m == -INFINITY ? 0.f : ex2(m - m_new);
        l *= alpha;
        m = m_new;
      }
      const float mu = m == -INFINITY ? 0.f : m;  // all-masked half: exponentials of -inf give 0
      uint32_t pk[kColsPerWarp / 2];
      const float2 sc2 = make_float2(scale_log2, scale_log2), nm2 = make_float2(-mu, -mu);
      float2 l2 = make_float2(0.f, 0.f);  // even / odd key sums
#pragma unroll
      for (int i = 0; i < kColsPerWarp; i += 2) {
        const float2 x = ffma2(make_float2(v[i], v[i + 1]), sc2, nm2);
        const float2 pp = make_float2(ex2(x.x), ex2(x.y));
        l2 = fadd2(l2, pp);
        pk[i / 2] = pack2<T>(pp.x, pp.y);
      }
      l += l2.x + l2.y;
      // this half's O must be stable (PV(j-1) complete) to rescale it; tcgen05.ld/st are
      // warp-collective, so the warp rescales together, other lanes by 1
      if (__any_sync(0xffffffffu, rescale)) {
        ok = __all_sync(0xffffffffu, wait(&pv_done[s ^ 1], ((j - 1) >> 1) & 1));
        if (!ok) break;
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < kD / 32; ++c) {
          float o[32];
          tmem_ld32(tOh + lane_off + c * 32, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= alpha;
          tmem_st32(tOh + lane_off + c * 32, o);
        }
      }
      // P over this warp's own S columns (already in registers): QK(j+2) waits for PV(j)
      tmem_st32u(tmem + s * kKeys + part * 64 + lane_off, pk);
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      tc_fence_before();
      mbar_arrive(&p_full[s]);
    }
    if (ok) ok = __all_sync(0xffffffffu, wait(&pv_done[(nsteps - 1) & 1], ((nsteps - 1) >> 1) & 1));
    if (ok) {
      tc_fence_after();
      // merge the halves: O = (O_0 2^(m_0 - M) + O_1 2^(m_1 - M)) / (l_0 2^(m_0 - M) + l_1 2^(m_1 - M))
      s_part[0][part][trow] = m;
      s_part[1][part][trow] = l;
      quad_sync(quad);
      const float m0 = s_part[0][0][trow], m1 = s_part[0][1][trow];
      const float M = fmaxf(m0, m1);  // finite: key 0 is in half 0 and visible to every row
      const float a0 = m0 == -INFINITY ? 0.f : ex2(m0 - M), a1 = m1 == -INFINITY ? 0.f : ex2(m1 - M);
      const float inv = 1.f / (s_part[1][0][trow] * a0 + s_part[1][1][trow] * a1);
      const float c0 = a0 * inv, c1 = a1 * inv;
      T* orow = out + ((long long)row * Hq + h) * kD + col;
#pragma unroll 1
      for (int c = 0; c < kColsPerWarp / 32; ++c) {
        float o0[32], o1[32];
        tmem_ld32(tmem + kTmemO + col + lane_off + c * 32, o0);
        tmem_ld32(tmem + kTmemO + 128 + col + lane_off + c * 32, o1);
        if (live) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            float w8[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) w8[e] = fmaf(o0[i + e], c0, o1[i + e] * c1);
            uint4 w = make_uint4(pack2<T>(w8[0], w8[1]), pack2<T>(w8[2], w8[3]), pack2<T>(w8[4], w8[5]),
                                 pack2<T>(w8[6], w8[7]));
            *reinterpret_cast<uint4*>(orow + c * 32 + i) = w;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (*s_abort && tid == 0) {
    if (err) atomicOr(err, 4u);
    // let copies and MMAs already issued land before the CTA's resources go away: each barrier
    // an async unit arrives on gets a short bounded wait on both parities
    for (int b = 0; b < 2; ++b)
      for (int i = 0; i < kNumBars; ++i)
        if (i != 7 && i != 8 && i != 9 && i != 10) mbar_wait(bars + i, b, kAbortWaitNs);
  }
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512) : "memory");
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
  dim3 grid(Hq, (R + kRows - 1) / kRows);
  attn_rows_tc_kernel<T><<<grid, kThreadsTC, kSmem, st>>>(mq, mk, mv, pos, R, Hq, Hq / Hkv, T_cache, sm_scale * log2e,
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
