// Few-row projection GEMM on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), sm_100a.
//
// out[M, N] = (accumulate ? out : 0) + X[M, K] W[N, K]^T + bias[N] for M <= 128 rows, fp32
// accumulation rounded once. It replaces the Linear layers of the query forward when only the
// query segment's rows run (tread/engine.py:131-132: the q/k/v, o, gate/up, down projections and
// the lm_head of model(query_ids, past_key_values=cache)). With 64 rows a 7B layer reads 466 MB of
// weights for 30 GFLOP, so the GEMMs are bound by HBM, not by the tensor pipe.
//
// Layout: the MMA's M side is a tile of 128 output features (rows of W, K-major as stored) and
// its N side the Mp = round_up(M, 16) input rows (X, K-major), so no MMA row is padding when M
// is small. D^T sits in TMEM with one feature per lane and one input row per column.
//
// Work items are (pair of feature tiles, K split): the two tiles share each X chunk, so X takes a
// fifth of the ring at 64 rows, and the ring fills shared memory (5 stages of 40 KB at 64 rows,
// one CTA per SM) so that about 200 KB of weights are in flight per SM. With fewer pairs than SMs,
// K is split so that every SM streams weights. Each split stores its fp32 partial tile in its own
// workspace slot, and a second launch adds the slots in split order (so the result does not
// depend on timing), then bias and the old output, and writes out.
//
// Roles per CTA (192 threads):
//   - lane 0 of warp 0: TMA loads (per stage two W tiles of 128 x 64 and X of Mp x 64, 128-byte
//     swizzle);
//   - warp 1: the MMAs (one elected lane, 2 x 4 x K = 16 per stage, one TMEM accumulator per tile);
//   - warps 2-5: the epilogue, one TMEM lane quadrant each.
// Every wait is bounded in wall time. A CTA that gives up records bit 2 in *err, lets issued
// copies and MMAs land, frees its TMEM and returns.
#include <cuda.h>

#include <algorithm>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "tcgen05.cuh"

namespace tread {
namespace {

using namespace tc;

constexpr int kFeat = 128;                    // output features per MMA tile (MMA M)
constexpr int kTiles = 2;                     // feature tiles per CTA, sharing each X chunk
constexpr int kChunk = 64;                    // K elements per stage (one 128-byte swizzle row)
constexpr int kThreads = 192;
constexpr int kWBytes = kFeat * kChunk * 2;   // 16 KB per feature tile and stage
constexpr int kMaxRows = 128;
constexpr int kMaxStages = 8;
constexpr size_t kSmemLimit = 232448;         // opt-in shared memory per CTA on sm_100
// workspace: the K splits' partial slots, [item][row][256 features] fp32 (item = pair * nsplit +
// split)
constexpr size_t kWsBytes = (size_t)32 << 20;

int stage_bytes(int Mp) { return kTiles * kWBytes + Mp * 128; }
int stages_for(int Mp) { return std::min(kMaxStages, (int)((kSmemLimit - 2048) / stage_bytes(Mp))); }
size_t smem_bytes(int Mp) { return 1024 + (size_t)stages_for(Mp) * stage_bytes(Mp) + 256; }

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    rows_gemm_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x, int M,
                     int Mp, int N, int nchunks, int nsplit, int nstages, const T* __restrict__ bias, T* out,
                     long long ld_out, int accumulate, float* slots, unsigned* err) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int sbytes = kTiles * kWBytes + Mp * 128;  // one stage: the W tiles, then X (1024-byte aligned)
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + (size_t)nstages * sbytes);
  uint64_t* full = bars;                  // [nstages] stage loaded
  uint64_t* empty = bars + kMaxStages;    // [nstages] stage read by its MMAs
  uint64_t* done = bars + 2 * kMaxStages;  // the item's last MMA complete
  constexpr int kNumBars = 2 * kMaxStages + 1;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + kNumBars);
  int* s_abort = reinterpret_cast<int*>(s_tmem + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int pair = blockIdx.x / nsplit, split = blockIdx.x - pair * nsplit;
  const int c0 = (int)((long long)split * nchunks / nsplit);
  const int c1 = (int)((long long)(split + 1) * nchunks / nsplit);
  const uint32_t tcols = Mp <= 32 ? 32u : Mp <= 64 ? 64u : 128u;  // one accumulator (D^T of a tile)

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(s_tmem)),
                 "r"(kTiles * tcols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 32) {
    for (int i = 0; i < kNumBars; ++i) mbar_init(bars + i, 1);
    *s_abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  const Waiter wait{s_abort};

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA loader (one lane)
    if (lane == 0) {
      auto load_w = [&](int i) {
        const int s = i % nstages, c = c0 + i;
        unsigned char* st = smem + (size_t)s * sbytes;
        mbar_expect_tx(&full[s], (uint32_t)sbytes);
#pragma unroll
        for (int t = 0; t < kTiles; ++t)
          tma_load_2d(st + t * kWBytes, &tm_w, &full[s], c * kChunk, (pair * kTiles + t) * kFeat);
      };
      auto load_x = [&](int i) {
        tma_load_2d(smem + (size_t)(i % nstages) * sbytes + kTiles * kWBytes, &tm_x, &full[i % nstages],
                    (c0 + i) * kChunk, 0);
      };
      // the weights do not depend on the kernels before this one (launched as a programmatic
      // dependent): the first ring of them loads while those kernels finish, x only after
      const int nc = c1 - c0, pre = min(nstages, nc);
      for (int i = 0; i < pre; ++i) load_w(i);
      griddep_wait();
      for (int i = 0; i < pre; ++i) load_x(i);
      for (int i = pre; i < nc; ++i) {
        if (!wait(&empty[i % nstages], (uint32_t)(((i / nstages) - 1) & 1))) break;
        load_w(i);
        load_x(i);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (one warp)
    constexpr uint32_t fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
    const uint32_t idesc = idesc_f16(fmt, 0, kFeat, (uint32_t)Mp);
    bool ok = true;
    for (int c = c0, i = 0; c < c1; ++c, ++i) {
      const int s = i % nstages;
      ok = __all_sync(0xffffffffu, wait(&full[s], (uint32_t)((i / nstages) & 1)));
      if (!ok) break;
      tc_fence_after();
      const uint32_t st = smem_u32(smem + (size_t)s * sbytes);
      const uint64_t b0 = sw128_desc(st + kTiles * kWBytes, 16, 1024);
#pragma unroll
      for (int t = 0; t < kTiles; ++t) {
        const uint64_t a0 = sw128_desc(st + t * kWBytes, 16, 1024);
#pragma unroll
        for (int kk = 0; kk < kChunk / 16; ++kk)  // K = 16 per MMA: 32 bytes along the swizzled row
          mma_f16_elect(tmem + t * tcols, a0 + (uint64_t)((kk * 32) >> 4), b0 + (uint64_t)((kk * 32) >> 4), idesc,
                        (i > 0 || kk > 0) ? 1u : 0u);
      }
      mma_commit_elect(&empty[s]);
    }
    if (ok) mma_commit_elect(done);
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2-5)
    const int quad = warp & 3;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    // slot layout: [row][256 features], a warp's 32 lanes on 32 consecutive features
    const size_t slot_floats = (size_t)M * kTiles * kFeat;
    bool ok = __all_sync(0xffffffffu, wait(done, 0));
    if (ok) {
      tc_fence_after();
      griddep_wait();  // out (read when accumulating, then written) belongs to the kernels before
      if (tid == 64) griddep_launch_dependents();  // the split-adding launch may start
      float* my_slot = nsplit > 1 ? slots + (size_t)blockIdx.x * slot_floats : nullptr;
#pragma unroll
      for (int t = 0; t < kTiles; ++t) {
        const int fl = t * kFeat + quad * 32 + lane;  // feature within the pair
        const int f = pair * kTiles * kFeat + fl;
        const bool live = f < N;
        const float b = (bias && live) ? Num<T>::to_f(bias[f]) : 0.f;
        for (int r0 = 0; r0 < M; r0 += 32) {
          float v[32];
          tmem_ld32(tmem + t * tcols + lane_off + (uint32_t)r0, v);
          const int nr = min(32, M - r0);
          if (nsplit == 1) {
            if (live) {
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                if (j >= nr) break;
                T* o = out + (long long)(r0 + j) * ld_out + f;
                const float x = v[j] + b + (accumulate ? Num<T>::to_f(*o) : 0.f);
                *o = Num<T>::from_f(x);
              }
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j < nr) __stcg(my_slot + (size_t)(r0 + j) * (kTiles * kFeat) + fl, v[j]);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (*s_abort && tid == 0) {
    if (err) atomicOr(err, 4u);
    // let copies and MMAs already issued land before the CTA's resources go away
    for (int ph = 0; ph < 2; ++ph) {
      for (int i = 0; i < nstages; ++i) {
        mbar_wait(&full[i], (uint32_t)ph, kAbortWaitNs);
        mbar_wait(&empty[i], (uint32_t)ph, kAbortWaitNs);
      }
      mbar_wait(done, (uint32_t)ph, kAbortWaitNs);
    }
  }
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTiles * tcols)
                 : "memory");
  }
}

// Sum of the K splits' partial slots in split order, plus bias and the old output: one thread per
// four consecutive features of one row.
template <typename T>
__global__ void __launch_bounds__(256)
    rows_gemm_finalize_kernel(const float* __restrict__ slots, int M, int N, int npairs, int nsplit,
                              const T* __restrict__ bias, T* out, long long ld_out, int accumulate) {
  constexpr int kPairF = kTiles * kFeat;
  griddep_wait();  // the splits' slots come from the GEMM launch before
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;  // (row, pair, group of 4)
  const long long per_row = (long long)npairs * (kPairF / 4);
  if (i >= per_row * M) return;
  const int r = (int)(i / per_row);
  const int rest = (int)(i - (long long)r * per_row);
  const int pair = rest / (kPairF / 4), fl = (rest - pair * (kPairF / 4)) * 4;
  const size_t slot_floats = (size_t)M * kPairF;
  const float* src = slots + (size_t)pair * nsplit * slot_floats + (size_t)r * kPairF + fl;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int sp = 0; sp < nsplit; ++sp) {
    const float4 v = __ldcg(reinterpret_cast<const float4*>(src + (size_t)sp * slot_floats));
    acc.x += v.x, acc.y += v.y, acc.z += v.z, acc.w += v.w;
  }
  const float a[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int f = pair * kPairF + fl + e;
    if (f >= N) break;
    T* o = out + (long long)r * ld_out + f;
    *o = Num<T>::from_f(a[e] + (bias ? Num<T>::to_f(bias[f]) : 0.f) + (accumulate ? Num<T>::to_f(*o) : 0.f));
  }
}

bool make_map_2d(CUtensorMap* m, const void* base, CUtensorMapDataType dt, uint64_t inner, uint64_t rows,
                 uint64_t row_stride_elems, uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {inner, rows};
  const cuuint64_t strides[1] = {row_stride_elems * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kChunk, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int sm_count_cached() {
  static int cache[128] = {0};
  int d = 0;
  if (cudaGetDevice(&d) != cudaSuccess || d < 0 || d >= 128) return 148;
  if (!cache[d]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d) != cudaSuccess || n <= 0) n = 148;
    cache[d] = n;
  }
  return cache[d];
}

template <typename T>
int launch(const void* x, long long ldx, const void* w, long long ldw, const void* bias, void* out, long long ld_out,
           int M, int N, int K, int accumulate, unsigned* err, void* ws, size_t ws_bytes, cudaStream_t st) {
  const CUtensorMapDataType dt =
      std::is_same<T, __nv_bfloat16>::value ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const int Mp = (M + 15) / 16 * 16;
  CUtensorMap mw, mx;
  if (!make_map_2d(&mw, w, dt, (uint64_t)K, (uint64_t)N, (uint64_t)ldw, kFeat) ||
      !make_map_2d(&mx, x, dt, (uint64_t)K, (uint64_t)M, (uint64_t)ldx, (uint32_t)Mp)) {
    set_error("rows_gemm: cuTensorMapEncodeTiled failed");
    return TREAD_ERR_CUDA;
  }
  static std::once_flag attr_once;
  static cudaError_t attr_rc = cudaSuccess;
  std::call_once(attr_once, [] {
    size_t mx_smem = 0;
    for (int mp = 16; mp <= kMaxRows; mp += 16) mx_smem = std::max(mx_smem, smem_bytes(mp));
    attr_rc = cudaFuncSetAttribute(rows_gemm_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)mx_smem);
    if (attr_rc == cudaSuccess)
      attr_rc = cudaFuncSetAttribute(rows_gemm_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)mx_smem);
  });
  TREAD_CHECK_CUDA(attr_rc);
  const int npairs = (N + kTiles * kFeat - 1) / (kTiles * kFeat);
  const int nchunks = (K + kChunk - 1) / kChunk;
  // K split while the pairs of feature tiles do not fill the SMs (one CTA per SM fits: a second
  // wave would double the time), at least two chunks per split, and the partial slots must fit
  // the workspace
  int nsplit = 1;
  const int sms = sm_count_cached();
  if (ws && ws_bytes >= kWsBytes && npairs < sms) {
    const size_t per_split = (size_t)npairs * M * kTiles * kFeat * 4;
    nsplit = std::min(sms / npairs, nchunks / 2);  // one wave: at most one CTA per SM
    nsplit = (int)std::min<size_t>((size_t)nsplit, kWsBytes / per_split);
    nsplit = std::max(1, nsplit);
  }
  float* slots = nsplit > 1 ? static_cast<float*>(ws) : nullptr;
  // both launches are programmatic dependents of the work before them on the stream: they may
  // start while it finishes, and wait (griddepcontrol.wait) before touching what it wrote
  cudaLaunchAttribute pdl[1];
  pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  pdl[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(npairs * nsplit));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem_bytes(Mp);
  cfg.stream = st;
  cfg.attrs = pdl;
  cfg.numAttrs = 1;
  TREAD_CHECK_CUDA(cudaLaunchKernelEx(&cfg, rows_gemm_kernel<T>, mw, mx, M, Mp, N, nchunks, nsplit, stages_for(Mp),
                                     static_cast<const T*>(bias), static_cast<T*>(out), (long long)ld_out, accumulate,
                                     slots, err));
  if (nsplit > 1) {
    const long long threads = (long long)M * npairs * (kTiles * kFeat / 4);
    cfg.gridDim = dim3((unsigned)((threads + 255) / 256));
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = 0;
    TREAD_CHECK_CUDA(cudaLaunchKernelEx(&cfg, rows_gemm_finalize_kernel<T>, static_cast<const float*>(slots), M, N,
                                       npairs, nsplit, static_cast<const T*>(bias), static_cast<T*>(out),
                                       (long long)ld_out, accumulate));
  }
  return TREAD_OK;
}

}  // namespace
}  // namespace tread

extern "C" size_t tread_rows_gemm_workspace_bytes(void) { return tread::kWsBytes; }

extern "C" int tread_rows_gemm(const void* x, int64_t ldx, const void* w, int64_t ldw, const void* bias, void* out,
                               int64_t ld_out, int M, int N, int K, int accumulate, int dtype, void* err_flag,
                               void* workspace, size_t workspace_bytes, tread_stream_t stream) {
  using namespace tread;
  TREAD_CHECK_ARG(M >= 0 && N >= 0 && K >= 0, "rows_gemm: negative size");
  if (M == 0 || N == 0) return TREAD_OK;
  TREAD_CHECK_ARG(M <= kMaxRows, "rows_gemm: M=%d rows above %d", M, kMaxRows);
  TREAD_CHECK_ARG(K > 0, "rows_gemm: K == 0");
  TREAD_CHECK_ARG(x && w && out, "rows_gemm: null pointer");
  TREAD_CHECK_ARG(dtype == TREAD_BF16 || dtype == TREAD_F16, "rows_gemm: dtype %d is not bf16 / fp16", dtype);
  TREAD_CHECK_ARG(aligned16(x) && aligned16(w), "rows_gemm: x / w not 16-byte aligned");
  TREAD_CHECK_ARG(ldx >= K && ldw >= K && ld_out >= N, "rows_gemm: row stride below the row length");
  TREAD_CHECK_ARG(ldx % 8 == 0 && ldw % 8 == 0 && K % 8 == 0, "rows_gemm: K and the x / w row strides must be "
                  "multiples of 8 elements");
  TREAD_CHECK_ARG(N <= 0x7fffffff - kFeat, "rows_gemm: N too large");
  TREAD_CHECK_ARG(workspace == nullptr || (reinterpret_cast<uintptr_t>(workspace) & 255u) == 0,
                  "rows_gemm: workspace not 256-byte aligned");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  unsigned* err = static_cast<unsigned*>(err_flag);
  if (dtype == TREAD_BF16)
    return launch<__nv_bfloat16>(x, ldx, w, ldw, bias, out, ld_out, M, N, K, accumulate, err, workspace,
                                 workspace ? workspace_bytes : 0, st);
  return launch<__half>(x, ldx, w, ldw, bias, out, ld_out, M, N, K, accumulate, err, workspace,
                        workspace ? workspace_bytes : 0, st);
}
