// Recompute attention over the assembled cache: rows at arbitrary (sorted or not) positions
// attend to every cache key at a position <= their own (sm_100a, CUDA-core path).
//
// Replaces tread/blend.py:76 (mask = arange(T) <= S[:, None]) and :110
// (F.scaled_dot_product_attention(q, repeat_kv(K), repeat_kv(V), attn_mask=mask)) without the
// repeat_kv copies or a materialised mask: one CTA per (row, KV head) runs one warp per query
// head of the GQA group; the group's warps share each 32-key K/V tile staged in shared memory
// (fp32), and every warp keeps a flash-style online softmax (running max / sum, fp32).
//
// This path serves fp32 and head_dims 64 / 256 (and any dtype when the caller asks for it);
// bf16 / fp16 with head_dim 128 run on the tensor-core kernel in attn_tc.cu.
#include "common.cuh"

namespace tread {
namespace {

constexpr int kTile = 32;

template <typename T, int D>
__global__ void attn_rows_simt_kernel(const T* __restrict__ q, const T* __restrict__ Kc, const T* __restrict__ Vc,
                                      long long c_sh, long long T_cache, const int64_t* __restrict__ pos, int Hq,
                                      int G, float sm_scale, T* __restrict__ out, unsigned* err) {
  constexpr int DPL = D / 32;  // output dims per lane
  extern __shared__ float smem[];
  float* qs = smem;                    // [G][D]
  float* ks = qs + G * D;              // [kTile][D + 1]
  float* vs = ks + kTile * (D + 1);    // [kTile][D]
  const int r = blockIdx.x, g = blockIdx.y;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nthr = blockDim.x;
  const long long p = pos[r];
  if (p < 0 || p >= T_cache) {
    if (threadIdx.x == 0 && err) atomicOr(err, 2u);
    return;
  }
  const long long nkeys = p + 1;
  const T* Kg = Kc + g * c_sh;
  const T* Vg = Vc + g * c_sh;
  for (int i = threadIdx.x; i < G * D; i += nthr) {
    const int hh = i / D, d = i - hh * D;
    qs[i] = Num<T>::to_f(q[((long long)r * Hq + g * G + hh) * D + d]);
  }
  float m = -INFINITY, l = 0.f, o[DPL];
#pragma unroll
  for (int k = 0; k < DPL; ++k) o[k] = 0.f;
  const float* qw = qs + w * D;
#pragma unroll 1
  for (long long t0 = 0; t0 < nkeys; t0 += kTile) {
    __syncthreads();
    const int nt = (int)(nkeys - t0 < kTile ? nkeys - t0 : kTile);
    for (int i = threadIdx.x; i < kTile * D; i += nthr) {
      const int j = i / D, d = i - j * D;
      float kv = 0.f, vv = 0.f;
      if (j < nt) {
        kv = Num<T>::to_f(Kg[(t0 + j) * D + d]);
        vv = Num<T>::to_f(Vg[(t0 + j) * D + d]);
      }
      ks[j * (D + 1) + d] = kv;
      vs[j * D + d] = vv;
    }
    __syncthreads();
    if (w < G) {
      float s = -INFINITY;
      if (lane < nt) {
        const float* kr = ks + lane * (D + 1);
        float acc = 0.f;
#pragma unroll 8
        for (int d = 0; d < D; ++d) acc = fmaf(qw[d], kr[d], acc);
        s = acc * sm_scale;
      }
      float tmax = s;
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, off));
      const float m_new = fmaxf(m, tmax);
      const float pj = lane < nt ? expf(s - m_new) : 0.f;
      const float alpha = expf(m - m_new);
      float psum = pj;
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, off);
      l = l * alpha + psum;
#pragma unroll
      for (int k = 0; k < DPL; ++k) o[k] *= alpha;
      for (int jj = 0; jj < nt; ++jj) {
        const float pb = __shfl_sync(0xffffffffu, pj, jj);
        const float* vr = vs + jj * D + lane;
#pragma unroll
        for (int k = 0; k < DPL; ++k) o[k] = fmaf(pb, vr[32 * k], o[k]);
      }
      m = m_new;
    }
  }
  if (w < G) {
    const float inv = 1.f / l;
    T* orow = out + ((long long)r * Hq + g * G + w) * D;
#pragma unroll
    for (int k = 0; k < DPL; ++k) orow[lane + 32 * k] = Num<T>::from_f(o[k] * inv);
  }
}

template <typename T, int D>
int launch_simt(const void* q, const void* K, const void* V, long long c_sh, long long T_cache, const int64_t* pos,
                int R, int Hq, int Hkv, float sm_scale, void* out, unsigned* err, cudaStream_t st) {
  const int G = Hq / Hkv;
  const size_t smem = sizeof(float) * ((size_t)G * D + (size_t)kTile * (D + 1) + (size_t)kTile * D);
  auto kern = attn_rows_simt_kernel<T, D>;
  if (smem > 48 * 1024) TREAD_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                              (int)smem));
  dim3 grid(R, Hkv);
  kern<<<grid, 32 * G, smem, st>>>(static_cast<const T*>(q), static_cast<const T*>(K), static_cast<const T*>(V), c_sh,
                                  T_cache, pos, Hq, G, sm_scale, static_cast<T*>(out), err);
  TREAD_CHECK_LAUNCH("attn_rows_simt_kernel");
  return TREAD_OK;
}

template <typename T>
int dispatch_d(int D, const void* q, const void* K, const void* V, long long c_sh, long long T_cache,
               const int64_t* pos, int R, int Hq, int Hkv, float sm_scale, void* out, unsigned* err, cudaStream_t st) {
  switch (D) {
    case 64: return launch_simt<T, 64>(q, K, V, c_sh, T_cache, pos, R, Hq, Hkv, sm_scale, out, err, st);
    case 128: return launch_simt<T, 128>(q, K, V, c_sh, T_cache, pos, R, Hq, Hkv, sm_scale, out, err, st);
    default: return launch_simt<T, 256>(q, K, V, c_sh, T_cache, pos, R, Hq, Hkv, sm_scale, out, err, st);
  }
}

}  // namespace

int attn_rows_dispatch(const void* q, const void* K, const void* V, long long c_sh, long long T_cache,
                       const int64_t* pos, int R, int Hq, int Hkv, int D, float sm_scale, void* out, int dtype,
                       unsigned* err, void* ws, size_t ws_bytes, cudaStream_t st, int flags);
size_t attn_tc_workspace_bytes();

// CUDA-core recompute attention (all dtypes); the tensor-core path calls back into it for
// shapes it does not cover.
int attn_rows_simt(const void* q, const void* K, const void* V, long long c_sh, long long T_cache, const int64_t* pos,
                   int R, int Hq, int Hkv, int D, float sm_scale, void* out, int dtype, unsigned* err,
                   cudaStream_t st) {
  switch (dtype) {
    case TREAD_BF16:
      return dispatch_d<__nv_bfloat16>(D, q, K, V, c_sh, T_cache, pos, R, Hq, Hkv, sm_scale, out, err, st);
    case TREAD_F16: return dispatch_d<__half>(D, q, K, V, c_sh, T_cache, pos, R, Hq, Hkv, sm_scale, out, err, st);
    default: return dispatch_d<float>(D, q, K, V, c_sh, T_cache, pos, R, Hq, Hkv, sm_scale, out, err, st);
  }
}

}  // namespace tread

extern "C" size_t tread_attn_rows_workspace_bytes(void) { return tread::attn_tc_workspace_bytes(); }

extern "C" int tread_attn_rows(const void* q, const void* K_cache, const void* V_cache, int64_t cache_stride_head,
                               int64_t T_cache, const int64_t* q_pos, int R, int Hq, int Hkv, int D, float sm_scale,
                               void* out, int dtype, int flags, void* err_flag, void* workspace,
                               size_t workspace_bytes, tread_stream_t stream) {
  using namespace tread;
  TREAD_CHECK_ARG(R >= 0, "attn_rows: R < 0");
  if (R == 0) return TREAD_OK;
  TREAD_CHECK_ARG(q && K_cache && V_cache && q_pos && out, "attn_rows: null pointer");
  TREAD_CHECK_ARG(Hq > 0 && Hkv > 0 && Hq % Hkv == 0 && Hq / Hkv <= 16, "attn_rows: bad heads Hq=%d Hkv=%d", Hq,
                  Hkv);
  TREAD_CHECK_ARG(D == 64 || D == 128 || D == 256, "attn_rows: head_dim %d not in {64,128,256}", D);
  TREAD_CHECK_ARG(T_cache > 0 && cache_stride_head >= T_cache * D, "attn_rows: bad cache geometry");
  TREAD_CHECK_ARG(R <= 2147483647 && Hkv <= 65535, "attn_rows: grid too large");
  TREAD_CHECK_ARG(dtype_size(dtype) != 0, "attn_rows: unknown dtype %d", dtype);
  TREAD_CHECK_ARG((flags & ~7) == 0 && (flags & 6) != 6, "attn_rows: unknown flags %#x", flags);
  TREAD_CHECK_ARG(workspace == nullptr || (reinterpret_cast<uintptr_t>(workspace) & 255u) == 0,
                  "attn_rows: workspace not 256-byte aligned");
  return attn_rows_dispatch(q, K_cache, V_cache, cache_stride_head, T_cache, q_pos, R, Hq, Hkv, D, sm_scale, out,
                            dtype, static_cast<unsigned*>(err_flag), workspace, workspace ? workspace_bytes : 0,
                            reinterpret_cast<cudaStream_t>(stream), flags);
}
