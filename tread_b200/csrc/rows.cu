// Per-row RoPE + K/V splice for recomputed token rows (sm_100a).
//
// Replaces, for the rows being recomputed at a layer, tread/blend.py:82-90 (`_qkv`: split the
// q/k/v projections, apply_rotary_pos_emb at each row's position) and tread/blend.py:106
// (`K[:, :, S], V[:, :, S] = k, v`): one CTA per row computes that row's D/2 cos/sin once,
// rotates the row's q heads into the attention input and its k heads straight into the layer
// cache at the row's position, and copies its v heads there too.
//
// RoPE at absolute position p (transformers Qwen2RotaryEmbedding + apply_rotary_pos_emb):
//   angle_i = float(p) * inv_freq[i];  c_i = cos(angle_i) * s;  s_i = sin(angle_i) * s
//   x'[i] = x[i]*c_i - x[i+D/2]*s_i,  x'[i+D/2] = x[i+D/2]*c_i + x[i]*s_i   (fp32, rounded once)
#include "common.cuh"

namespace tread {
namespace {

constexpr int kThreads = 128;
constexpr int kMaxHalf = 128;

struct Freq {
  float inv[kMaxHalf];
};

template <typename T>
__global__ void __launch_bounds__(kThreads)
    rope_rows_kernel(const T* __restrict__ qkv, long long ld, const int64_t* __restrict__ pos, int Hq, int Hkv,
                     int D, T* __restrict__ q_out, T* __restrict__ Kc, T* __restrict__ Vc, long long c_sh,
                     long long T_cache, int kv_by_row, const __grid_constant__ Freq f, float scale, unsigned* err,
                     int vec) {
  __shared__ float s_cos[kMaxHalf], s_sin[kMaxHalf];
  const int r = blockIdx.x;
  const long long p = pos[r];
  const long long slot = kv_by_row ? r : p;  // cache row that receives this row's k/v
  if (p < 0 || (!kv_by_row && p >= T_cache)) {
    if (threadIdx.x == 0 && err) atomicOr(err, 1u);
    return;
  }
  const int half = D >> 1;
  for (int i = threadIdx.x; i < half; i += kThreads) {
    float sn, cs;
    sincosf(__fmul_rn((float)p, f.inv[i]), &sn, &cs);
    s_cos[i] = __fmul_rn(cs, scale);
    s_sin[i] = __fmul_rn(sn, scale);
  }
  __syncthreads();
  const T* row = qkv + (long long)r * ld;
  const int q0 = q_out ? 0 : Hq;  // no q output: rotate the k heads only
  if (vec) {
    // 16-byte vectors: VEC consecutive pairs (i, i + D/2) of one head per step, same fp32 math
    constexpr int VEC = 16 / sizeof(T);
    const int hv = half / VEC;
    const int nvec = (Hq + Hkv - q0) * hv;
    for (int w = threadIdx.x; w < nvec; w += kThreads) {
      const int head = q0 + w / hv, i0 = (w % hv) * VEC;
      const T* src = row + head * D + i0;
      Vec16<T> a, b, oa, ob;
      a.raw = __ldg(reinterpret_cast<const int4*>(src));
      b.raw = __ldg(reinterpret_cast<const int4*>(src + half));
#pragma unroll
      for (int e = 0; e < VEC; ++e) {
        const float x1 = Num<T>::to_f(a.e[e]), x2 = Num<T>::to_f(b.e[e]);
        oa.e[e] = Num<T>::from_f(__fsub_rn(__fmul_rn(x1, s_cos[i0 + e]), __fmul_rn(x2, s_sin[i0 + e])));
        ob.e[e] = Num<T>::from_f(__fadd_rn(__fmul_rn(x2, s_cos[i0 + e]), __fmul_rn(x1, s_sin[i0 + e])));
      }
      T* dst = head < Hq ? q_out + ((long long)r * Hq + head) * D : Kc + (head - Hq) * c_sh + slot * D;
      *reinterpret_cast<int4*>(dst + i0) = oa.raw;
      *reinterpret_cast<int4*>(dst + i0 + half) = ob.raw;
    }
    const T* vsrc = row + (Hq + Hkv) * D;
    const int vpd = D / VEC;
    for (int w = threadIdx.x; w < Hkv * vpd; w += kThreads) {
      const int g = w / vpd, d = (w - g * vpd) * VEC;
      *reinterpret_cast<int4*>(Vc + g * c_sh + slot * D + d) =
          __ldg(reinterpret_cast<const int4*>(vsrc + g * D + d));
    }
    return;
  }
  const int nrot = (Hq + Hkv - q0) * half;  // rotation pairs over q heads then k heads
  for (int w = threadIdx.x; w < nrot; w += kThreads) {
    const int head = q0 + w / half, i = w % half;
    const T* src = row + head * D;
    const float x1 = Num<T>::to_f(src[i]), x2 = Num<T>::to_f(src[i + half]);
    const float o1 = __fsub_rn(__fmul_rn(x1, s_cos[i]), __fmul_rn(x2, s_sin[i]));
    const float o2 = __fadd_rn(__fmul_rn(x2, s_cos[i]), __fmul_rn(x1, s_sin[i]));
    T* dst = head < Hq ? q_out + ((long long)r * Hq + head) * D : Kc + (head - Hq) * c_sh + slot * D;
    dst[i] = Num<T>::from_f(o1);
    dst[i + half] = Num<T>::from_f(o2);
  }
  const T* vsrc = row + (Hq + Hkv) * D;
  for (int w = threadIdx.x; w < Hkv * D; w += kThreads) {
    const int g = w / D, d = w - g * D;
    Vc[g * c_sh + slot * D + d] = vsrc[w];
  }
}

}  // namespace
}  // namespace tread

extern "C" int tread_rope_rows(const void* qkv, int64_t ld_qkv, const int64_t* pos, int R, int Hq, int Hkv, int D,
                               void* q_out, void* K_cache, void* V_cache, int64_t cache_stride_head,
                               int64_t T_cache, int kv_by_row, const float* inv_freq, float attn_scaling,
                               int dtype, void* err_flag, tread_stream_t stream) {
  using namespace tread;
  TREAD_CHECK_ARG(R >= 0, "rope_rows: R < 0");
  if (R == 0) return TREAD_OK;
  TREAD_CHECK_ARG(qkv && pos && K_cache && V_cache && inv_freq, "rope_rows: null pointer");
  // Hq == 0 (no q output): the rows hold only [k heads | v heads]
  TREAD_CHECK_ARG(Hkv > 0 && (Hq > 0 ? Hq % Hkv == 0 : (Hq == 0 && q_out == nullptr)),
                  "rope_rows: bad heads Hq=%d Hkv=%d (Hq = 0 needs q_out == NULL)", Hq, Hkv);
  TREAD_CHECK_ARG(D >= 2 && D % 2 == 0 && D / 2 <= kMaxHalf, "rope_rows: bad head_dim %d", D);
  TREAD_CHECK_ARG(ld_qkv >= (int64_t)(Hq + 2 * Hkv) * D, "rope_rows: ld_qkv %lld too small", (long long)ld_qkv);
  TREAD_CHECK_ARG(T_cache > 0 && cache_stride_head >= T_cache * D, "rope_rows: bad cache geometry");
  TREAD_CHECK_ARG(!kv_by_row || T_cache >= R, "rope_rows: kv_by_row needs T_cache >= R");
  TREAD_CHECK_ARG(dtype_size(dtype) != 0, "rope_rows: unknown dtype %d", dtype);
  Freq f;
  for (int i = 0; i < D / 2; ++i) f.inv[i] = inv_freq[i];
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  unsigned* err = static_cast<unsigned*>(err_flag);
  // 16-byte vector path when every row, head half and cache slot starts on a 16-byte boundary
  const int64_t vec_el = 16 / (int64_t)dtype_size(dtype);
  auto al16 = [](const void* p) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  const int vec = (D / 2) % vec_el == 0 && ld_qkv % vec_el == 0 && cache_stride_head % vec_el == 0 && al16(qkv) &&
                  al16(q_out) && al16(K_cache) && al16(V_cache);
  switch (dtype) {
    case TREAD_BF16:
      rope_rows_kernel<__nv_bfloat16><<<R, kThreads, 0, st>>>(
          static_cast<const __nv_bfloat16*>(qkv), ld_qkv, pos, Hq, Hkv, D, static_cast<__nv_bfloat16*>(q_out),
          static_cast<__nv_bfloat16*>(K_cache), static_cast<__nv_bfloat16*>(V_cache), cache_stride_head, T_cache, kv_by_row, f,
          attn_scaling, err, vec);
      break;
    case TREAD_F16:
      rope_rows_kernel<__half><<<R, kThreads, 0, st>>>(
          static_cast<const __half*>(qkv), ld_qkv, pos, Hq, Hkv, D, static_cast<__half*>(q_out),
          static_cast<__half*>(K_cache), static_cast<__half*>(V_cache), cache_stride_head, T_cache, kv_by_row, f, attn_scaling,
          err, vec);
      break;
    default:
      rope_rows_kernel<float><<<R, kThreads, 0, st>>>(
          static_cast<const float*>(qkv), ld_qkv, pos, Hq, Hkv, D, static_cast<float*>(q_out),
          static_cast<float*>(K_cache), static_cast<float*>(V_cache), cache_stride_head, T_cache, kv_by_row, f, attn_scaling,
          err, vec);
      break;
  }
  TREAD_CHECK_LAUNCH("rope_rows_kernel");
  return TREAD_OK;
}
