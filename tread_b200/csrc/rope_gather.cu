// Fused gather + RoPE re-rotation + append of cached KV blocks (sm_100a).
//
// Replaces tread/engine.py:108-120 (per-block rotate_keys, tread/blend.py:22-39, then one
// torch.cat per K/V) with a single memory-bound pass: every byte of the hit blocks is read
// once and every byte of the assembled cache is written once, with no temporaries.
//
// Work decomposition: one CTA per (segment, layer*head, 64-token tile). A (layer, head)
// slice of a block is contiguous in both the block ([L, Hkv, n, D]) and the assembled cache
// ([L, Hkv, T_out, D]), so a tile is two contiguous 64*D-element runs (K and V) on each side.
// The rotation angle depends only on (segment, frequency), so a CTA computes its D/2 cos/sin
// pairs once in shared memory; each thread then always touches the same D/2-column group
// and keeps its cos/sin in registers. All global traffic is 16-byte vectors with streaming
// cache hints (the source pool and the assembled cache are both far larger than L2).
#include "common.cuh"

namespace tread {
namespace {

constexpr int kMaxSeg = 48;    // segments per launch (kernel-parameter table)
constexpr int kMaxHalf = 128;  // D <= 256
constexpr int kThreads = 256;
constexpr int kTileTok = 64;

struct RopeTable {
  const void* k[kMaxSeg];
  const void* v[kMaxSeg];
  long long dst0[kMaxSeg];
  int n[kMaxSeg];
  int delta[kMaxSeg];
  int tile0[kMaxSeg + 1];  // exclusive prefix sum of tiles per segment
  float inv_freq[kMaxHalf];
};

template <typename T>
__device__ __forceinline__ int4 rot_first(int4 a, int4 b, const float* c, const float* s) {
  constexpr int VEC = 16 / sizeof(T);
  Vec16<T> A, B, O;
  A.raw = a;
  B.raw = b;
#pragma unroll
  for (int j = 0; j < VEC; ++j) {
    const float x1 = Num<T>::to_f(A.e[j]), x2 = Num<T>::to_f(B.e[j]);
    // fl(fl(x1*c) + fl(-x2*s)): the fp32 order of K*cos + rotate_half(K)*sin.
    O.e[j] = Num<T>::from_f(__fsub_rn(__fmul_rn(x1, c[j]), __fmul_rn(x2, s[j])));
  }
  return O.raw;
}

template <typename T>
__device__ __forceinline__ int4 rot_second(int4 a, int4 b, const float* c, const float* s) {
  constexpr int VEC = 16 / sizeof(T);
  Vec16<T> A, B, O;
  A.raw = a;
  B.raw = b;
#pragma unroll
  for (int j = 0; j < VEC; ++j) {
    const float x1 = Num<T>::to_f(A.e[j]), x2 = Num<T>::to_f(B.e[j]);
    O.e[j] = Num<T>::from_f(__fadd_rn(__fmul_rn(x2, c[j]), __fmul_rn(x1, s[j])));
  }
  return O.raw;
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
    rope_gather_append_kernel(const __grid_constant__ RopeTable p, int nseg, T* __restrict__ out_k,
                              T* __restrict__ out_v, int D, long long T_out, float scale) {
  constexpr int VEC = 16 / sizeof(T);
  __shared__ float s_cos[kMaxHalf];
  __shared__ float s_sin[kMaxHalf];

  const int tile = blockIdx.x;
  int s = 0;
#pragma unroll 1
  while (s + 1 < nseg && p.tile0[s + 1] <= tile) ++s;
  const int n = p.n[s];
  const int ntt = (n + kTileTok - 1) / kTileTok;
  const int local = tile - p.tile0[s];
  const int lh = local / ntt;
  const int t0 = (local - lh * ntt) * kTileTok;
  const int rows = min(kTileTok, n - t0);
  const int half = D >> 1;
  const int delta = p.delta[s];

  const size_t src_off = ((size_t)lh * n + t0) * D;
  const size_t dst_off = ((size_t)lh * T_out + p.dst0[s] + t0) * D;
  const int4* ks = reinterpret_cast<const int4*>(static_cast<const T*>(p.k[s]) + src_off);
  const int4* vs = reinterpret_cast<const int4*>(static_cast<const T*>(p.v[s]) + src_off);
  int4* kd = reinterpret_cast<int4*>(out_k + dst_off);
  int4* vd = reinterpret_cast<int4*>(out_v + dst_off);
  const int nvec = rows * D / VEC;  // 16-byte vectors per tile, for K and for V
  const int tid = threadIdx.x;

  if (delta == 0) {
    // Zero shift: K is returned unchanged by the reference (blend.py:32-33); copy both.
#pragma unroll 1
    for (int base = tid; base < nvec; base += 4 * kThreads) {
      int4 a[4], b[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int w = base + u * kThreads;
        if (w < nvec) {
          a[u] = ld_stream(ks + w);
          b[u] = ld_stream(vs + w);
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int w = base + u * kThreads;
        if (w < nvec) {
          st_stream(kd + w, a[u]);
          st_stream(vd + w, b[u]);
        }
      }
    }
    return;
  }

  for (int i = tid; i < half; i += kThreads) {
    const float a = __fmul_rn((float)delta, p.inv_freq[i]);
    float sn, cs;
    sincosf(a, &sn, &cs);
    s_cos[i] = __fdiv_rn(__fmul_rn(cs, scale), scale);
    s_sin[i] = __fdiv_rn(__fmul_rn(sn, scale), scale);
  }
  __syncthreads();

  // Slots: one slot = VEC rotation pairs (i, i + D/2) of one row. Slots per row (spr) is a
  // power of two dividing kThreads, so a thread's column group is fixed: tid % spr.
  const int spr = half / VEC;
  const int vpr = D / VEC;  // vectors per row
  const int col = (tid & (spr - 1)) * VEC;
  float c[VEC], sn[VEC];
#pragma unroll
  for (int j = 0; j < VEC; ++j) {
    c[j] = s_cos[col + j];
    sn[j] = s_sin[col + j];
  }
  const int nslot = nvec >> 1;
  // Per iteration a thread moves 2 K slots (4 vectors) and 4 V vectors, all loads first.
#pragma unroll 1
  for (int it = 0; it * 2 * kThreads < nslot; ++it) {
    int4 a[2], b[2], v[4];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int q = tid + (it * 2 + u) * kThreads;
      if (q < nslot) {
        const int r = q / spr;
        const int off = r * vpr + (q & (spr - 1));
        a[u] = ld_stream(ks + off);
        b[u] = ld_stream(ks + off + spr);
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int w = tid + (it * 4 + u) * kThreads;
      if (w < nvec) v[u] = ld_stream(vs + w);
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int q = tid + (it * 2 + u) * kThreads;
      if (q < nslot) {
        const int r = q / spr;
        const int off = r * vpr + (q & (spr - 1));
        st_stream(kd + off, rot_first<T>(a[u], b[u], c, sn));
        st_stream(kd + off + spr, rot_second<T>(a[u], b[u], c, sn));
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int w = tid + (it * 4 + u) * kThreads;
      if (w < nvec) st_stream(vd + w, v[u]);
    }
  }
}

template <typename T>
int launch_rope(const RopeTable& tab, int nseg, int tiles, void* out_k, void* out_v, int D,
                long long T_out, float scale, cudaStream_t stream) {
  rope_gather_append_kernel<T><<<tiles, kThreads, 0, stream>>>(
      tab, nseg, static_cast<T*>(out_k), static_cast<T*>(out_v), D, T_out, scale);
  TREAD_CHECK_LAUNCH("rope_gather_append_kernel");
  return TREAD_OK;
}

}  // namespace
}  // namespace tread

extern "C" int tread_rope_gather_append(const void* const* k_src, const void* const* v_src,
                                        const int32_t* n_tok, const int64_t* delta,
                                        const int64_t* dst_tok0, int nseg, void* out_k,
                                        void* out_v, int L, int Hkv, int D, int64_t T_out,
                                        const float* inv_freq, float attn_scaling, int dtype,
                                        tread_stream_t stream) {
  using namespace tread;
  TREAD_CHECK_ARG(nseg >= 0, "rope_gather_append: nseg=%d < 0", nseg);
  if (nseg == 0) return TREAD_OK;
  TREAD_CHECK_ARG(k_src && v_src && n_tok && delta && dst_tok0, "rope_gather_append: null host array");
  TREAD_CHECK_ARG(out_k && out_v, "rope_gather_append: null output");
  TREAD_CHECK_ARG(L > 0 && Hkv > 0 && T_out >= 0, "rope_gather_append: bad L=%d Hkv=%d T_out=%lld", L, Hkv,
                  (long long)T_out);
  const size_t es = dtype_size(dtype);
  TREAD_CHECK_ARG(es != 0, "rope_gather_append: unknown dtype %d", dtype);
  const int vec = (int)(16 / es);
  const int spr = D / 2 / vec;
  TREAD_CHECK_ARG(D >= 2 * vec && D <= 2 * kMaxHalf && D % (2 * vec) == 0 && (spr & (spr - 1)) == 0,
                  "rope_gather_append: head_dim %d unsupported for dtype %d (need D/2 = power-of-two "
                  "multiple of %d, D <= %d)",
                  D, dtype, vec, 2 * kMaxHalf);
  TREAD_CHECK_ARG(aligned16(out_k) && aligned16(out_v), "rope_gather_append: outputs not 16-byte aligned");
  TREAD_CHECK_ARG(isfinite(attn_scaling) && attn_scaling != 0.f, "rope_gather_append: bad attn_scaling");
  const long long LH = (long long)L * Hkv;
  TREAD_CHECK_ARG(LH < (1LL << 24), "rope_gather_append: L*Hkv too large");

  bool any_rot = false;
  for (int j = 0; j < nseg; ++j) {
    TREAD_CHECK_ARG(n_tok[j] >= 0, "rope_gather_append: n_tok[%d]=%d < 0", j, n_tok[j]);
    if (n_tok[j] == 0) continue;
    TREAD_CHECK_ARG(k_src[j] && v_src[j] && aligned16(k_src[j]) && aligned16(v_src[j]),
                    "rope_gather_append: segment %d source null or not 16-byte aligned", j);
    TREAD_CHECK_ARG(dst_tok0[j] >= 0 && dst_tok0[j] + n_tok[j] <= T_out,
                    "rope_gather_append: segment %d rows [%lld, %lld) outside T_out=%lld", j,
                    (long long)dst_tok0[j], (long long)(dst_tok0[j] + n_tok[j]), (long long)T_out);
    TREAD_CHECK_ARG(delta[j] > -(1LL << 24) && delta[j] < (1LL << 24),
                    "rope_gather_append: |delta[%d]|=%lld >= 2^24", j, (long long)delta[j]);
    any_rot |= delta[j] != 0;
  }
  TREAD_CHECK_ARG(!any_rot || inv_freq, "rope_gather_append: inv_freq is null");

  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  RopeTable tab;
  if (inv_freq)
    for (int i = 0; i < D / 2; ++i) tab.inv_freq[i] = inv_freq[i];
  else
    for (int i = 0; i < D / 2; ++i) tab.inv_freq[i] = 0.f;
  int j = 0;
  while (j < nseg) {
    int m = 0;
    long long tiles = 0;
    while (j < nseg && m < kMaxSeg && tiles < (1LL << 30)) {
      if (n_tok[j] > 0) {
        const long long seg_tiles = LH * ((n_tok[j] + kTileTok - 1) / kTileTok);
        TREAD_CHECK_ARG(seg_tiles < (1LL << 30), "rope_gather_append: segment %d too large", j);
        tab.k[m] = k_src[j];
        tab.v[m] = v_src[j];
        tab.dst0[m] = dst_tok0[j];
        tab.n[m] = n_tok[j];
        tab.delta[m] = (int)delta[j];
        tab.tile0[m] = (int)tiles;
        tiles += seg_tiles;
        ++m;
      }
      ++j;
    }
    if (m == 0) break;
    tab.tile0[m] = (int)tiles;
    int rc;
    switch (dtype) {
      case TREAD_BF16:
        rc = launch_rope<__nv_bfloat16>(tab, m, (int)tiles, out_k, out_v, D, T_out, attn_scaling, st);
        break;
      case TREAD_F16:
        rc = launch_rope<__half>(tab, m, (int)tiles, out_k, out_v, D, T_out, attn_scaling, st);
        break;
      default:
        rc = launch_rope<float>(tab, m, (int)tiles, out_k, out_v, D, T_out, attn_scaling, st);
        break;
    }
    if (rc != TREAD_OK) return rc;
  }
  return TREAD_OK;
}
