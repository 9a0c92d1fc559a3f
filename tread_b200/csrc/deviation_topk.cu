// Fused layer-1 KV deviation + deterministic top-k selection (sm_100a).
//
// Replaces tread/blend.py:129 (dev = Σ_h‖k1−K1[S]‖₂ + Σ_h‖v1−V1[S]‖₂, a chain of sub / norm /
// sum kernels over gathered copies), :145/:160 (budget, torch.topk) and :165 (sort) with one
// launch:
//   phase 1  one warp per candidate reads the fresh and cached layer-1 rows of every KV head
//            straight from their tensors (the cache rows gathered by position, no copy) and
//            writes dev in fp32 with a fixed summation order (below);
//   phase 2  the last CTA to finish (an atomic ticket in `workspace`) selects the `budget`
//            largest dev values with an MSB-first radix select on order-preserving uint32 keys,
//            breaks ties toward the lower candidate index, and compacts the selection in
//            ascending index order. That is the set `S = sort(all_c[topk(dev, budget)])`.
//
// Fixed fp32 order (restated exactly by the CPU oracle, so selections compare bit-for-bit):
//   lane l of the warp owns elements [l*E, (l+1)*E) of a D-row (E = D/32) and accumulates
//   fl(p + fl(d*d)) in element order, d = fl(fresh - cached); lanes then combine by an xor
//   butterfly with offsets 16, 8, 4, 2, 1; norm = sqrt (IEEE); per token
//   a = (((n_k0 + n_k1) + n_k2) + ...), b likewise over V heads, dev = a + b.
#include <algorithm>

#include "common.cuh"

namespace tread {
namespace {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;

template <typename T, int E>
__device__ __forceinline__ void load_row(const T* p, float (&x)[E]) {
  if constexpr (E * sizeof(T) == 16) {
    Vec16<T> v;
    v.raw = __ldg(reinterpret_cast<const int4*>(p));
#pragma unroll
    for (int e = 0; e < E; ++e) x[e] = Num<T>::to_f(v.e[e]);
  } else if constexpr (E * sizeof(T) == 8) {
    union {
      uint2 raw;
      T e[E];
    } v;
    v.raw = __ldg(reinterpret_cast<const uint2*>(p));
#pragma unroll
    for (int e = 0; e < E; ++e) x[e] = Num<T>::to_f(v.e[e]);
  } else {
#pragma unroll
    for (int e = 0; e < E; ++e) x[e] = Num<T>::to_f(p[e]);
  }
}

// A lane's E elements of a row, kept as the loaded bytes until they are used: rows of several
// heads can then be in flight at once within the register budget (bf16 E = 4: 2 registers).
template <typename T, int E>
struct RawRow {
  static constexpr int kWords = (E * (int)sizeof(T) + 3) / 4;
  uint32_t w[kWords];
  __device__ __forceinline__ void load(const T* p) {
    if constexpr (kWords == 4) {
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(p));
      w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
    } else if constexpr (kWords == 2) {
      const uint2 v = __ldg(reinterpret_cast<const uint2*>(p));
      w[0] = v.x; w[1] = v.y;
    } else if constexpr (kWords == 1) {
      w[0] = __ldg(reinterpret_cast<const unsigned*>(p));
    } else {
#pragma unroll
      for (int i = 0; i < kWords; ++i) w[i] = __ldg(reinterpret_cast<const unsigned*>(p) + i);
    }
  }
  __device__ __forceinline__ void to_float(float (&x)[E]) const {
    const T* e = reinterpret_cast<const T*>(w);
#pragma unroll
    for (int i = 0; i < E; ++i) x[i] = Num<T>::to_f(e[i]);
  }
};

template <int E>
__device__ __forceinline__ float row_norm(const float (&a)[E], const float (&b)[E]) {
  float p = 0.f;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const float d = __fsub_rn(a[e], b[e]);
    p = __fadd_rn(p, __fmul_rn(d, d));
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) p = __fadd_rn(p, __shfl_xor_sync(0xffffffffu, p, off));
  return __fsqrt_rn(p);
}

// Order-preserving uint32 image of an fp32 value; every NaN maps to the top key (torch.topk
// ranks NaN above +inf).
__device__ __forceinline__ unsigned order_key(float f) {
  const unsigned u = __float_as_uint(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return 0xffffffffu;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Exclusive block-wide prefix sum of one value per thread; `total` receives the block sum.
__device__ __forceinline__ unsigned block_exclusive_sum(unsigned v, unsigned* s_scan, unsigned& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned incl = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const unsigned o = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += o;
  }
  if (lane == 31) s_scan[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const unsigned w = lane < kWarps ? s_scan[lane] : 0u;
    unsigned wi = w;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const unsigned o = __shfl_up_sync(0xffffffffu, wi, off);
      if (lane >= off) wi += o;
    }
    if (lane < kWarps) s_scan[lane] = wi - w;
    if (lane == kWarps - 1) s_scan[kWarps] = wi;
  }
  __syncthreads();
  const unsigned r = s_scan[warp] + incl - v;
  total = s_scan[kWarps];
  __syncthreads();
  return r;
}

// Adds 1 to hist[bin] for every lane with `act`; lanes that share a bin add once, together
// (the top digits of nearby fp32 values coincide, so per-lane atomics would serialise on one
// bin). All 32 lanes of the warp must call it.
__device__ __forceinline__ void hist_add(unsigned* hist, bool act, unsigned bin) {
  const unsigned b = act ? bin : 0x100u;
  const unsigned peers = __match_any_sync(0xffffffffu, b);
  if (act && (threadIdx.x & 31) == (unsigned)(__ffs(peers) - 1)) atomicAdd(&hist[bin], (unsigned)__popc(peers));
}

constexpr int kKeyCache = 16;  // keys per thread kept in registers when n <= kThreads * kKeyCache

// Top-`budget` of dev[0..n) (largest first, lower index wins ties), written ascending by index.
// Thread t owns the contiguous index chunk [t*C, (t+1)*C). With C <= kKeyCache the thread's keys
// stay in registers and the threshold key is found by narrowing a value interval (below); larger
// inputs re-read their keys from L2 each pass and run an MSB-first radix select over 8-bit digits
// (warp-aggregated histogram). Either way a suffix scan over 256 bins by threads 0..255 picks the
// bucket each pass, then one pass of per-chunk counts and two block scans place every selected
// index.
template <bool CACHED>
__device__ void select_topk_impl(const float* __restrict__ dev, int n, int budget,
                                 const int64_t* __restrict__ cand_pos, int64_t* __restrict__ sel_idx,
                                 int64_t* __restrict__ sel_pos) {
  __shared__ unsigned hist[256];
  __shared__ unsigned s_scan[kWarps + 1];
  __shared__ unsigned s_digit, s_rem;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int C = (n + kThreads - 1) / kThreads;
  const int lo = min(n, tid * C), hi = min(n, lo + C);
  constexpr int KC = CACHED ? kKeyCache : 1;
  unsigned kc[KC];
  if constexpr (CACHED) {
#pragma unroll
    for (int k = 0; k < KC; ++k) kc[k] = (k < C && lo + k < hi) ? order_key(__ldcg(dev + lo + k)) : 0u;
  }
  auto key_at = [&](int k) -> unsigned {
    if constexpr (CACHED) {
      return kc[k];
    } else {
      return order_key(__ldcg(dev + lo + k));
    }
  };
  unsigned prefix = 0u, remaining = (unsigned)budget;
  if constexpr (CACHED) {
    // Narrow a key interval [L, U] that holds the budget-th largest key: bucket the keys inside it
    // into 256 equal-width buckets, keep the bucket that holds it, until L == U. Buckets of the
    // values' own range spread even nearly equal floats (fixed 8-bit digits would put them all in
    // one bin), so per-lane shared atomics rarely collide; at most 4 passes.
    __shared__ unsigned s_min[kWarps], s_max[kWarps];
    unsigned kmin = 0xffffffffu, kmax = 0u;
#pragma unroll
    for (int k = 0; k < KC; ++k)
      if (lo + k < hi) {
        kmin = min(kmin, kc[k]);
        kmax = max(kmax, kc[k]);
      }
    kmin = __reduce_min_sync(0xffffffffu, kmin);
    kmax = __reduce_max_sync(0xffffffffu, kmax);
    if (lane == 0) {
      s_min[warp] = kmin;
      s_max[warp] = kmax;
    }
    __syncthreads();
    unsigned L = 0xffffffffu, U = 0u;
#pragma unroll 1
    for (int w = 0; w < kWarps; ++w) {
      L = min(L, s_min[w]);
      U = max(U, s_max[w]);
    }
    while (L < U) {
      const unsigned span = U - L;
      const int bits = 32 - __clz(span);
      const int shift = bits > 8 ? bits - 8 : 0;  // (U - L) >> shift < 256
      if (tid < 256) hist[tid] = 0u;
      __syncthreads();
#pragma unroll
      for (int k = 0; k < KC; ++k)
        if (lo + k < hi && kc[k] >= L && kc[k] <= U) atomicAdd(&hist[(kc[k] - L) >> shift], 1u);
      __syncthreads();
      unsigned c = 0u, incl = 0u;
      if (tid < 256) {  // thread j takes bucket 255 - j: its inclusive prefix counts keys in buckets >= it
        c = hist[255 - tid];
        incl = c;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
          const unsigned o = __shfl_up_sync(0xffffffffu, incl, off);
          if (lane >= off) incl += o;
        }
        if (lane == 31) s_scan[warp] = incl;
      }
      __syncthreads();
      if (tid < 256) {
        for (int w = 0; w < warp; ++w) incl += s_scan[w];
        const unsigned above = incl - c;
        if (above < remaining && incl >= remaining) {
          s_digit = 255u - (unsigned)tid;
          s_rem = remaining - above;
        }
      }
      __syncthreads();
      const unsigned b = s_digit;
      remaining = s_rem;
      const unsigned nl = L + (b << shift);
      const unsigned top = nl + ((1u << shift) - 1u);
      U = top < nl ? U : min(U, top);  // (no wrap: nl + width - 1 stays below 2^32 within [L, U])
      L = nl;
      __syncthreads();
    }
    prefix = L;
  } else {
    unsigned mask = 0u;
#pragma unroll 1
    for (int shift = 24; shift >= 0; shift -= 8) {
      if (tid < 256) hist[tid] = 0u;
      __syncthreads();
      for (int k = 0; k < C; ++k) {
        const bool valid = lo + k < hi;
        const unsigned key = valid ? key_at(k) : 0u;
        hist_add(hist, valid && (key & mask) == prefix, (key >> shift) & 255u);
      }
      __syncthreads();
      // thread j < 256 handles bin 255 - j: its inclusive prefix over j is the count of keys whose
      // digit is >= that bin
      unsigned c = 0u, incl = 0u;
      if (tid < 256) {
        c = hist[255 - tid];
        incl = c;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
          const unsigned o = __shfl_up_sync(0xffffffffu, incl, off);
          if (lane >= off) incl += o;
        }
        if (lane == 31) s_scan[warp] = incl;
      }
      __syncthreads();
      if (tid < 256) {
        for (int w = 0; w < warp; ++w) incl += s_scan[w];
        const unsigned above = incl - c;
        if (above < remaining && incl >= remaining) {
          s_digit = 255u - (unsigned)tid;
          s_rem = remaining - above;
        }
      }
      __syncthreads();
      prefix |= s_digit << shift;
      mask |= 255u << shift;
      remaining = s_rem;
      __syncthreads();
    }
  }
  // prefix is the key of the budget-th largest value; `remaining` of its ties are taken, lowest
  // indices first.
  unsigned gt = 0u, eq = 0u;
  auto count = [&](int k) {
    const unsigned key = key_at(k);
    gt += key > prefix;
    eq += key == prefix;
  };
  if constexpr (CACHED) {
#pragma unroll
    for (int k = 0; k < KC; ++k)
      if (lo + k < hi) count(k);
  } else {
    for (int k = 0; lo + k < hi; ++k) count(k);
  }
  unsigned tot;
  const unsigned eq_before = block_exclusive_sum(eq, s_scan, tot);
  const unsigned take_eq = eq_before >= remaining ? 0u : min(eq, remaining - eq_before);
  unsigned r = block_exclusive_sum(gt + take_eq, s_scan, tot);
  unsigned taken = 0u;
  if constexpr (CACHED) {
    // selection as a bit mask first, then the writes: every cand_pos load can be in flight at once
    unsigned selm = 0u;
#pragma unroll
    for (int k = 0; k < KC; ++k) {
      if (lo + k < hi) {
        const unsigned key = kc[k];
        bool sel = key > prefix;
        if (key == prefix && taken < take_eq) {
          sel = true;
          ++taken;
        }
        selm |= (sel ? 1u : 0u) << k;
      }
    }
#pragma unroll
    for (int k = 0; k < KC; ++k)
      if ((selm >> k) & 1u) sel_idx[r + __popc(selm & ((1u << k) - 1u))] = lo + k;
    if (sel_pos) {
      int64_t cp[KC];
#pragma unroll
      for (int k = 0; k < KC; ++k) cp[k] = ((selm >> k) & 1u) ? __ldg(cand_pos + lo + k) : 0;
#pragma unroll
      for (int k = 0; k < KC; ++k)
        if ((selm >> k) & 1u) sel_pos[r + __popc(selm & ((1u << k) - 1u))] = cp[k];
    }
    return;
  }
  auto place = [&](int k) {
    const unsigned key = key_at(k);
    bool sel = key > prefix;
    if (key == prefix && taken < take_eq) {
      sel = true;
      ++taken;
    }
    if (sel) {
      const int i = lo + k;
      sel_idx[r] = i;
      if (sel_pos) sel_pos[r] = cand_pos[i];
      ++r;
    }
  };
  for (int k = 0; lo + k < hi; ++k) place(k);
}

__device__ void select_topk(const float* dev, int n, int budget, const int64_t* cand_pos, int64_t* sel_idx,
                            int64_t* sel_pos) {
  if (n <= kThreads * kKeyCache)
    select_topk_impl<true>(dev, n, budget, cand_pos, sel_idx, sel_pos);
  else
    select_topk_impl<false>(dev, n, budget, cand_pos, sel_idx, sel_pos);
}

template <typename T, int E>
__global__ void __launch_bounds__(kThreads, 2)
    deviation_topk_kernel(const T* __restrict__ k1, const T* __restrict__ v1, long long f_st, long long f_sh,
                          const T* __restrict__ K1, const T* __restrict__ V1, long long c_st, long long c_sh,
                          long long T_cache, const int64_t* __restrict__ cand_pos, int n, int H, int budget,
                          float* __restrict__ dev_out, int64_t* __restrict__ sel_idx, int64_t* __restrict__ sel_pos,
                          unsigned* __restrict__ workspace) {
  const int lane = threadIdx.x & 31;
  const int stride = gridDim.x * kWarps;
  int t = blockIdx.x * kWarps + (threadIdx.x >> 5);
  long long pos = t < n ? cand_pos[t] : 0;
  for (; t < n; t += stride) {
    // the next candidate's position loads while this one's rows do
    const long long pos_next = t + stride < n ? cand_pos[t + stride] : 0;
    float dev;
    if (pos < 0 || pos >= T_cache) {
      if (lane == 0) atomicOr(workspace + 1, 1u);  // sticky error flag for the caller
      dev = __int_as_float(0x7fc00000);
    } else {
      float a = 0.f, b = 0.f;
      // heads whose rows are in flight together (raw bytes: 8 x HU registers for bf16 D = 128)
      constexpr int HU = RawRow<T, E>::kWords <= 2 ? 4 : (RawRow<T, E>::kWords <= 4 ? 2 : 1);
#pragma unroll 1
      for (int h0 = 0; h0 < H; h0 += HU) {
        RawRow<T, E> fk[HU], ck[HU], fv[HU], cv[HU];
#pragma unroll
        for (int j = 0; j < HU; ++j) {
          if (h0 + j < H) {
            const long long fo = (long long)t * f_st + (long long)(h0 + j) * f_sh + lane * E;
            const long long co = pos * c_st + (long long)(h0 + j) * c_sh + lane * E;
            fk[j].load(k1 + fo);
            ck[j].load(K1 + co);
            fv[j].load(v1 + fo);
            cv[j].load(V1 + co);
          }
        }
#pragma unroll
        for (int j = 0; j < HU; ++j) {
          if (h0 + j < H) {
            float x[E], y[E];
            fk[j].to_float(x);
            ck[j].to_float(y);
            a = __fadd_rn(a, row_norm<E>(x, y));
            fv[j].to_float(x);
            cv[j].to_float(y);
            b = __fadd_rn(b, row_norm<E>(x, y));
          }
        }
      }
      dev = __fadd_rn(a, b);
    }
    if (lane == 0) dev_out[t] = dev;
    pos = pos_next;
  }
  if (budget <= 0) return;
  __shared__ bool s_last;
  if (lane == 0) __threadfence();  // this warp's dev writes, before the CTA's ticket
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(workspace, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  select_topk(dev_out, n, budget, cand_pos, sel_idx, sel_pos);
  if (threadIdx.x == 0) workspace[0] = 0u;  // ready for the next call
}

// Resident CTAs of the deviation kernel on the current device (2 per SM by its launch bounds).
int resident_ctas() {
  static int cache[128] = {0};
  int d = 0;
  if (cudaGetDevice(&d) != cudaSuccess || d < 0 || d >= 128) return 296;
  if (!cache[d]) {
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, d) != cudaSuccess || sms <= 0) sms = 148;
    cache[d] = 2 * sms;
  }
  return cache[d];
}

template <typename T, int E>
int launch_dev(const void* k1, const void* v1, long long f_st, long long f_sh, const void* K1, const void* V1,
               long long c_st, long long c_sh, long long T_cache, const int64_t* cand_pos, int n, int H, int budget,
               float* dev_out, int64_t* sel_idx, int64_t* sel_pos, unsigned* ws, cudaStream_t st) {
  // one wave: every warp loops over candidates, no partly filled second wave
  const int grid = std::min((n + kWarps - 1) / kWarps, resident_ctas());
  deviation_topk_kernel<T, E><<<grid, kThreads, 0, st>>>(
      static_cast<const T*>(k1), static_cast<const T*>(v1), f_st, f_sh, static_cast<const T*>(K1),
      static_cast<const T*>(V1), c_st, c_sh, T_cache, cand_pos, n, H, budget, dev_out, sel_idx, sel_pos, ws);
  TREAD_CHECK_LAUNCH("deviation_topk_kernel");
  return TREAD_OK;
}

template <typename T>
int dispatch_e(int D, const void* k1, const void* v1, long long f_st, long long f_sh, const void* K1,
               const void* V1, long long c_st, long long c_sh, long long T_cache, const int64_t* cand_pos, int n,
               int H, int budget, float* dev_out, int64_t* sel_idx, int64_t* sel_pos, unsigned* ws, cudaStream_t st) {
  switch (D) {
    case 64:
      return launch_dev<T, 2>(k1, v1, f_st, f_sh, K1, V1, c_st, c_sh, T_cache, cand_pos, n, H, budget, dev_out,
                              sel_idx, sel_pos, ws, st);
    case 128:
      return launch_dev<T, 4>(k1, v1, f_st, f_sh, K1, V1, c_st, c_sh, T_cache, cand_pos, n, H, budget, dev_out,
                              sel_idx, sel_pos, ws, st);
    default:
      return launch_dev<T, 8>(k1, v1, f_st, f_sh, K1, V1, c_st, c_sh, T_cache, cand_pos, n, H, budget, dev_out,
                              sel_idx, sel_pos, ws, st);
  }
}

}  // namespace
}  // namespace tread

extern "C" int tread_deviation_topk(const void* k1, const void* v1, int64_t fresh_stride_tok,
                                    int64_t fresh_stride_head, const void* K1, const void* V1,
                                    int64_t cache_stride_tok, int64_t cache_stride_head, int64_t T_cache,
                                    const int64_t* cand_pos, int n, int Hkv, int D, int budget, int dtype,
                                    float* dev_out, int64_t* sel_idx, int64_t* sel_pos, void* workspace,
                                    tread_stream_t stream) {
  using namespace tread;
  TREAD_CHECK_ARG(n >= 0 && budget >= 0 && budget <= n, "deviation_topk: need 0 <= budget (%d) <= n (%d)", budget,
                  n);
  if (n == 0) return TREAD_OK;
  TREAD_CHECK_ARG(k1 && v1 && K1 && V1 && cand_pos && dev_out && workspace, "deviation_topk: null pointer");
  TREAD_CHECK_ARG(budget == 0 || sel_idx, "deviation_topk: sel_idx is null");
  TREAD_CHECK_ARG(Hkv > 0 && (D == 64 || D == 128 || D == 256), "deviation_topk: need Hkv > 0 and D in {64,128,256}");
  const size_t es = dtype_size(dtype);
  TREAD_CHECK_ARG(es != 0, "deviation_topk: unknown dtype %d", dtype);
  const int E = D / 32;
  const size_t vec_bytes = E * es;
  auto al = [&](const void* p) { return (reinterpret_cast<uintptr_t>(p) % vec_bytes) == 0; };
  TREAD_CHECK_ARG(al(k1) && al(v1) && al(K1) && al(V1), "deviation_topk: row pointers not %zu-byte aligned",
                  vec_bytes);
  TREAD_CHECK_ARG(fresh_stride_tok % E == 0 && fresh_stride_head % E == 0 && cache_stride_tok % E == 0 &&
                      cache_stride_head % E == 0,
                  "deviation_topk: strides must be multiples of D/32");
  TREAD_CHECK_ARG(T_cache > 0, "deviation_topk: T_cache must be > 0");
  TREAD_CHECK_ARG((reinterpret_cast<uintptr_t>(workspace) & 15u) == 0, "deviation_topk: workspace not aligned");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  unsigned* ws = static_cast<unsigned*>(workspace);
  switch (dtype) {
    case TREAD_BF16:
      return dispatch_e<__nv_bfloat16>(D, k1, v1, fresh_stride_tok, fresh_stride_head, K1, V1, cache_stride_tok,
                                       cache_stride_head, T_cache, cand_pos, n, Hkv, budget, dev_out, sel_idx,
                                       sel_pos, ws, st);
    case TREAD_F16:
      return dispatch_e<__half>(D, k1, v1, fresh_stride_tok, fresh_stride_head, K1, V1, cache_stride_tok,
                                cache_stride_head, T_cache, cand_pos, n, Hkv, budget, dev_out, sel_idx, sel_pos, ws,
                                st);
    default:
      return dispatch_e<float>(D, k1, v1, fresh_stride_tok, fresh_stride_head, K1, V1, cache_stride_tok,
                               cache_stride_head, T_cache, cand_pos, n, Hkv, budget, dev_out, sel_idx, sel_pos, ws,
                               st);
  }
}

// ---- tensor-parallel split: per-head norms on each rank, selection on the gathered norms ------------
//
// Under KV-head tensor parallelism each rank holds a contiguous slice of the KV heads. A rank
// writes the per-head norms of its slice (the phase-1 values before the head sums); after an
// all-gather every rank holds all heads' norms, sums them in global head order exactly as the
// fused kernel does (a = ((n_k0 + n_k1) + ...), b likewise, dev = a + b) and runs the same
// selection, so every rank selects the same tokens and a single-rank run selects the same set.

namespace tread {
namespace {

template <typename T, int E>
__global__ void __launch_bounds__(kThreads)
    head_norms_kernel(const T* __restrict__ k1, const T* __restrict__ v1, long long f_st, long long f_sh,
                      const T* __restrict__ K1, const T* __restrict__ V1, long long c_st, long long c_sh,
                      long long T_cache, const int64_t* __restrict__ cand_pos, int n, int H,
                      float* __restrict__ norms, unsigned* __restrict__ workspace) {
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (t >= n) return;
  const long long pos = cand_pos[t];
  if (pos < 0 || pos >= T_cache) {
    if (lane == 0) atomicOr(workspace + 1, 1u);
    if (lane < H) {
      norms[(long long)lane * n + t] = __int_as_float(0x7fc00000);
      norms[(long long)(H + lane) * n + t] = __int_as_float(0x7fc00000);
    }
    return;
  }
#pragma unroll 1
  for (int h = 0; h < H; ++h) {
    float fk[E], ck[E], fv[E], cv[E];
    const long long fo = (long long)t * f_st + (long long)h * f_sh + lane * E;
    const long long co = pos * c_st + (long long)h * c_sh + lane * E;
    load_row<T, E>(k1 + fo, fk);
    load_row<T, E>(K1 + co, ck);
    load_row<T, E>(v1 + fo, fv);
    load_row<T, E>(V1 + co, cv);
    const float nk = row_norm<E>(fk, ck);
    const float nv = row_norm<E>(fv, cv);
    if (lane == 0) {
      norms[(long long)h * n + t] = nk;
      norms[(long long)(H + h) * n + t] = nv;
    }
  }
}

// norms: [2][H][n] fp32 (K heads, then V heads, in global head order).
__global__ void __launch_bounds__(kThreads)
    select_head_norms_kernel(const float* __restrict__ norms, int n, int H, int budget,
                             const int64_t* __restrict__ cand_pos, float* __restrict__ dev_out,
                             int64_t* __restrict__ sel_idx, int64_t* __restrict__ sel_pos,
                             unsigned* __restrict__ workspace) {
  for (int t = blockIdx.x * kThreads + threadIdx.x; t < n; t += gridDim.x * kThreads) {
    float a = 0.f, b = 0.f;
    for (int h = 0; h < H; ++h) a = __fadd_rn(a, norms[(long long)h * n + t]);
    for (int h = 0; h < H; ++h) b = __fadd_rn(b, norms[(long long)(H + h) * n + t]);
    dev_out[t] = __fadd_rn(a, b);
  }
  if (budget <= 0) return;
  __shared__ bool s_last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(workspace, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  select_topk(dev_out, n, budget, cand_pos, sel_idx, sel_pos);
  if (threadIdx.x == 0) workspace[0] = 0u;
}

template <typename T>
int launch_head_norms(int D, const void* k1, const void* v1, long long f_st, long long f_sh, const void* K1,
                      const void* V1, long long c_st, long long c_sh, long long T_cache, const int64_t* cand_pos,
                      int n, int H, float* norms, unsigned* ws, cudaStream_t st) {
  const int grid = (n + kWarps - 1) / kWarps;
#define TREAD_HN(E_)                                                                                              \
  head_norms_kernel<T, E_><<<grid, kThreads, 0, st>>>(static_cast<const T*>(k1), static_cast<const T*>(v1), f_st, \
                                                      f_sh, static_cast<const T*>(K1), static_cast<const T*>(V1),  \
                                                      c_st, c_sh, T_cache, cand_pos, n, H, norms, ws)
  switch (D) {
    case 64: TREAD_HN(2); break;
    case 128: TREAD_HN(4); break;
    default: TREAD_HN(8); break;
  }
#undef TREAD_HN
  TREAD_CHECK_LAUNCH("head_norms_kernel");
  return TREAD_OK;
}

}  // namespace
}  // namespace tread

extern "C" int tread_deviation_head_norms(const void* k1, const void* v1, int64_t fresh_stride_tok,
                                          int64_t fresh_stride_head, const void* K1, const void* V1,
                                          int64_t cache_stride_tok, int64_t cache_stride_head, int64_t T_cache,
                                          const int64_t* cand_pos, int n, int Hkv, int D, int dtype,
                                          float* norms_out, void* workspace, tread_stream_t stream) {
  using namespace tread;
  TREAD_CHECK_ARG(n >= 0, "deviation_head_norms: n < 0");
  if (n == 0) return TREAD_OK;
  TREAD_CHECK_ARG(k1 && v1 && K1 && V1 && cand_pos && norms_out && workspace, "deviation_head_norms: null pointer");
  TREAD_CHECK_ARG(Hkv > 0 && Hkv <= 32 && (D == 64 || D == 128 || D == 256),
                  "deviation_head_norms: need 0 < Hkv <= 32 and D in {64,128,256}");
  const size_t es = dtype_size(dtype);
  TREAD_CHECK_ARG(es != 0, "deviation_head_norms: unknown dtype %d", dtype);
  const int E = D / 32;
  const size_t vec_bytes = E * es;
  auto al = [&](const void* p) { return (reinterpret_cast<uintptr_t>(p) % vec_bytes) == 0; };
  TREAD_CHECK_ARG(al(k1) && al(v1) && al(K1) && al(V1), "deviation_head_norms: row pointers not %zu-byte aligned",
                  vec_bytes);
  TREAD_CHECK_ARG(fresh_stride_tok % E == 0 && fresh_stride_head % E == 0 && cache_stride_tok % E == 0 &&
                      cache_stride_head % E == 0,
                  "deviation_head_norms: strides must be multiples of D/32");
  TREAD_CHECK_ARG(T_cache > 0, "deviation_head_norms: T_cache must be > 0");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  unsigned* ws = static_cast<unsigned*>(workspace);
  switch (dtype) {
    case TREAD_BF16:
      return launch_head_norms<__nv_bfloat16>(D, k1, v1, fresh_stride_tok, fresh_stride_head, K1, V1,
                                              cache_stride_tok, cache_stride_head, T_cache, cand_pos, n, Hkv,
                                              norms_out, ws, st);
    case TREAD_F16:
      return launch_head_norms<__half>(D, k1, v1, fresh_stride_tok, fresh_stride_head, K1, V1, cache_stride_tok,
                                       cache_stride_head, T_cache, cand_pos, n, Hkv, norms_out, ws, st);
    default:
      return launch_head_norms<float>(D, k1, v1, fresh_stride_tok, fresh_stride_head, K1, V1, cache_stride_tok,
                                      cache_stride_head, T_cache, cand_pos, n, Hkv, norms_out, ws, st);
  }
}

extern "C" int tread_select_head_norms(const float* norms, int n, int Hkv, int budget, const int64_t* cand_pos,
                                       float* dev_out, int64_t* sel_idx, int64_t* sel_pos, void* workspace,
                                       tread_stream_t stream) {
  using namespace tread;
  TREAD_CHECK_ARG(n >= 0 && budget >= 0 && budget <= n, "select_head_norms: need 0 <= budget (%d) <= n (%d)",
                  budget, n);
  if (n == 0) return TREAD_OK;
  TREAD_CHECK_ARG(norms && dev_out && workspace && Hkv > 0, "select_head_norms: null pointer or Hkv <= 0");
  TREAD_CHECK_ARG(budget == 0 || (sel_idx && (cand_pos || !sel_pos)), "select_head_norms: sel_idx/cand_pos null");
  TREAD_CHECK_ARG((reinterpret_cast<uintptr_t>(workspace) & 15u) == 0, "select_head_norms: workspace not aligned");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int grid = std::min((n + kThreads - 1) / kThreads, 148 * 4);
  select_head_norms_kernel<<<grid, kThreads, 0, st>>>(norms, n, Hkv, budget, cand_pos, dev_out, sel_idx, sel_pos,
                                                      static_cast<unsigned*>(workspace));
  TREAD_CHECK_LAUNCH("select_head_norms_kernel");
  return TREAD_OK;
}

// ---- allocation-free variant -------------------------------------------------------------------
//
// Some callers cannot hand this library device scratch: serving loops whose HBM is owned
// entirely by a pooling allocator reserved at start-up (a raw cudaMalloc there fails or
// fragments memory outside the pool), latency-critical loops that avoid cudaMalloc because it
// can synchronise the device, and thin FFI hosts (ctypes, cgo, JNI) that have no device
// allocator of their own. For them the selector's scratch — the CTA ticket / error words and the
// fp32 deviation of every candidate — lives in one file-scope device array instead, so the call
// allocates nothing; the caller still passes every input and output.


namespace tread {
namespace {

constexpr int kNoAllocMaxCandidates = 65536;
constexpr size_t kNoAllocTicketBytes = 256;
// 256 B of ticket/flag words + 256 KB of per-candidate deviation; every GPU that loads the
// library holds this array until the process exits.
static __device__ __align__(256) unsigned char
    g_selector_scratch[kNoAllocTicketBytes + sizeof(float) * kNoAllocMaxCandidates];

// Device address of the static scratch in the current context, looked up on every call (a host
// table lookup once the module is loaded), so that it stays right after the context is torn down
// and created again (cudaDeviceReset) and the module loads at another address.
int scratch_address(void** out) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_selector_scratch);
  if (e != cudaSuccess || p == nullptr) {
    set_error("deviation_topk_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
    return TREAD_ERR_CUDA;
  }
  *out = p;
  return TREAD_OK;
}

}  // namespace
}  // namespace tread

extern "C" int tread_deviation_topk_noalloc(const void* k1, const void* v1, int64_t fresh_stride_tok,
                                            int64_t fresh_stride_head, const void* K1, const void* V1,
                                            int64_t cache_stride_tok, int64_t cache_stride_head, int64_t T_cache,
                                            const int64_t* cand_pos, int n, int Hkv, int D, int budget, int dtype,
                                            int64_t* sel_idx, int64_t* sel_pos, unsigned* err_flag,
                                            tread_stream_t stream) {
  using namespace tread;
  TREAD_CHECK_ARG(n >= 0 && n <= kNoAllocMaxCandidates,
                  "deviation_topk_noalloc: n=%d candidates exceeds the static scratch maximum of %d", n,
                  kNoAllocMaxCandidates);
  if (n == 0) return TREAD_OK;
  void* scratch = nullptr;
  const int rc = scratch_address(&scratch);
  if (rc != TREAD_OK) return rc;
  // The array keeps the previous call's contents: the ticket and error words must start at zero.
  TREAD_CHECK_CUDA(cudaMemsetAsync(scratch, 0, kNoAllocTicketBytes, reinterpret_cast<cudaStream_t>(stream)));
  float* dev = reinterpret_cast<float*>(static_cast<unsigned char*>(scratch) + kNoAllocTicketBytes);
  const int st = tread_deviation_topk(k1, v1, fresh_stride_tok, fresh_stride_head, K1, V1, cache_stride_tok,
                                      cache_stride_head, T_cache, cand_pos, n, Hkv, D, budget, dtype, dev, sel_idx,
                                      sel_pos, scratch, stream);
  if (st != TREAD_OK || err_flag == nullptr) return st;
  // Word 1 of the scratch is this call's out-of-range flag (cleared above): hand it to the caller
  // in stream order, before a later call clears it again.
  TREAD_CHECK_CUDA(cudaMemcpyAsync(err_flag, static_cast<unsigned char*>(scratch) + sizeof(unsigned),
                                   sizeof(unsigned), cudaMemcpyDeviceToDevice,
                                   reinterpret_cast<cudaStream_t>(stream)));
  return TREAD_OK;
}
