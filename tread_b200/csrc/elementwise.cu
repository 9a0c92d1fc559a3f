// Fused row-wise pieces of the recompute layer (sm_100a): RMSNorm and SwiGLU.
//
// The reference runs HF's Qwen2RMSNorm and Qwen2MLP on the recomputed rows (tread/blend.py:105,
// 112-113), i.e. 6-8 separate elementwise kernels per norm (to fp32, pow, mean, add, rsqrt,
// mul, cast, mul) and 2 for the activation (silu, mul), each a full pass over HBM. Here each is
// one pass with the same rounding points as HF's modules:
//   rmsnorm : y = to_dtype( w * to_dtype( x * rsqrt(mean(x^2) + eps) ) )   (x in fp32)
//   silu_mul: y = to_dtype( to_dtype(silu(g)) * u ),  silu(g) = g / (1 + exp(-g)) in fp32 (for
//             16-bit types with the fast exponential and division intrinsics)
#include <algorithm>
#include <type_traits>

#include "common.cuh"

namespace tread {
namespace {

constexpr int kNormThreads = 256;

constexpr int kNormCache = 4;  // 16-byte vectors of the row a thread keeps in registers

// CACHED: the row (<= kNormThreads * kNormCache vectors) is read from memory once and kept in
// registers for the normalisation; otherwise it is read twice. Same arithmetic either way.
template <typename T, bool CACHED>
__global__ void __launch_bounds__(kNormThreads)
    rmsnorm_kernel(const T* __restrict__ x, long long ldx, const T* __restrict__ w, T* __restrict__ y,
                   long long ldy, int H, float eps) {
  constexpr int VEC = 16 / sizeof(T);
  const T* xr = x + (long long)blockIdx.x * ldx;
  T* yr = y + (long long)blockIdx.x * ldy;
  const int nvec = H / VEC;
  float ss = 0.f;
  Vec16<T> xc[CACHED ? kNormCache : 1];
  if constexpr (CACHED) {
#pragma unroll
    for (int k = 0; k < kNormCache; ++k) {
      const int i = threadIdx.x + k * kNormThreads;
      if (i < nvec) xc[k].raw = __ldg(reinterpret_cast<const int4*>(xr) + i);
    }
#pragma unroll
    for (int k = 0; k < kNormCache; ++k) {
      if (threadIdx.x + k * kNormThreads < nvec) {
#pragma unroll
        for (int e = 0; e < VEC; ++e) {
          const float f = Num<T>::to_f(xc[k].e[e]);
          ss = fmaf(f, f, ss);
        }
      }
    }
  } else {
    for (int i = threadIdx.x; i < nvec; i += kNormThreads) {
      Vec16<T> a;
      a.raw = __ldg(reinterpret_cast<const int4*>(xr) + i);
#pragma unroll
      for (int e = 0; e < VEC; ++e) {
        const float f = Num<T>::to_f(a.e[e]);
        ss = fmaf(f, f, ss);
      }
    }
  }
  __shared__ float s_red[kNormThreads / 32];
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < kNormThreads / 32 ? s_red[threadIdx.x] : 0.f;
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) t += __shfl_xor_sync(0xffffffffu, t, off);
    if (threadIdx.x == 0) s_red[0] = t;
  }
  __syncthreads();
  const float r = rsqrtf(s_red[0] / (float)H + eps);
  auto norm_store = [&](int i, const Vec16<T>& a) {
    Vec16<T> b, o;
    b.raw = __ldg(reinterpret_cast<const int4*>(w) + i);
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      const float n = Num<T>::to_f(Num<T>::from_f(Num<T>::to_f(a.e[e]) * r));
      o.e[e] = Num<T>::from_f(Num<T>::to_f(b.e[e]) * n);
    }
    reinterpret_cast<int4*>(yr)[i] = o.raw;
  };
  if constexpr (CACHED) {
#pragma unroll
    for (int k = 0; k < kNormCache; ++k) {
      const int i = threadIdx.x + k * kNormThreads;
      if (i < nvec) norm_store(i, xc[k]);
    }
  } else {
    for (int i = threadIdx.x; i < nvec; i += kNormThreads) {
      Vec16<T> a;
      a.raw = __ldg(reinterpret_cast<const int4*>(xr) + i);
      norm_store(i, a);
    }
  }
}

constexpr int kSiluThreads = 256;
constexpr int kSiluUnroll = 2;  // 16-byte vectors of gate and of up in flight per thread

// One CTA per row (no index division), kSiluUnroll vectors per thread per iteration.
template <typename T>
__global__ void __launch_bounds__(kSiluThreads)
    silu_mul_kernel(const T* __restrict__ gu, long long ld, T* __restrict__ y, long long ldy, int I) {
  constexpr int VEC = 16 / sizeof(T);
  const int vpr = I / VEC;
  const long long r = blockIdx.x;
  const int4* g = reinterpret_cast<const int4*>(gu + r * ld);
  const int4* u = reinterpret_cast<const int4*>(gu + r * ld + I);
  int4* o = reinterpret_cast<int4*>(y + r * ldy);
  for (int v0 = threadIdx.x; v0 < vpr; v0 += kSiluThreads * kSiluUnroll) {
    Vec16<T> gv[kSiluUnroll], uv[kSiluUnroll];
#pragma unroll
    for (int k = 0; k < kSiluUnroll; ++k) {
      const int v = v0 + k * kSiluThreads;
      if (v < vpr) {
        gv[k].raw = __ldg(g + v);
        uv[k].raw = __ldg(u + v);
      }
    }
#pragma unroll
    for (int k = 0; k < kSiluUnroll; ++k) {
      const int v = v0 + k * kSiluThreads;
      if (v < vpr) {
        Vec16<T> ov;
#pragma unroll
        for (int e = 0; e < VEC; ++e) {
          const float gf = Num<T>::to_f(gv[k].e[e]);
          // 16-bit outputs: the fast exponential / division differ from the exact ones by ~1e-6
          // relative, which moves the 16-bit rounding of silu(g) by at most one unit, rarely;
          // fp32 keeps the exact functions
          const float sg = std::is_same<T, float>::value ? gf / (1.f + expf(-gf))
                                                         : __fdividef(gf, 1.f + __expf(-gf));
          const float sv = Num<T>::to_f(Num<T>::from_f(sg));
          ov.e[e] = Num<T>::from_f(sv * Num<T>::to_f(uv[k].e[e]));
        }
        o[v] = ov.raw;
      }
    }
  }
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace tread

extern "C" int tread_rmsnorm(const void* x, int64_t ld_x, const void* weight, void* y, int64_t ld_y, int64_t rows,
                             int hidden, float eps, int dtype, tread_stream_t stream) {
  using namespace tread;
  if (rows == 0) return TREAD_OK;
  TREAD_CHECK_ARG(x && weight && y && rows > 0 && rows < (1LL << 31), "rmsnorm: bad pointers or rows");
  const size_t es = dtype_size(dtype);
  TREAD_CHECK_ARG(es != 0, "rmsnorm: unknown dtype %d", dtype);
  TREAD_CHECK_ARG(hidden > 0 && (hidden * es) % 16 == 0 && ld_x >= hidden && ld_y >= hidden &&
                      (ld_x * es) % 16 == 0 && (ld_y * es) % 16 == 0,
                  "rmsnorm: hidden/ld must be multiples of 16 bytes");
  TREAD_CHECK_ARG(al16(x) && al16(weight) && al16(y), "rmsnorm: pointers not 16-byte aligned");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const unsigned grid = (unsigned)rows;
  const bool cached = (long long)hidden * (long long)es / 16 <= (long long)kNormThreads * kNormCache;
  auto launch = [&](auto tag) {
    using T = decltype(tag);
    const T* xp = static_cast<const T*>(x);
    const T* wp = static_cast<const T*>(weight);
    T* yp = static_cast<T*>(y);
    if (cached)
      rmsnorm_kernel<T, true><<<grid, kNormThreads, 0, st>>>(xp, ld_x, wp, yp, ld_y, hidden, eps);
    else
      rmsnorm_kernel<T, false><<<grid, kNormThreads, 0, st>>>(xp, ld_x, wp, yp, ld_y, hidden, eps);
  };
  switch (dtype) {
    case TREAD_BF16:
      launch(__nv_bfloat16());
      break;
    case TREAD_F16:
      launch(__half());
      break;
    default:
      launch(float());
      break;
  }
  TREAD_CHECK_LAUNCH("rmsnorm_kernel");
  return TREAD_OK;
}

extern "C" int tread_silu_mul(const void* gate_up, int64_t ld_gu, void* y, int64_t ld_y, int64_t rows, int inter,
                              int dtype, tread_stream_t stream) {
  using namespace tread;
  if (rows == 0) return TREAD_OK;
  TREAD_CHECK_ARG(gate_up && y && rows > 0, "silu_mul: bad pointers or rows");
  const size_t es = dtype_size(dtype);
  TREAD_CHECK_ARG(es != 0, "silu_mul: unknown dtype %d", dtype);
  TREAD_CHECK_ARG(inter > 0 && (inter * es) % 16 == 0 && ld_gu >= 2LL * inter && ld_y >= inter &&
                      (ld_gu * es) % 16 == 0 && (ld_y * es) % 16 == 0,
                  "silu_mul: inter/ld must be multiples of 16 bytes");
  TREAD_CHECK_ARG(al16(gate_up) && al16(y), "silu_mul: pointers not 16-byte aligned");
  TREAD_CHECK_ARG(rows < (1LL << 31), "silu_mul: rows >= 2^31");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const unsigned grid = (unsigned)rows;
  switch (dtype) {
    case TREAD_BF16:
      silu_mul_kernel<__nv_bfloat16><<<grid, kSiluThreads, 0, st>>>(
          static_cast<const __nv_bfloat16*>(gate_up), ld_gu, static_cast<__nv_bfloat16*>(y), ld_y, inter);
      break;
    case TREAD_F16:
      silu_mul_kernel<__half><<<grid, kSiluThreads, 0, st>>>(static_cast<const __half*>(gate_up), ld_gu,
                                                            static_cast<__half*>(y), ld_y, inter);
      break;
    default:
      silu_mul_kernel<float><<<grid, kSiluThreads, 0, st>>>(static_cast<const float*>(gate_up), ld_gu,
                                                           static_cast<float*>(y), ld_y, inter);
      break;
  }
  TREAD_CHECK_LAUNCH("silu_mul_kernel");
  return TREAD_OK;
}
