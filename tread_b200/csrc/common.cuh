// Shared helpers for the tread_b200 C-ABI library (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdio.h>
#include <stdarg.h>

#include "../../include/tread_b200.h"

namespace tread {

// Per-thread last-error text, returned by tread_last_error().
void set_error(const char* fmt, ...);

#define TREAD_CHECK_ARG(cond, ...)                 \
  do {                                             \
    if (!(cond)) {                                 \
      ::tread::set_error(__VA_ARGS__);             \
      return TREAD_ERR_INVALID;                    \
    }                                              \
  } while (0)

#define TREAD_CHECK_LAUNCH(what)                                                   \
  do {                                                                             \
    cudaError_t e_ = cudaGetLastError();                                           \
    if (e_ != cudaSuccess) {                                                       \
      ::tread::set_error("%s: %s", what, cudaGetErrorString(e_));                  \
      return TREAD_ERR_CUDA;                                                       \
    }                                                                              \
  } while (0)

#define TREAD_CHECK_CUDA(call)                                                     \
  do {                                                                             \
    cudaError_t e_ = (call);                                                       \
    if (e_ != cudaSuccess) {                                                       \
      ::tread::set_error("%s: %s", #call, cudaGetErrorString(e_));                 \
      return TREAD_ERR_CUDA;                                                       \
    }                                                                              \
  } while (0)

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline size_t dtype_size(int dtype) {
  switch (dtype) {
    case TREAD_BF16: return 2;
    case TREAD_F16: return 2;
    case TREAD_F32: return 4;
    default: return 0;
  }
}

// Conversions between storage types and fp32 arithmetic.
template <typename T> struct Num;
template <> struct Num<float> {
  static __device__ __forceinline__ float to_f(float x) { return x; }
  static __device__ __forceinline__ float from_f(float x) { return x; }
};
template <> struct Num<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
};
template <> struct Num<__half> {
  static __device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
  static __device__ __forceinline__ __half from_f(float x) { return __float2half_rn(x); }
};

// 16-byte vector of storage elements.
template <typename T>
union Vec16 {
  int4 raw;
  T e[16 / sizeof(T)];
};

__device__ __forceinline__ int4 ld_stream(const void* p) {
  return __ldcs(reinterpret_cast<const int4*>(p));
}
__device__ __forceinline__ void st_stream(void* p, int4 v) { __stcs(reinterpret_cast<int4*>(p), v); }

}  // namespace tread
