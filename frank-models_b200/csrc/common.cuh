// Shared helpers for the MoE FFN kernels: status handling, bf16 packing,
// small device utilities.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <string>

#include "frank_moe.h"

namespace frank {

// Thread-local last-error message (frank_last_error()).
void set_error(const char* fmt, ...);

#define FRANK_CHECK_ARG(cond, ...)   \
  do {                               \
    if (!(cond)) {                   \
      ::frank::set_error(__VA_ARGS__); \
      return FRANK_EINVAL;           \
    }                                \
  } while (0)

#define FRANK_CUDA_TRY(expr)                                                   \
  do {                                                                         \
    cudaError_t err__ = (expr);                                                \
    if (err__ != cudaSuccess) {                                                \
      ::frank::set_error("%s failed: %s (%s:%d)", #expr,                       \
                         cudaGetErrorString(err__), __FILE__, __LINE__);       \
      return FRANK_ECUDA;                                                      \
    }                                                                          \
  } while (0)

void count_launch();
#define FRANK_LAUNCH_CHECK()               \
  do {                                     \
    ::frank::count_launch();               \
    FRANK_CUDA_TRY(cudaGetLastError());    \
  } while (0)

#define FRANK_TRY(expr)        \
  do {                         \
    int st__ = (expr);         \
    if (st__ != FRANK_OK) return st__; \
  } while (0)

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Bump allocator over a caller-provided workspace.
struct Carve {
  char* base;
  size_t cap;
  size_t used = 0;
  Carve(void* b, size_t c) : base(static_cast<char*>(b)), cap(c) {}
  template <class T>
  T* take(size_t n) {
    used = align_up(used, 256);
    T* p = reinterpret_cast<T*>(base ? base + used : nullptr);
    used += n * sizeof(T);
    return p;
  }
  bool fits() const { return used <= cap; }
};

int num_sms();

// Device error word (bounded-wait timeouts inside persistent kernels).
int32_t* device_error_word();

}  // namespace frank

// ---------------------------------------------------------------- device --

__device__ __forceinline__ float bf16_to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

template <class T>
__device__ __forceinline__ float load_as_f32(const T* p, int64_t i);
template <>
__device__ __forceinline__ float load_as_f32<float>(const float* p, int64_t i) { return p[i]; }
template <>
__device__ __forceinline__ float load_as_f32<__nv_bfloat16>(const __nv_bfloat16* p, int64_t i) {
  return __bfloat162float(p[i]);
}

template <class T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// silu(u) = u / (1 + exp(-u)) exactly as the reference writes it
// (swiglu.mlir:40-45); expf is CUDA's own.
__device__ __forceinline__ float silu_ref(float u) { return u / (1.0f + expf(-u)); }
