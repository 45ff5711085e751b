// Shared helpers for the evie-cuda kernels and the C ABI: status/error plumbing and small device utilities.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <string>

#include "../../include/evie_cuda.h"

namespace evie {

// Message of the last failure on this host thread (calls without a context, and context creation).
std::string& thread_error();

inline evie_status fail(evie_status code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  thread_error() = buf;
  return code;
}

#define EVIE_CUDA_TRY(expr)                                                                       \
  do {                                                                                            \
    cudaError_t e_ = (expr);                                                                      \
    if (e_ != cudaSuccess)                                                                        \
      return ::evie::fail(EVIE_ERR_CUDA, "%s: %s (%s:%d)", #expr, cudaGetErrorString(e_), __FILE__, \
                          __LINE__);                                                              \
  } while (0)

#define EVIE_CHECK_LAUNCH(name)                                                                        \
  do {                                                                                                 \
    cudaError_t e_ = cudaGetLastError();                                                               \
    if (e_ != cudaSuccess) return ::evie::fail(EVIE_ERR_CUDA, "launch of %s: %s", name, cudaGetErrorString(e_)); \
  } while (0)

#define EVIE_ARG(cond, ...)                                  \
  do {                                                       \
    if (!(cond)) return ::evie::fail(EVIE_ERR_ARG, __VA_ARGS__); \
  } while (0)

__device__ __forceinline__ float bf2f(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float bfbits2f(uint32_t bits16) { return __uint_as_float(bits16 << 16); }

// 8 bf16 packed in a uint4 -> 8 floats (exact widening).
__device__ __forceinline__ void bf16x8_to_f32(const uint4& u, float* f) {
  f[0] = __uint_as_float(u.x << 16); f[1] = __uint_as_float(u.x & 0xffff0000u);
  f[2] = __uint_as_float(u.y << 16); f[3] = __uint_as_float(u.y & 0xffff0000u);
  f[4] = __uint_as_float(u.z << 16); f[5] = __uint_as_float(u.z & 0xffff0000u);
  f[6] = __uint_as_float(u.w << 16); f[7] = __uint_as_float(u.w & 0xffff0000u);
}

__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }
__device__ __forceinline__ float siluf_(float x) { return x / (1.0f + expf(-x)); }

// Streaming (evict-first) vector accesses for data touched exactly once per step.
__device__ __forceinline__ float4 ld_stream4(const float* p) { return __ldcs(reinterpret_cast<const float4*>(p)); }
__device__ __forceinline__ void st_stream4(float* p, float4 v) { __stcs(reinterpret_cast<float4*>(p), v); }

}  // namespace evie
