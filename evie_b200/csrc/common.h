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

// Device ordinals the library's per-device tables cover (0 .. kMaxDevices - 1).
constexpr int kMaxDevices = 64;

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

#define EVIE_TRY(expr)                  \
  do {                                  \
    evie_status s_ = (expr);            \
    if (s_ != EVIE_OK) return s_;       \
  } while (0)

#define EVIE_ARG(cond, ...)                                  \
  do {                                                       \
    if (!(cond)) return ::evie::fail(EVIE_ERR_ARG, __VA_ARGS__); \
  } while (0)

// Lets the next kernel in the stream start early when it was launched with programmatic stream serialisation (the
// projection GEMM, which streams its first weight tiles before it waits for this grid to complete). Kernels call it
// first; a kernel launched without that attribute after this one is unaffected.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
// Waits until the grids this one depends on have completed and their writes are visible (a no-op when the kernel was
// launched without programmatic stream serialisation). Every kernel of the forward pass calls it right after
// pdl_trigger(), before any memory access or early return, so each grid completes only after its predecessors.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Launch mode of the forward pass's per-row kernels: ordinary launches unless EVIE_PDL_ALL=1 asks for programmatic
// dependent launch on every kernel. Measured on one B200 box, in alternating runs: 6.14 ms per 4B decode step with
// every kernel launched that way against 6.00-6.02 ms with it on the projection GEMMs only (the default; EVIE_NO_PDL=1
// turns those off too), and 5.51 against 5.26 ms with the later attention and mixer kernels. Kernels that start
// early and wait hold the SM resources the GEMM's CTAs need to become resident and stream their first weight tiles.
bool pdl_enabled();
// Streaming multiprocessors of the current device (cached per device).
int sm_count();
template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                            Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// Raises the dynamic shared-memory limit of kernel `fn` to `bytes` on the current device, once per (kernel, device);
// safe to call from several host threads.
evie_status max_dynamic_smem(const void* fn, int bytes);
// Sets kernel attribute `attr` of `fn` to `value` on the current device, once per (kernel, device, attribute, value).
evie_status func_attr(const void* fn, cudaFuncAttribute attr, int value);

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
__device__ __forceinline__ float softplus_(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

// Streaming (evict-first) vector accesses for data touched exactly once per step.
__device__ __forceinline__ float4 ld_stream4(const float* p) { return __ldcs(reinterpret_cast<const float4*>(p)); }
__device__ __forceinline__ void st_stream4(float* p, float4 v) { __stcs(reinterpret_cast<float4*>(p), v); }

}  // namespace evie
