// Reduced captures: the k most active neurons of each captured frame, on the device.
//
// evie's `top_active` tool (crates/evie/src/mcp.rs:242-256) ranks one token's frame (layers x neurons sqrt-companded
// i8 activations) by |q| and returns the k largest, largest first. Its selection (select_nth_unstable_by) leaves
// the order of equal |q| undefined; here it is fixed as the lower flat index first, so the indices are
// reproducible bit for bit. One CTA per frame row: a histogram of |q| gives the cut value t (fewer than k entries
// above it, at least k at or above it); entries above t are gathered in any order, entries equal to t in index
// order (ballot ranks per 1024-entry tile) until k are taken, and a bitonic sort of (|q|, index) keys puts them in
// the reference's order.
#include <cuda_runtime.h>

#include "model_kernels.h"

namespace evie {

namespace {

constexpr int kThreads = 1024;
constexpr int kMaxK = 128;  // the tool clamps k to 1..100

__device__ __forceinline__ uint32_t absq(int8_t q) { return (uint32_t)(q < 0 ? -(int)q : (int)q); }
// larger key = larger |q|, then lower index
__device__ __forceinline__ unsigned long long key_of(uint32_t a, uint32_t i) {
  return ((unsigned long long)a << 32) | (0xFFFFFFFFu - i);
}

__global__ void __launch_bounds__(kThreads) top_active_kernel(const int8_t* __restrict__ frames, long long width,
                                                              int k, int32_t* __restrict__ out) {
  __shared__ int hist[256];
  __shared__ unsigned long long cand[kMaxK];
  __shared__ int wsum[32];
  __shared__ int s_cut, s_above, s_cnt;
  const int8_t* f = frames + (long long)blockIdx.x * width;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int kk = (long long)k < width ? k : (int)width;
  for (int i = tid; i < 256; i += kThreads) hist[i] = 0;
  for (int i = tid; i < kMaxK; i += kThreads) cand[i] = 0ull;
  if (tid == 0) s_cnt = 0;
  __syncthreads();
  for (long long i = tid; i < width; i += kThreads) atomicAdd(&hist[absq(f[i])], 1);
  __syncthreads();
  if (tid == 0) {  // cut: the largest t with (entries >= t) >= k
    int above = 0, t = 255;
    for (; t > 0; t--) {
      if (above + hist[t] >= kk) break;
      above += hist[t];
    }
    s_cut = t;
    s_above = above;  // entries with |q| > t
  }
  __syncthreads();
  const uint32_t cut = (uint32_t)s_cut;
  const int above = s_above, need = kk - above;  // need >= 1 entries equal to the cut, lowest indices first
  for (long long i = tid; i < width; i += kThreads) {
    const uint32_t a = absq(f[i]);
    if (a > cut) {
      const int p = atomicAdd(&s_cnt, 1);
      if (p < kMaxK) cand[p] = key_of(a, (uint32_t)i);
    }
  }
  int taken = 0;
  for (long long t0 = 0; t0 < width && taken < need; t0 += kThreads) {
    const long long i = t0 + tid;
    const bool eq = i < width && absq(f[i]) == cut;
    const unsigned bal = __ballot_sync(0xffffffffu, eq);
    if (lane == 0) wsum[w] = __popc(bal);
    __syncthreads();
    int before = 0, tile = 0;
    for (int q = 0; q < 32; q++) {
      const int c = wsum[q];
      before += q < w ? c : 0;
      tile += c;
    }
    const int rank = taken + before + __popc(bal & ((1u << lane) - 1u));
    if (eq && rank < need && above + rank < kMaxK) cand[above + rank] = key_of(cut, (uint32_t)i);
    taken += tile;
    __syncthreads();
  }
  // bitonic sort of the kMaxK keys, descending (unused slots are 0 and sort last)
  for (int size = 2; size <= kMaxK; size <<= 1)
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      __syncthreads();
      if (tid < kMaxK) {
        const int j = tid ^ stride;
        if (j > tid) {
          const bool desc = (tid & size) == 0;
          const unsigned long long x = cand[tid], y = cand[j];
          if ((x < y) == desc) cand[tid] = y, cand[j] = x;
        }
      }
    }
  __syncthreads();
  if (tid < kk) out[(long long)blockIdx.x * k + tid] = (int32_t)(0xFFFFFFFFu - (uint32_t)cand[tid]);
}

}  // namespace

evie_status k_top_active(const int8_t* frames, int rows, long long width, int k, int32_t* out, cudaStream_t st) {
  if (rows == 0) return EVIE_OK;
  top_active_kernel<<<rows, kThreads, 0, st>>>(frames, width, k, out);
  EVIE_CHECK_LAUNCH("top_active_kernel");
  return EVIE_OK;
}

}  // namespace evie

extern "C" evie_status evie_top_active(const int8_t* frames, int rows, long long width, int k, int32_t* out,
                                       void* stream) {
  if (rows < 0 || width < 1 || k < 1 || k > 100)
    return evie::fail(EVIE_ERR_ARG, "evie_top_active: rows >= 0, width >= 1, 1 <= k <= 100");
  if (rows > 0 && (!frames || !out)) return evie::fail(EVIE_ERR_ARG, "evie_top_active: null pointer");
  return evie::k_top_active(frames, rows, width, k, out, (cudaStream_t)stream);
}
