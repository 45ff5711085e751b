// Kernels of the full-model forward pass between the projections (see model_kernels.h for the operand format).
// Each follows the corresponding step of evie-core's CPU engine, crates/evie-core/src/model.rs (line numbers
// below), in f32 with the same formulas; only summation orders differ.
#include "model_kernels.h"
#include "gdn_chunk.h"
#include "tc.h"

#include <algorithm>
#include <climits>
#include <cstdlib>

namespace evie {

namespace {

template <int NT>
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();  // red may still be read from a previous call
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < NT / 32; w++) t += red[w];
  return t;
}

// worker.rs:97-112: q = round(127 sqrt(min(|v|, 1))) with the sign of v.
__device__ __forceinline__ int8_t compand(float v) {
  const float q = roundf(sqrtf(fminf(fabsf(v), 1.0f)) * 127.0f);
  return v < 0.0f ? (int8_t)(-(int)q) : (int8_t)(int)q;
}

constexpr int kNormThreads = 256;

// model.rs:230-241 (embedding rows, then the first pre-mixer RMSNorm)
__global__ void __launch_bounds__(kNormThreads) embed_norm_kernel(const RowInfo* __restrict__ rows,
                                                                  const __nv_bfloat16* __restrict__ embed,
                                                                  float* __restrict__ x, const float* __restrict__ gain,
                                                                  float eps, int d, __nv_bfloat16* __restrict__ X2,
                                                                  size_t xplane, uint32_t* __restrict__ seen,
                                                                  int seen_words) {
  pdl_trigger();
  pdl_wait();
  __shared__ float red[kNormThreads / 32];
  const int r = blockIdx.x;
  const RowInfo ri = rows[r];
  if (threadIdx.x == 0 && seen)
    atomicOr(seen + (size_t)ri.slot * seen_words + (ri.token >> 5), 1u << (ri.token & 31));
  const __nv_bfloat16* e = embed + (size_t)ri.token * d;
  float* xr = x + (size_t)r * d;
  float ss = 0.f;
  for (int i = threadIdx.x; i < d; i += kNormThreads) {
    const float v = __bfloat162float(e[i]);
    xr[i] = v;
    ss += v * v;
  }
  ss = block_sum<kNormThreads>(ss, red);
  const float inv = 1.0f / sqrtf(ss / (float)d + eps);
  for (int i = threadIdx.x; i < d; i += kNormThreads) store_split(X2, xplane, (size_t)r * d + i, xr[i] * inv * gain[i]);
}

// model.rs:246-248, 260-263 (residual add, residual hook, next RMSNorm). One CTA per row, one float4 of the row
// per thread (two beyond 4096 columns), every plane of the projection output loaded before any is added.
__device__ __forceinline__ void store_split4(__nv_bfloat16* X2, size_t plane, size_t idx, float4 v) {
  const __nv_bfloat162 h0 = __floats2bfloat162_rn(v.x, v.y), h1 = __floats2bfloat162_rn(v.z, v.w);
  const float2 f0 = __bfloat1622float2(h0), f1 = __bfloat1622float2(h1);
  const __nv_bfloat162 l0 = __floats2bfloat162_rn(v.x - f0.x, v.y - f0.y);
  const __nv_bfloat162 l1 = __floats2bfloat162_rn(v.z - f1.x, v.w - f1.y);
  uint2 hi, lo;
  hi.x = *reinterpret_cast<const uint32_t*>(&h0);
  hi.y = *reinterpret_cast<const uint32_t*>(&h1);
  lo.x = *reinterpret_cast<const uint32_t*>(&l0);
  lo.y = *reinterpret_cast<const uint32_t*>(&l1);
  *reinterpret_cast<uint2*>(X2 + idx) = hi;
  *reinterpret_cast<uint2*>(X2 + plane + idx) = lo;
}

__device__ __forceinline__ void store_f16x4(uint16_t* dst, float4 v) {
  const __half2 a = __floats2half2_rn(v.x, v.y), b = __floats2half2_rn(v.z, v.w);
  uint2 u;
  u.x = *reinterpret_cast<const uint32_t*>(&a);
  u.y = *reinterpret_cast<const uint32_t*>(&b);
  *reinterpret_cast<uint2*>(dst) = u;
}

__device__ __forceinline__ float block_sum_any(float v, float* red) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
  for (int w = 0; w < nw; w++) t += red[w];
  return t;
}

// x[r] += y[r] (all planes), optional f16 capture, then (if do_norm) X2 row out_row = split(rmsnorm(x[r]) * gain).
__device__ __forceinline__ void add_norm_row(float* __restrict__ x, const YView& y, int ldy, int r, int d,
                                             const float* __restrict__ gain, float eps, __nv_bfloat16* X2,
                                             size_t xplane, int out_row, bool do_norm, uint16_t* resid, int cap_layer,
                                             int L, float* red) {
  const int n4 = d >> 2;
  float* xr = x + (size_t)r * d;
  float4 v[2];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < 2; k++) {
    const int i4 = threadIdx.x + k * blockDim.x;
    if (i4 < n4) {
      float4 a = *reinterpret_cast<const float4*>(xr + 4 * i4);
      const float4 b = y.at4((size_t)r * ldy + 4 * i4);
      a.x += b.x, a.y += b.y, a.z += b.z, a.w += b.w;
      v[k] = a;
      *reinterpret_cast<float4*>(xr + 4 * i4) = a;
      if (resid) store_f16x4(resid + ((size_t)r * L + cap_layer) * d + 4 * i4, a);
      ss += a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w;
    }
  }
  float4 gv[2];
#pragma unroll
  for (int k = 0; k < 2; k++) {  // issued before the reduction's barriers
    const int i4 = threadIdx.x + k * blockDim.x;
    if (do_norm && i4 < n4) gv[k] = *reinterpret_cast<const float4*>(gain + 4 * i4);
  }
  ss = block_sum_any(ss, red);
  if (!do_norm) return;
  const float inv = 1.0f / sqrtf(ss / (float)d + eps);
#pragma unroll
  for (int k = 0; k < 2; k++) {
    const int i4 = threadIdx.x + k * blockDim.x;
    if (i4 < n4) {
      const float4 g = gv[k];
      const float4 a = v[k];
      store_split4(X2, xplane, (size_t)out_row * d + 4 * i4,
                   make_float4(a.x * inv * g.x, a.y * inv * g.y, a.z * inv * g.z, a.w * inv * g.w));
    }
  }
}

__global__ void __launch_bounds__(1024) add_norm_kernel(float* __restrict__ x, YView y, int ldy,
                                                        const float* __restrict__ gain, float eps, int d,
                                                        __nv_bfloat16* __restrict__ X2, size_t xplane,
                                                        uint16_t* __restrict__ resid, int cap_layer, int L) {
  pdl_trigger();
  pdl_wait();
  __shared__ float red[32];
  const int r = blockIdx.x;
  add_norm_row(x, y, ldy, r, d, gain, eps, X2, xplane, r, true, resid, cap_layer, L, red);
}

// model.rs:260-263 for the last layer, then model.rs:271-290 (last row of each sequence, final norm into X2 row s)
__global__ void __launch_bounds__(1024) add_final_kernel(float* __restrict__ x, YView y, int ldy,
                                                         const RowInfo* __restrict__ rows,
                                                         const SegInfo* __restrict__ segs, int nseg,
                                                         const float* __restrict__ gain, float eps, int d,
                                                         __nv_bfloat16* __restrict__ X2,
                                                         uint16_t* __restrict__ resid, int cap_layer, int L) {
  pdl_trigger();
  pdl_wait();
  __shared__ float red[32];
  const int r = blockIdx.x;
  const int s = rows[r].seg;
  const bool last = r == segs[s].start + segs[s].count - 1;
  add_norm_row(x, y, ldy, r, d, gain, eps, X2, (size_t)nseg * d, s, last, resid, cap_layer, L, red);
}

// model.rs:324-353: causal depthwise conv over [conv state ; rows] + SiLU; L2 norm of q and k heads, q * 1/sqrt(dk).
// One CTA = one row x one 128-channel head block.
__global__ void __launch_bounds__(128) conv_silu_norm_kernel(YView y, int ldy,
                                                             const RowInfo* __restrict__ rows,
                                                             const SegInfo* __restrict__ segs,
                                                             float* __restrict__ conv_state, size_t cs_slot,
                                                             const float* __restrict__ conv_w, int K, int conv_dim,
                                                             int hk, float qscale, float* __restrict__ act,
                                                             bool update_window) {
  pdl_trigger();
  pdl_wait();
  __shared__ float red[4];
  const int c = blockIdx.x * 128 + threadIdx.x;
  const int r = blockIdx.y;
  const SegInfo sg = segs[rows[r].seg];
  const int t = r - sg.start;
  float* cs = conv_state + (size_t)sg.slot * cs_slot;
  constexpr int kMaxK = 8;
  float win[kMaxK];  // [state ; rows] inputs of this output, oldest first
  float acc = 0.f;
  for (int j = 0; j < K; j++) {
    const int tt = t - (K - 1) + j;
    const float u = tt >= 0 ? y.at((size_t)(sg.start + tt) * ldy + c) : cs[(size_t)(K - 1 + tt) * conv_dim + c];
    if (j < kMaxK) win[j] = u;
    acc += conv_w[(size_t)c * K + j] * u;
  }
  if (update_window) {
    // Single-row segments (decode): this thread is the only reader of its channel's window, so it can shift the
    // window in place (model.rs:339: keep the last K-1 raw inputs).
    for (int j = 1; j < K && j < kMaxK; j++) cs[(size_t)(j - 1) * conv_dim + c] = win[j];
  }
  float out = siluf_(acc);
  if ((int)blockIdx.x < 2 * hk) {  // q or k head: L2 normalise (kernels.rs dot + 1e-6), q also by 1/sqrt(dk)
    const float ss = block_sum<128>(out * out, red);
    const float inv = 1.0f / sqrtf(ss + 1e-6f);
    out *= inv * ((int)blockIdx.x < hk ? qscale : 1.0f);
  }
  act[(size_t)r * conv_dim + c] = out;
}

// Decode form of the same conv (one row per segment, 4 taps): one warp per 128-channel head block, four consecutive
// channels per lane (float4 loads and stores), so the q/k head norm reduces with warp shuffles and no CTA barrier.
// Same products and sums as conv_silu_norm_kernel, bit for bit: the taps are accumulated in the same order, and the
// shuffle tree below adds the squares in the order of block_sum<128> over one channel per thread. There, channel i of
// a 32-channel group is lane i and the butterfly pairs i ^ 16, i ^ 8, i ^ 4, i ^ 2, i ^ 1. Here, channel i of the
// group is element i % 4 of lane i / 4, so the first three levels are lane xors 4, 2, 1 and the last two are inside
// the lane. The four group sums are then added in group order.
__global__ void __launch_bounds__(128) conv_decode4_kernel(YView y, int ldy, const RowInfo* __restrict__ rows,
                                                           const SegInfo* __restrict__ segs,
                                                           float* __restrict__ conv_state, size_t cs_slot,
                                                           const float* __restrict__ conv_w, int conv_dim, int hk,
                                                           float qscale, float* __restrict__ act) {
  pdl_trigger();
  pdl_wait();
  constexpr int K = 4;
  const int lane = threadIdx.x & 31;
  const int blk = blockIdx.x * 4 + (threadIdx.x >> 5);  // 128-channel block of this warp
  if (blk * 128 >= conv_dim) return;                    // the whole warp leaves together
  const int c = blk * 128 + lane * 4;
  const int r = blockIdx.y;
  const SegInfo sg = segs[rows[r].seg];
  const int t = r - sg.start;
  float* cs = conv_state + (size_t)sg.slot * cs_slot;
  float4 win[K];  // [state ; rows] inputs of this output, oldest first
#pragma unroll
  for (int j = 0; j < K; j++) {
    const int tt = t - (K - 1) + j;
    win[j] = tt >= 0 ? y.at4((size_t)(sg.start + tt) * ldy + c)
                     : *reinterpret_cast<const float4*>(cs + (size_t)(K - 1 + tt) * conv_dim + c);
  }
  float4 w4[K];  // taps of channels c .. c + 3: w4[e] = conv_w[(c + e) * K + 0 .. 3]
#pragma unroll
  for (int e = 0; e < 4; e++) w4[e] = *reinterpret_cast<const float4*>(conv_w + (size_t)(c + e) * K);
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int j = 0; j < K; j++) {
    const float u[4] = {win[j].x, win[j].y, win[j].z, win[j].w};
#pragma unroll
    for (int e = 0; e < 4; e++) {
      const float w = j == 0 ? w4[e].x : j == 1 ? w4[e].y : j == 2 ? w4[e].z : w4[e].w;
      acc[e] += w * u[e];
    }
  }
  // model.rs:339: the window keeps the last K-1 raw inputs; this lane is the only reader of its four channels
#pragma unroll
  for (int j = 1; j < K; j++) *reinterpret_cast<float4*>(cs + (size_t)(j - 1) * conv_dim + c) = win[j];
  float out[4];
#pragma unroll
  for (int e = 0; e < 4; e++) out[e] = siluf_(acc[e]);
  if (blk < 2 * hk) {  // q or k head: L2 normalise (kernels.rs dot + 1e-6), q also by 1/sqrt(dk)
    float sq[4];
#pragma unroll
    for (int e = 0; e < 4; e++) {
      sq[e] = out[e] * out[e];
      sq[e] += __shfl_xor_sync(0xffffffffu, sq[e], 4);
      sq[e] += __shfl_xor_sync(0xffffffffu, sq[e], 2);
      sq[e] += __shfl_xor_sync(0xffffffffu, sq[e], 1);
    }
    const float grp = (sq[0] + sq[2]) + (sq[1] + sq[3]);  // one 32-channel group, in every lane of its 8
    const float g0 = __shfl_sync(0xffffffffu, grp, 0), g1 = __shfl_sync(0xffffffffu, grp, 8);
    const float g2 = __shfl_sync(0xffffffffu, grp, 16), g3 = __shfl_sync(0xffffffffu, grp, 24);
    const float ss = ((g0 + g1) + g2) + g3;
    const float inv = 1.0f / sqrtf(ss + 1e-6f);
    const float scl = inv * (blk < hk ? qscale : 1.0f);
#pragma unroll
    for (int e = 0; e < 4; e++) out[e] *= scl;
  }
  *reinterpret_cast<float4*>(act + (size_t)r * conv_dim + c) = make_float4(out[0], out[1], out[2], out[3]);
}

// The same conv for segments of many rows (prefill): one CTA per (128-channel block, segment, 64 consecutive rows),
// one thread per channel walking the rows with its K-1 previous inputs in registers, so every input is read once.
// Same products, summation order and head-norm reduction as conv_silu_norm_kernel.
// split_qk: the q and k channels are written as two bf16 planes, hi = bf16(x) and lo = bf16(x - hi), into the bytes
// of the row's q/k columns (bf16 [2][2 key_dim] in place of f32 [2 key_dim]), the operand format of the chunked
// prefill's tensor-core tiles; v stays f32.
constexpr int kConvRows = 64;
template <int K>
__global__ void __launch_bounds__(128) conv_rows_kernel(YView y, int ldy, const SegInfo* __restrict__ segs,
                                                        const float* __restrict__ conv_state, size_t cs_slot,
                                                        const float* __restrict__ conv_w, int conv_dim, int hk,
                                                        float qscale, float* __restrict__ act, bool split_qk) {
  pdl_trigger();
  pdl_wait();
  __shared__ float red[4];
  const int c = blockIdx.x * 128 + threadIdx.x;
  const SegInfo sg = segs[blockIdx.y];
  const int t0 = blockIdx.z * kConvRows;
  if (t0 >= sg.count) return;
  const int nt = min(kConvRows, sg.count - t0);
  const float* cs = conv_state + (size_t)sg.slot * cs_slot;
  float w[K], win[K];
#pragma unroll
  for (int j = 0; j < K; j++) w[j] = conv_w[(size_t)c * K + j];
#pragma unroll
  for (int j = 0; j < K - 1; j++) {
    const int tt = t0 - (K - 1) + j;
    win[j] = tt >= 0 ? y.at((size_t)(sg.start + tt) * ldy + c) : cs[(size_t)(K - 1 + tt) * conv_dim + c];
  }
  const bool head_norm = (int)blockIdx.x < 2 * hk;
  const float scl = (int)blockIdx.x < hk ? qscale : 1.0f;
  for (int t = 0; t < nt; t++) {
    const size_t row = (size_t)sg.start + t0 + t;
    win[K - 1] = y.at(row * ldy + c);
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < K; j++) acc += w[j] * win[j];
#pragma unroll
    for (int j = 0; j < K - 1; j++) win[j] = win[j + 1];
    float out = siluf_(acc);
    if (head_norm) {  // q or k head: L2 normalise (kernels.rs dot + 1e-6), q also by 1/sqrt(dk)
      const float ss = block_sum<128>(out * out, red);
      out *= (1.0f / sqrtf(ss + 1e-6f)) * scl;
    }
    if (split_qk && head_norm) {
      __nv_bfloat16* qk = reinterpret_cast<__nv_bfloat16*>(act + row * conv_dim);
      const __nv_bfloat16 hi = __float2bfloat16_rn(out);
      qk[c] = hi;
      qk[(size_t)256 * hk + c] = __float2bfloat16_rn(out - __bfloat162float(hi));  // 2 key_dim = 256 hk channels
    } else {
      act[row * conv_dim + c] = out;
    }
  }
}

// The rows form with the decode conv's layout: one warp per (128-channel head block, segment, 64 consecutive rows),
// four consecutive channels per lane, so the q/k head norm of a row reduces with shuffles alone (the tree of
// conv_decode4_kernel, which adds the squares in block_sum<128>'s order) and no CTA barrier stands between rows.
// Each lane keeps its channels' last three inputs in registers and loads the next rows' inputs ahead (kConvAhead
// rows in flight; 8 measured slower, 15.9 against 13.7 ms per 4B prefill call: more registers, fewer CTAs per SM).
// ONE: the input projection has a single plane (no K slices), read by plain float4 loads. Same products, order of
// operations and outputs as conv_rows_kernel, bit for bit.
constexpr int kConvAhead = 4;
template <bool ONE>
__global__ void __launch_bounds__(128) conv_rows4_kernel(YView y, int ldy, const SegInfo* __restrict__ segs,
                                                         const float* __restrict__ conv_state, size_t cs_slot,
                                                         const float* __restrict__ conv_w, int conv_dim, int hk,
                                                         float qscale, float* __restrict__ act, bool split_qk) {
  pdl_trigger();
  pdl_wait();
  constexpr int K = 4;
  const auto ld4 = [&](size_t i) { return ONE ? *reinterpret_cast<const float4*>(y.p + i) : y.at4(i); };
  const int lane = threadIdx.x & 31;
  const int blk = blockIdx.x * 4 + (threadIdx.x >> 5);  // 128-channel block of this warp
  if (blk * 128 >= conv_dim) return;                    // the whole warp leaves together
  const SegInfo sg = segs[blockIdx.y];
  const int t0 = blockIdx.z * kConvRows;
  if (t0 >= sg.count) return;
  const int nt = min(kConvRows, sg.count - t0);
  const int c = blk * 128 + lane * 4;
  const float* cs = conv_state + (size_t)sg.slot * cs_slot;
  float4 w4[K];  // taps of channels c .. c + 3: w4[e] = conv_w[(c + e) * K + 0 .. 3]
#pragma unroll
  for (int e = 0; e < 4; e++) w4[e] = *reinterpret_cast<const float4*>(conv_w + (size_t)(c + e) * K);
  float4 win[K];  // [state ; rows] inputs, oldest first; win[K - 1] is the current row's
#pragma unroll
  for (int j = 0; j < K - 1; j++) {
    const int tt = t0 - (K - 1) + j;
    win[j] = tt >= 0 ? ld4((size_t)(sg.start + tt) * ldy + c)
                     : *reinterpret_cast<const float4*>(cs + (size_t)(K - 1 + tt) * conv_dim + c);
  }
  const bool head_norm = blk < 2 * hk;
  const float scl0 = blk < hk ? qscale : 1.0f;
  float4 ahead[kConvAhead];  // inputs of rows t .. t + kConvAhead - 1
#pragma unroll
  for (int i = 0; i < kConvAhead; i++)
    ahead[i] = i < nt ? ld4((size_t)(sg.start + t0 + i) * ldy + c) : make_float4(0.f, 0.f, 0.f, 0.f);
  for (int t = 0; t < nt; t++) {
    const size_t row = (size_t)sg.start + t0 + t;
    win[K - 1] = ahead[0];
#pragma unroll
    for (int i = 0; i + 1 < kConvAhead; i++) ahead[i] = ahead[i + 1];
    const int tn = t + kConvAhead;
    ahead[kConvAhead - 1] = tn < nt ? ld4((row + kConvAhead) * ldy + c) : make_float4(0.f, 0.f, 0.f, 0.f);
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int j = 0; j < K; j++) {
      const float u[4] = {win[j].x, win[j].y, win[j].z, win[j].w};
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const float w = j == 0 ? w4[e].x : j == 1 ? w4[e].y : j == 2 ? w4[e].z : w4[e].w;
        acc[e] += w * u[e];
      }
    }
#pragma unroll
    for (int j = 0; j < K - 1; j++) win[j] = win[j + 1];
    float out[4];
#pragma unroll
    for (int e = 0; e < 4; e++) out[e] = siluf_(acc[e]);
    if (head_norm) {  // q or k head: L2 normalise (kernels.rs dot + 1e-6), q also by 1/sqrt(dk)
      float sq[4];
#pragma unroll
      for (int e = 0; e < 4; e++) {
        sq[e] = out[e] * out[e];
        sq[e] += __shfl_xor_sync(0xffffffffu, sq[e], 4);
        sq[e] += __shfl_xor_sync(0xffffffffu, sq[e], 2);
        sq[e] += __shfl_xor_sync(0xffffffffu, sq[e], 1);
      }
      const float grp = (sq[0] + sq[2]) + (sq[1] + sq[3]);  // one 32-channel group, in every lane of its 8
      const float g0 = __shfl_sync(0xffffffffu, grp, 0), g1 = __shfl_sync(0xffffffffu, grp, 8);
      const float g2 = __shfl_sync(0xffffffffu, grp, 16), g3 = __shfl_sync(0xffffffffu, grp, 24);
      const float ss = ((g0 + g1) + g2) + g3;
      const float scl = (1.0f / sqrtf(ss + 1e-6f)) * scl0;
#pragma unroll
      for (int e = 0; e < 4; e++) out[e] *= scl;
    }
    if (split_qk && head_norm) {  // hi and lo bf16 planes in the bytes of the row's q/k columns
      __nv_bfloat16* qk = reinterpret_cast<__nv_bfloat16*>(act + row * conv_dim);
      const __nv_bfloat162 h0 = __floats2bfloat162_rn(out[0], out[1]), h1 = __floats2bfloat162_rn(out[2], out[3]);
      const float2 f0 = __bfloat1622float2(h0), f1 = __bfloat1622float2(h1);
      const __nv_bfloat162 l0 = __floats2bfloat162_rn(out[0] - f0.x, out[1] - f0.y);
      const __nv_bfloat162 l1 = __floats2bfloat162_rn(out[2] - f1.x, out[3] - f1.y);
      uint2 hi, lo;
      hi.x = *reinterpret_cast<const uint32_t*>(&h0);
      hi.y = *reinterpret_cast<const uint32_t*>(&h1);
      lo.x = *reinterpret_cast<const uint32_t*>(&l0);
      lo.y = *reinterpret_cast<const uint32_t*>(&l1);
      *reinterpret_cast<uint2*>(qk + c) = hi;
      *reinterpret_cast<uint2*>(qk + (size_t)256 * hk + c) = lo;  // 2 key_dim = 256 hk channels
    } else {
      *reinterpret_cast<float4*>(act + row * conv_dim + c) = make_float4(out[0], out[1], out[2], out[3]);
    }
  }
}

// model.rs:339: the conv window keeps the last K-1 raw inputs of [state ; rows].
__global__ void conv_state_update_kernel(YView y, int ldy,
                                         const SegInfo* __restrict__ segs, float* __restrict__ conv_state,
                                         size_t cs_slot, int K, int conv_dim) {
  pdl_trigger();
  pdl_wait();
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= conv_dim) return;
  const SegInfo sg = segs[blockIdx.y];
  if (sg.count == 0) return;
  float* cs = conv_state + (size_t)sg.slot * cs_slot;
  for (int i = 0; i < K - 1; i++) {
    const int src = sg.count + i;  // index into [state (K-1) ; rows (count)]
    const float v = src < K - 1 ? cs[(size_t)src * conv_dim + c]
                                : y.at((size_t)(sg.start + src - (K - 1)) * ldy + c);
    cs[(size_t)i * conv_dim + c] = v;
  }
}

// model.rs:362-387 (+ recur_body model.rs:503-524): the rows of one segment for one value head, 256 threads, the
// head's [128][128] state resident in registers across the rows (thread (warp, lane) holds rows warp + 8 r, columns
// 4 lane .. 4 lane + 3); gated RMSNorm (model.rs:377-383) of each row's output into X2.
constexpr int kMixThreads = 256;
struct MixShared {
  float sq[128], sk[128];
  float4 red[8][32];
  float sred[4];
  float s_o[128];
  float s_db[2];  // the row's decay and beta
};
__device__ __forceinline__ void mixer_rows(float4 (&s)[16], MixShared& sh, const float* __restrict__ act,
                                           const YView& y, int ldy, const SegInfo& sg, int head,
                                           const float* __restrict__ neg_a, const float* __restrict__ dt_bias,
                                           const float* __restrict__ norm_w, int conv_dim, int key_dim, int vd, int hv,
                                           int ratio, float eps, __nv_bfloat16* __restrict__ X2, size_t xplane) {
  constexpr int DK = 128, DV = 128;
  const int kh = head / ratio;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;  // lane: 4 columns; warp: rows warp + 8 r
  for (int t = 0; t < sg.count; t++) {
    const int row = sg.start + t;
    const float* ar = act + (size_t)row * conv_dim;
    if (tid < DK) sh.sq[tid] = ar[kh * DK + tid];
    else sh.sk[tid - DK] = ar[key_dim + kh * DK + (tid - DK)];
    const float4 v4 = *reinterpret_cast<const float4*>(ar + 2 * key_dim + head * DV + lane * 4);
    if (tid == DK) {  // one thread reads the head's b and a logits (all K-slice planes) for the whole CTA
      const float bb = y.at((size_t)row * ldy + conv_dim + vd + head);
      const float aa = y.at((size_t)row * ldy + conv_dim + vd + hv + head);
      sh.s_db[0] = expf(neg_a[head] * softplus_(aa + dt_bias[head]));
      sh.s_db[1] = sigmoidf_(bb);
    }
    // the output gate is read here, with the other inputs, so its latency is not exposed after the state update
    const float z = tid < DV ? y.at((size_t)row * ldy + conv_dim + head * DV + tid) : 0.f;
    __syncthreads();
    const float decay = sh.s_db[0], beta = sh.s_db[1];
    float4 kv = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int r = 0; r < 16; r++) {
      const float kr = sh.sk[warp + 8 * r];
      kv.x += s[r].x * kr; kv.y += s[r].y * kr; kv.z += s[r].z * kr; kv.w += s[r].w * kr;
    }
    sh.red[warp][lane] = kv;
    __syncthreads();
    kv = sh.red[0][lane];
#pragma unroll
    for (int w = 1; w < 8; w++) {
      const float4 u = sh.red[w][lane];
      kv.x += u.x; kv.y += u.y; kv.z += u.z; kv.w += u.w;
    }
    const float d0 = (v4.x - decay * kv.x) * beta, d1 = (v4.y - decay * kv.y) * beta;
    const float d2 = (v4.z - decay * kv.z) * beta, d3 = (v4.w - decay * kv.w) * beta;
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int r = 0; r < 16; r++) {
      const int i = warp + 8 * r;
      const float kr = sh.sk[i], qr = sh.sq[i];
      s[r].x = s[r].x * decay + kr * d0; s[r].y = s[r].y * decay + kr * d1;
      s[r].z = s[r].z * decay + kr * d2; s[r].w = s[r].w * decay + kr * d3;
      o.x += s[r].x * qr; o.y += s[r].y * qr; o.z += s[r].z * qr; o.w += s[r].w * qr;
    }
    __syncthreads();  // everyone has read red (kv) before it is reused
    sh.red[warp][lane] = o;
    __syncthreads();
    if (tid < DV) {  // thread j finishes output column j
      const float* rf = reinterpret_cast<const float*>(&sh.red[0][0]);
      float oj = 0.f;
#pragma unroll
      for (int w = 0; w < 8; w++) oj += rf[w * DV + tid];
      sh.s_o[tid] = oj;
      float ss = oj * oj;
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
      if (lane == 0) sh.sred[warp] = ss;
    }
    __syncthreads();
    if (tid < DV) {  // gated RMSNorm, model.rs:377-383: o * rsqrt(mean o^2 + eps) * w * silu(z)
      const float ms = (sh.sred[0] + sh.sred[1] + sh.sred[2] + sh.sred[3]) / (float)DV;
      const float inv = 1.0f / sqrtf(ms + eps);
      store_split(X2, xplane, (size_t)row * vd + head * DV + tid, sh.s_o[tid] * inv * norm_w[tid] * siluf_(z));
    }
  }
}

// One CTA per (segment, value head).
__global__ void __launch_bounds__(kMixThreads) gdn_mixer_kernel(
    const float* __restrict__ act, YView y, int ldy,
    const SegInfo* __restrict__ segs, float* __restrict__ rec_state, size_t rs_slot, const float* __restrict__ neg_a,
    const float* __restrict__ dt_bias, const float* __restrict__ norm_w, int conv_dim, int key_dim, int vd, int hv,
    int ratio, float eps, __nv_bfloat16* __restrict__ X2, size_t xplane) {
  pdl_trigger();
  pdl_wait();
  constexpr int DK = 128, DV = 128;
  const int head = blockIdx.x;
  const SegInfo sg = segs[blockIdx.y];
  if (sg.count == 0) return;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  __shared__ MixShared sh;
  float* Sh = rec_state + (size_t)sg.slot * rs_slot + (size_t)head * DK * DV + lane * 4;
  float4 s[16];
#pragma unroll
  for (int r = 0; r < 16; r++) s[r] = *reinterpret_cast<const float4*>(Sh + (size_t)(warp + 8 * r) * DV);
  mixer_rows(s, sh, act, y, ldy, sg, head, neg_a, dt_bias, norm_w, conv_dim, key_dim, vd, hv, ratio, eps, X2, xplane);
#pragma unroll
  for (int r = 0; r < 16; r++) *reinterpret_cast<float4*>(Sh + (size_t)(warp + 8 * r) * DV) = s[r];
}

// The same units as a persistent kernel (decode, one row per segment): each CTA walks units u = blockIdx.x,
// blockIdx.x + gridDim.x, ... of (segment, value head). A head's 64 KB state is one contiguous block, so it arrives
// by one bulk copy into shared memory, in the register layout's row order (thread (warp, lane) reads rows
// warp + 8 r, columns 4 lane .. 4 lane + 3: 512 consecutive bytes per warp, no bank conflicts). The unit's inputs
// come with it on the same mbarrier phase, into one of two staging buffers: the q, k and v rows (512 bytes each,
// from the conv's output row), the output gate z of every K-slice plane of the input projection (512 bytes each),
// and, per plane, the 16-byte chunks that hold the head's b and a logits. The next unit's copies are issued as soon
// as every thread has moved the current state into registers, so its HBM and L2 reads overlap this unit's
// recurrence, norm and state store. Every thread sums the planes of b and a and forms decay and beta itself (same
// operations in every thread), so the unit starts without a barrier on them. Same arithmetic per unit as
// gdn_mixer_kernel (planes added in plane order, as YView::at adds them). The copies' wait is bounded: a give-up
// ends the CTA's walk (after one more bounded wait for the copies in flight) and counts in the device counter.
constexpr int kMixStateBytes = 128 * 128 * 4;
__host__ __device__ constexpr int mix_stage_floats(int planes) { return 3 * 128 + planes * 128 + planes * 8; }
__global__ void __launch_bounds__(kMixThreads, 2) gdn_mixer_persist_kernel(
    const float* __restrict__ act, YView y, int ldy,
    const SegInfo* __restrict__ segs, int nseg, float* __restrict__ rec_state, size_t rs_slot,
    const float* __restrict__ neg_a, const float* __restrict__ dt_bias, const float* __restrict__ norm_w, int conv_dim,
    int key_dim, int vd, int hv, int ratio, float eps, __nv_bfloat16* __restrict__ X2, size_t xplane,
    unsigned int* timeouts) {
  pdl_trigger();
  pdl_wait();
  constexpr int DK = 128, DV = 128;
  extern __shared__ __align__(128) float4 mix_state[];  // [128 rows][32 float4], then two staging buffers
  float* stage0 = reinterpret_cast<float*>(mix_state + kMixStateBytes / 16);
  const int np = y.n;
  const int stage_floats = mix_stage_floats(np);
  __shared__ float4 red[8][32];
  __shared__ float sred[4];
  __shared__ float s_o[DV];
  __shared__ __align__(8) uint64_t bar;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int units = nseg * hv;
  if (tid == 0) {
    tc::mbar_init(&bar, 1);
    tc::fence_barrier_init();
  }
  __syncthreads();
  auto state_of = [&](int u) {
    return rec_state + (size_t)segs[u / hv].slot * rs_slot + (size_t)(u % hv) * DK * DV;
  };
  auto issue = [&](int u, int buf) {
    if (tid == 0) {
      const int head = u % hv, kh = head / ratio;
      const size_t row = (size_t)segs[u / hv].start;
      float* st = stage0 + buf * stage_floats;
      const float* ar = act + row * conv_dim;
      const size_t ib = row * ldy + conv_dim + vd + head, ia = ib + hv, iz = row * ldy + conv_dim + (size_t)head * DV;
      tc::fence_proxy_async();
      tc::mbar_arrive_expect_tx(&bar, kMixStateBytes + (3 + np) * 512 + np * 32);
      tc::bulk_load(mix_state, state_of(u), kMixStateBytes, &bar);
      tc::bulk_load(st, ar + kh * DK, 512, &bar);                          // q
      tc::bulk_load(st + 128, ar + key_dim + kh * DK, 512, &bar);          // k
      tc::bulk_load(st + 256, ar + 2 * key_dim + head * DV, 512, &bar);    // v
      for (int p = 0; p < np; p++) {
        const float* yp = y.p + (size_t)p * y.plane;
        tc::bulk_load(st + 384 + p * 128, yp + iz, 512, &bar);                           // z
        tc::bulk_load(st + 384 + np * 128 + p * 4, yp + (ib & ~(size_t)3), 16, &bar);     // b's chunk
        tc::bulk_load(st + 384 + np * 132 + p * 4, yp + (ia & ~(size_t)3), 16, &bar);     // a's chunk
      }
    }
  };
  uint32_t phase = 0;
  bool pending = false;
  int u = blockIdx.x, k = 0;
  if (u < units) {
    issue(u, 0);
    pending = true;
  }
  for (; u < units; u += gridDim.x, k++) {
    const bool got = tc::mbar_wait(&bar, phase);
    float4 s[16];
#pragma unroll
    for (int r = 0; r < 16; r++) s[r] = mix_state[(warp + 8 * r) * 32 + lane];
    if (!__syncthreads_and(got)) break;  // every thread has also read the state out of shared memory
    phase ^= 1;
    pending = false;
    if (u + (int)gridDim.x < units) {
      issue(u + gridDim.x, (k + 1) & 1);
      pending = true;
    }
    const float* st = stage0 + (k & 1) * stage_floats;
    const float* sq = st;
    const float* sk = st + 128;
    const int head = u % hv;
    const size_t row = (size_t)segs[u / hv].start;
    // model.rs:374-375 from the planes of b and a, added in plane order
    const size_t ib = row * ldy + conv_dim + vd + head, ia = ib + hv;
    float bb = st[384 + np * 128 + (ib & 3)], aa = st[384 + np * 132 + (ia & 3)];
    for (int p = 1; p < np; p++) {
      bb += st[384 + np * 128 + p * 4 + (ib & 3)];
      aa += st[384 + np * 132 + p * 4 + (ia & 3)];
    }
    const float decay = expf(neg_a[head] * softplus_(aa + dt_bias[head]));
    const float beta = sigmoidf_(bb);
    float z = 0.f;
    if (tid < DV) {
      z = st[384 + tid];
      for (int p = 1; p < np; p++) z += st[384 + p * 128 + tid];
    }
    const float4 v4 = *reinterpret_cast<const float4*>(st + 256 + lane * 4);
    float4 kv = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int r = 0; r < 16; r++) {
      const float kr = sk[warp + 8 * r];
      kv.x += s[r].x * kr; kv.y += s[r].y * kr; kv.z += s[r].z * kr; kv.w += s[r].w * kr;
    }
    red[warp][lane] = kv;
    __syncthreads();
    kv = red[0][lane];
#pragma unroll
    for (int w = 1; w < 8; w++) {
      const float4 t = red[w][lane];
      kv.x += t.x; kv.y += t.y; kv.z += t.z; kv.w += t.w;
    }
    const float d0 = (v4.x - decay * kv.x) * beta, d1 = (v4.y - decay * kv.y) * beta;
    const float d2 = (v4.z - decay * kv.z) * beta, d3 = (v4.w - decay * kv.w) * beta;
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int r = 0; r < 16; r++) {
      const int i = warp + 8 * r;
      const float kr = sk[i], qr = sq[i];
      s[r].x = s[r].x * decay + kr * d0; s[r].y = s[r].y * decay + kr * d1;
      s[r].z = s[r].z * decay + kr * d2; s[r].w = s[r].w * decay + kr * d3;
      o.x += s[r].x * qr; o.y += s[r].y * qr; o.z += s[r].z * qr; o.w += s[r].w * qr;
    }
    float* Sh = state_of(u) + lane * 4;
#pragma unroll
    for (int r = 0; r < 16; r++) *reinterpret_cast<float4*>(Sh + (size_t)(warp + 8 * r) * DV) = s[r];
    __syncthreads();  // everyone has read red (kv) before it is reused
    red[warp][lane] = o;
    __syncthreads();
    if (tid < DV) {  // thread j finishes output column j
      const float* rf = reinterpret_cast<const float*>(&red[0][0]);
      float oj = 0.f;
#pragma unroll
      for (int w = 0; w < 8; w++) oj += rf[w * DV + tid];
      s_o[tid] = oj;
      float ss = oj * oj;
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
      if (lane == 0) sred[warp] = ss;
    }
    __syncthreads();
    if (tid < DV) {  // gated RMSNorm, model.rs:377-383: o * rsqrt(mean o^2 + eps) * w * silu(z)
      const float ms = (sred[0] + sred[1] + sred[2] + sred[3]) / (float)DV;
      const float inv = 1.0f / sqrtf(ms + eps);
      store_split(X2, xplane, row * vd + head * DV + tid, s_o[tid] * inv * norm_w[tid] * siluf_(z));
    }
  }
  if (pending && tid == 0) {  // the walk ended on a give-up: wait once more for those copies, count the give-up
    tc::mbar_wait(&bar, phase);
    atomicAdd(timeouts, 1u);
  }
}

// Prefill form of the mixer (segments of many rows): one CTA per (segment, value head), the head's state in registers
// with warp w owning columns 16w .. 16w + 15 and lane (rg, cg) = (lane / 4, lane % 4) rows rg + 8 r, columns
// 16 w + 4 cg .. + 3, so both reductions over the key index (S^T k and S^T q) stay inside a warp: no CTA barrier per
// token. q, k, v, z, decay and beta of 32 tokens are staged in shared memory at a time, and the gated RMSNorm of
// those 32 outputs runs in parallel after them. Same recurrence and order of operations per token as
// gdn_mixer_kernel (model.rs:501-524; gated RMSNorm model.rs:377-383).
constexpr int kSeqChunk = 32;
__global__ void __launch_bounds__(kMixThreads, 2) gdn_mixer_seq_kernel(
    const float* __restrict__ act, YView y, int ldy, const SegInfo* __restrict__ segs, float* __restrict__ rec_state,
    size_t rs_slot, const float* __restrict__ neg_a, const float* __restrict__ dt_bias, const float* __restrict__ norm_w,
    int conv_dim, int key_dim, int vd, int hv, int ratio, float eps, __nv_bfloat16* __restrict__ X2, size_t xplane) {
  pdl_trigger();
  pdl_wait();
  constexpr int DK = 128, DV = 128;
  extern __shared__ __align__(16) float smf[];
  float* sq = smf;                          // [32][128]
  float* sk = sq + kSeqChunk * DK;          // [32][128]
  float* sv = sk + kSeqChunk * DK;          // [32][128]
  float* sz = sv + kSeqChunk * DV;          // [32][128]
  float* so = sz + kSeqChunk * DV;          // [32][128] outputs before the norm
  float* sdec = so + kSeqChunk * DV;        // [32]
  float* sbeta = sdec + kSeqChunk;          // [32]
  const int head = blockIdx.x;
  const SegInfo sg = segs[blockIdx.y];
  if (sg.count == 0) return;
  const int kh = head / ratio;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int rg = lane >> 2, cg = lane & 3;
  const int c0 = 16 * warp + 4 * cg;
  float* Sh = rec_state + (size_t)sg.slot * rs_slot + (size_t)head * DK * DV + c0;
  float4 s[16];
#pragma unroll
  for (int r = 0; r < 16; r++) s[r] = *reinterpret_cast<const float4*>(Sh + (size_t)(rg + 8 * r) * DV);

  for (int t0 = 0; t0 < sg.count; t0 += kSeqChunk) {
    const int nt = min(kSeqChunk, sg.count - t0);
    // ---- stage the chunk's inputs (rows of act and y for this head); unrolled so that each thread has several
    // loads in flight instead of waiting out one load per iteration
#pragma unroll 4
    for (int i = tid; i < nt * 128; i += kMixThreads) {
      const int t = i >> 7, part = (i >> 5) & 3, j = (i & 31) * 4;  // per token: q, k, v, z, 32 float4 each
      const size_t row = (size_t)sg.start + t0 + t;
      float4 val;
      if (part == 3) {
        val = y.at4(row * ldy + conv_dim + head * DV + j);
      } else {
        const int off = part == 0 ? kh * DK : part == 1 ? key_dim + kh * DK : 2 * key_dim + head * DV;
        val = *reinterpret_cast<const float4*>(act + row * conv_dim + off + j);
      }
      *reinterpret_cast<float4*>(smf + (size_t)part * kSeqChunk * DK + t * DK + j) = val;
    }
    if (tid < nt) {
      const int row = sg.start + t0 + tid;
      const float bb = y.at((size_t)row * ldy + conv_dim + vd + head);
      const float aa = y.at((size_t)row * ldy + conv_dim + vd + hv + head);
      sdec[tid] = expf(neg_a[head] * softplus_(aa + dt_bias[head]));
      sbeta[tid] = sigmoidf_(bb);
    }
    __syncthreads();
    // ---- the recurrence, token by token, warp-local
    for (int t = 0; t < nt; t++) {
      const float* kt = sk + t * DK;
      const float* qt = sq + t * DK;
      const float decay = sdec[t], beta = sbeta[t];
      float4 kv = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int r = 0; r < 16; r++) {
        const float kr = kt[rg + 8 * r];
        kv.x += s[r].x * kr; kv.y += s[r].y * kr; kv.z += s[r].z * kr; kv.w += s[r].w * kr;
      }
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        kv.x += __shfl_xor_sync(0xffffffffu, kv.x, off);
        kv.y += __shfl_xor_sync(0xffffffffu, kv.y, off);
        kv.z += __shfl_xor_sync(0xffffffffu, kv.z, off);
        kv.w += __shfl_xor_sync(0xffffffffu, kv.w, off);
      }
      const float4 v4 = *reinterpret_cast<const float4*>(sv + t * DV + c0);
      const float d0 = (v4.x - decay * kv.x) * beta, d1 = (v4.y - decay * kv.y) * beta;
      const float d2 = (v4.z - decay * kv.z) * beta, d3 = (v4.w - decay * kv.w) * beta;
      float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int r = 0; r < 16; r++) {
        const int i = rg + 8 * r;
        const float kr = kt[i], qr = qt[i];
        s[r].x = s[r].x * decay + kr * d0; s[r].y = s[r].y * decay + kr * d1;
        s[r].z = s[r].z * decay + kr * d2; s[r].w = s[r].w * decay + kr * d3;
        o.x += s[r].x * qr; o.y += s[r].y * qr; o.z += s[r].z * qr; o.w += s[r].w * qr;
      }
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        o.x += __shfl_xor_sync(0xffffffffu, o.x, off);
        o.y += __shfl_xor_sync(0xffffffffu, o.y, off);
        o.z += __shfl_xor_sync(0xffffffffu, o.z, off);
        o.w += __shfl_xor_sync(0xffffffffu, o.w, off);
      }
      if (rg == 0) *reinterpret_cast<float4*>(so + t * DV + c0) = o;
    }
    __syncthreads();
    // ---- gated RMSNorm of the chunk's outputs: 8 threads per token, 16 columns each
    {
      // Every lane takes part in the shuffles (a full-mask shuffle must be reached by the whole warp); only the
      // loads and stores are limited to the chunk's tokens.
      const int t = tid >> 3, part = tid & 7;
      const bool live = t < nt;
      const float* ot = so + t * DV + 16 * part;
      float ss = 0.f;
      if (live) {
#pragma unroll
        for (int j = 0; j < 16; j++) ss += ot[j] * ot[j];
      }
#pragma unroll
      for (int off = 1; off < 8; off <<= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
      if (live) {
        const float inv = 1.0f / sqrtf(ss / (float)DV + eps);
        const int row = sg.start + t0 + t;
#pragma unroll
        for (int j = 0; j < 16; j++) {
          const int col = 16 * part + j;
          store_split(X2, xplane, (size_t)row * vd + head * DV + col,
                      ot[j] * inv * norm_w[col] * siluf_(sz[t * DV + col]));
        }
      }
    }
    __syncthreads();  // the chunk buffers are refilled next
  }
#pragma unroll
  for (int r = 0; r < 16; r++) *reinterpret_cast<float4*>(Sh + (size_t)(rg + 8 * r) * DV) = s[r];
}

// Gated RMSNorm (model.rs:377-383) of the chunked prefill's outputs: o (f32, written over the v columns of act)
// * rsqrt(mean o^2 + eps) * w * silu(z) -> X2 planes. One warp per (row, value head), four columns per lane.
__global__ void __launch_bounds__(256) gdn_gated_norm_kernel(const float* __restrict__ act, YView y, int ldy, int R,
                                                             int conv_dim, int key_dim, int hv,
                                                             const float* __restrict__ norm_w, float eps,
                                                             __nv_bfloat16* __restrict__ X2, size_t xplane, int vd) {
  pdl_trigger();
  pdl_wait();
  constexpr int DV = 128;
  const int pair = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (pair >= R * hv) return;  // whole warps leave together
  const int row = pair / hv, head = pair % hv, c = lane * 4;
  const float4 o = *reinterpret_cast<const float4*>(act + (size_t)row * conv_dim + 2 * key_dim + head * DV + c);
  const float4 z = y.at4((size_t)row * ldy + conv_dim + head * DV + c);
  const float4 w = *reinterpret_cast<const float4*>(norm_w + c);
  float ss = o.x * o.x + o.y * o.y + o.z * o.z + o.w * o.w;
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  const float inv = 1.0f / sqrtf(ss / (float)DV + eps);
  store_split4(X2, xplane, (size_t)row * vd + head * DV + c,
               make_float4(o.x * inv * w.x * siluf_(z.x), o.y * inv * w.y * siluf_(z.y),
                           o.z * inv * w.z * siluf_(z.z), o.w * inv * w.w * siluf_(z.w)));
}

// model.rs:419-442, rope model.rs:470-479: q_norm / k_norm (gains 1+w) + rotate-half RoPE on the first `rot` dims;
// K and V appended to the paged cache. One CTA per (row, head) with one thread per head dim (hd = 256).
template <typename KV>
__global__ void __launch_bounds__(256) attn_prep_kernel(YView y, int ldy,
                                                        const RowInfo* __restrict__ rows,
                                                        const float* __restrict__ q_norm,
                                                        const float* __restrict__ k_norm,
                                                        const float* __restrict__ inv_freq, int nh, int nkv, int hd,
                                                        int rot, float eps, float* __restrict__ q_rot, KV* __restrict__ kc,
                                                        KV* __restrict__ vc, const int* __restrict__ page_table,
                                                        int pages_per_slot, int page_size) {
  pdl_trigger();
  pdl_wait();
  __shared__ float red[8];
  __shared__ float yn_s[256];
  const int idx = blockIdx.x, r = blockIdx.y, d = threadIdx.x;
  const RowInfo ri = rows[r];
  const bool is_q = idx < nh;
  const int kh = idx - nh;
  const size_t base = (size_t)r * ldy;
  const float raw = is_q ? y.at(base + (size_t)idx * 2 * hd + d)
                         : y.at(base + (size_t)2 * nh * hd + (size_t)kh * hd + d);
  const float ss = block_sum<256>(raw * raw, red);
  const float inv = 1.0f / sqrtf(ss / (float)hd + eps);
  const float yn = raw * inv * (is_q ? q_norm[d] : k_norm[d]);
  yn_s[d] = yn;
  __syncthreads();
  float out = yn;
  const int half = rot / 2;
  if (d < rot) {
    const int i = d < half ? d : d - half;
    float sn, cs;
    sincosf((float)ri.pos * inv_freq[i], &sn, &cs);
    out = d < half ? yn_s[d] * cs - yn_s[d + half] * sn : yn_s[d] * cs + yn_s[d - half] * sn;
  }
  if (is_q) {
    q_rot[((size_t)r * nh + idx) * hd + d] = out;
  } else {
    const int page = page_table[(size_t)ri.slot * pages_per_slot + ri.pos / page_size];
    const size_t off = (((size_t)page * nkv + kh) * page_size + ri.pos % page_size) * hd + d;
    const float v = y.at(base + (size_t)2 * nh * hd + (size_t)nkv * hd + (size_t)kh * hd + d);
    if constexpr (sizeof(KV) == 2) {
      kc[off] = __float2bfloat16_rn(out);
      vc[off] = __float2bfloat16_rn(v);
    } else {
      kc[off] = out;
      vc[off] = v;
    }
  }
}

// The same prep with one warp per (row, head) for head dim 256 and 64 rotary dims: lane l holds dims 8 l .. 8 l + 7
// (two float4 per vector), so the head norm reduces with shuffles and no CTA barrier. The sum of squares follows
// block_sum<256>'s order bit for bit: there dim d sits in lane d % 32 of warp d / 32 and the butterfly pairs lanes
// i ^ 16, i ^ 8, i ^ 4, i ^ 2, i ^ 1; here dim d is element d % 8 of lane d / 8, so the first two levels are lane xors
// 2 and 1 and the last three are inside the lane; the eight warp sums are then added in warp order. RoPE's partner of
// dim d (d + 32 or d - 32) is the same element of lane l ^ 4. Outputs equal attn_prep_kernel's.
__global__ void __launch_bounds__(256) attn_prep_warp_kernel(YView y, int ldy, int R,
                                                             const RowInfo* __restrict__ rows,
                                                             const float* __restrict__ q_norm,
                                                             const float* __restrict__ k_norm,
                                                             const float* __restrict__ inv_freq, int nh, int nkv,
                                                             float eps, float* __restrict__ q_rot,
                                                             __nv_bfloat16* __restrict__ kc,
                                                             __nv_bfloat16* __restrict__ vc,
                                                             const int* __restrict__ page_table, int pages_per_slot,
                                                             int page_size) {
  pdl_trigger();
  pdl_wait();
  constexpr int HD = 256, HALF = 32;
  const int lane = threadIdx.x & 31;
  const long u = (long)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int heads = nh + nkv;
  if (u >= (long)R * heads) return;  // the whole warp leaves together
  const int r = (int)(u / heads), idx = (int)(u % heads);
  const bool is_q = idx < nh;
  const int kh = idx - nh;
  const int d0 = lane * 8;
  const size_t base = (size_t)r * ldy;
  const size_t src = is_q ? base + (size_t)idx * 2 * HD : base + (size_t)2 * nh * HD + (size_t)kh * HD;
  float x[8];
  {
    const float4 a = y.at4_few(src + d0), b = y.at4_few(src + d0 + 4);
    x[0] = a.x, x[1] = a.y, x[2] = a.z, x[3] = a.w, x[4] = b.x, x[5] = b.y, x[6] = b.z, x[7] = b.w;
  }
  float4 va = make_float4(0.f, 0.f, 0.f, 0.f), vb = va;
  if (!is_q) {  // issued with the other loads
    const size_t vs = base + (size_t)2 * nh * HD + (size_t)nkv * HD + (size_t)kh * HD + d0;
    va = y.at4_few(vs);
    vb = y.at4_few(vs + 4);
  }
  const RowInfo ri = rows[r];
  float s[8];
#pragma unroll
  for (int e = 0; e < 8; e++) s[e] = x[e] * x[e];
#pragma unroll
  for (int e = 0; e < 8; e++) s[e] += __shfl_xor_sync(0xffffffffu, s[e], 2);  // block_sum's xor 16
#pragma unroll
  for (int e = 0; e < 8; e++) s[e] += __shfl_xor_sync(0xffffffffu, s[e], 1);  // xor 8
#pragma unroll
  for (int m = 4; m >= 1; m >>= 1) {  // xor 4, 2, 1
    float t[8];
#pragma unroll
    for (int e = 0; e < 8; e++) t[e] = s[e] + s[e ^ m];
#pragma unroll
    for (int e = 0; e < 8; e++) s[e] = t[e];
  }
  float ss = 0.f;  // the eight warp sums of block_sum, in warp order
#pragma unroll
  for (int w = 0; w < 8; w++) ss += __shfl_sync(0xffffffffu, s[0], 4 * w);
  const float inv = 1.0f / sqrtf(ss / (float)HD + eps);
  const float* nw = (is_q ? q_norm : k_norm) + d0;
  float yn[8], out[8];
#pragma unroll
  for (int e = 0; e < 8; e++) yn[e] = x[e] * inv * nw[e];
  float pr[8];  // the rotary partner of each dim (lanes 0-7)
#pragma unroll
  for (int e = 0; e < 8; e++) pr[e] = __shfl_xor_sync(0xffffffffu, yn[e], 4);
#pragma unroll
  for (int e = 0; e < 8; e++) out[e] = yn[e];
  if (lane < 8) {  // dims below 2 HALF = 64
#pragma unroll
    for (int e = 0; e < 8; e++) {
      const int d = d0 + e;
      const int i = d < HALF ? d : d - HALF;
      float sn, cs;
      sincosf((float)ri.pos * inv_freq[i], &sn, &cs);
      out[e] = d < HALF ? yn[e] * cs - pr[e] * sn : yn[e] * cs + pr[e] * sn;
    }
  }
  if (is_q) {
    float4* q4 = reinterpret_cast<float4*>(q_rot + ((size_t)r * nh + idx) * HD + d0);
    q4[0] = make_float4(out[0], out[1], out[2], out[3]);
    q4[1] = make_float4(out[4], out[5], out[6], out[7]);
  } else {
    const int page = page_table[(size_t)ri.slot * pages_per_slot + ri.pos / page_size];
    const size_t off = (((size_t)page * nkv + kh) * page_size + ri.pos % page_size) * HD + d0;
    const auto pack = [](float a, float b) {  // two bf16, round to nearest even, a in the low half
      const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
      return *reinterpret_cast<const uint32_t*>(&h);
    };
    *reinterpret_cast<uint4*>(kc + off) =
        make_uint4(pack(out[0], out[1]), pack(out[2], out[3]), pack(out[4], out[5]), pack(out[6], out[7]));
    *reinterpret_cast<uint4*>(vc + off) = make_uint4(pack(va.x, va.y), pack(va.z, va.w), pack(vb.x, vb.y),
                                                     pack(vb.z, vb.w));
  }
}

// silu(g) * u with the product rounded on its own, so that the gate detectors (which recompute a few of these
// activations) see exactly the values the SwiGLU kernel steers and captures.
__device__ __forceinline__ float swiglu_act(float g, float u) { return __fmul_rn(siluf_(g), u); }

// model.rs:249-258 with the Probe hook (worker.rs:136-141): silu(gate) * up, the slot's steering ops of this layer
// in order (steering.rs:189-208), companded capture (worker.rs:97-112) and max |a| over positions > 0
// (gpu/mod.rs:577-593). One CTA = one row x 1024 neurons.
__global__ void __launch_bounds__(256) swiglu_kernel(YView y, int ldy,
                                                     const RowInfo* __restrict__ rows, int layer, int n, int L,
                                                     SteerTables steer, const float* __restrict__ scale,
                                                     int8_t* __restrict__ frames, uint32_t* __restrict__ maxbuf,
                                                     __nv_bfloat16* __restrict__ X2, size_t xplane) {
  pdl_trigger();
  pdl_wait();
  __shared__ evie_op s_ops[64];
  __shared__ int s_cnt;
  const int r = blockIdx.y;
  const int j0 = blockIdx.x * 1024 + threadIdx.x * 4;  // n is a multiple of 4
  const bool active = j0 < n;
  const size_t yr = (size_t)r * ldy;
  float4 g4 = make_float4(0.f, 0.f, 0.f, 0.f), u4 = g4, sc = g4;
  if (active) {  // issued before the row and steering lookups, which then overlap these loads
    g4 = y.at4_few(yr + j0);
    u4 = y.at4_few(yr + n + j0);
    if (frames) sc = *reinterpret_cast<const float4*>(scale + (size_t)layer * n + j0);
  }
  const RowInfo ri = rows[r];
  if (threadIdx.x == 0) {
    const int* rg = steer.range + ((size_t)ri.slot * L + layer) * 2;
    s_cnt = min(rg[1], 64);
  }
  __syncthreads();
  const int cnt = s_cnt;
  if (threadIdx.x < cnt) {
    const int first = steer.range[((size_t)ri.slot * L + layer) * 2];
    const size_t oi = (size_t)ri.slot * steer.max_ops + first + threadIdx.x;
    evie_op op = steer.ops[oi];
    const int g = steer.op_gate[oi];
    if (g >= 0) {  // steering.rs:190-199: closed -> skip; opened in this call -> from the trigger row at/after its layer
      const size_t gi = (size_t)ri.slot * steer.max_gates + g;
      const bool on = steer.open[gi] && (layer < steer.gates[gi].last_layer || ri.pos >= steer.from[gi]);
      if (!on) op.mode = 0;
    }
    s_ops[threadIdx.x] = op;
  }
  __syncthreads();
  if (!active) return;
  float a[4] = {swiglu_act(g4.x, u4.x), swiglu_act(g4.y, u4.y), swiglu_act(g4.z, u4.z), swiglu_act(g4.w, u4.w)};
  for (int i = 0; i < cnt; i++) {  // steering.rs:189-208, in the slot's order
    const evie_op op = s_ops[i];
    const int e = op.neuron - j0;
    if (e < 0 || e > 3) continue;
    if (op.mode == 1) a[e] += op.value;
    else if (op.mode == 2) a[e] *= op.value;
    else if (op.mode == 3) a[e] = op.value;
  }
  store_split4(X2, xplane, (size_t)r * n + j0, make_float4(a[0], a[1], a[2], a[3]));
  if (frames) {
    const uint32_t packed = (uint32_t)(uint8_t)compand(a[0] / sc.x) | ((uint32_t)(uint8_t)compand(a[1] / sc.y) << 8) |
                            ((uint32_t)(uint8_t)compand(a[2] / sc.z) << 16) |
                            ((uint32_t)(uint8_t)compand(a[3] / sc.w) << 24);
    *reinterpret_cast<uint32_t*>(frames + ((size_t)r * L + layer) * n + j0) = packed;
  }
  if (maxbuf && ri.pos > 0)
#pragma unroll
    for (int e = 0; e < 4; e++) atomicMax(maxbuf + (size_t)layer * n + j0 + e, __float_as_uint(fabsf(a[e])));
}

// The same step for RPC consecutive rows per CTA (many-row calls): every thread issues the gate and up loads of all
// its rows first, then the rows' steering lookups run once per CTA (thread i < RPC reads row i's RowInfo and op
// range; then 64 threads per row load its ops), so a CTA keeps RPC rows' inputs in flight behind one lookup chain
// (4 rows against 1: 39.0 against 40.9 ms per 4B prefill call, measured with the plane-summing loads; with ONE the
// kernel takes ~18 ms). ONE: a single input plane, read by plain float4 loads. Per row and neuron: the same
// activation, ops in the slot's order, capture and max as swiglu_kernel, bit for bit.
template <int RPC, bool ONE>
__global__ void __launch_bounds__(256) swiglu_rows_kernel(YView y, int ldy, const RowInfo* __restrict__ rows, int R,
                                                          int layer, int n, int L, SteerTables steer,
                                                          const float* __restrict__ scale,
                                                          int8_t* __restrict__ frames, uint32_t* __restrict__ maxbuf,
                                                          __nv_bfloat16* __restrict__ X2, size_t xplane) {
  static_assert(RPC * 64 <= 256, "one op-loading thread per (row, op)");
  pdl_trigger();
  pdl_wait();
  __shared__ evie_op s_ops[RPC][64];
  __shared__ int s_cnt[RPC], s_first[RPC], s_slot[RPC], s_pos[RPC];
  const int r0 = blockIdx.y * RPC;
  const int nr = min(RPC, R - r0);
  const int j0 = blockIdx.x * 1024 + threadIdx.x * 4;
  const bool active = j0 < n;
  float4 g4[RPC], u4[RPC], sc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int i = 0; i < RPC; i++) {
    g4[i] = u4[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (active && i < nr) {
      const size_t yr = (size_t)(r0 + i) * ldy;
      g4[i] = ONE ? *reinterpret_cast<const float4*>(y.p + yr + j0) : y.at4(yr + j0);
      u4[i] = ONE ? *reinterpret_cast<const float4*>(y.p + yr + n + j0) : y.at4(yr + n + j0);
    }
  }
  if (active && frames) sc = *reinterpret_cast<const float4*>(scale + (size_t)layer * n + j0);
  if (threadIdx.x < nr) {
    const RowInfo ri = rows[r0 + threadIdx.x];
    const int* rg = steer.range + ((size_t)ri.slot * L + layer) * 2;
    s_first[threadIdx.x] = rg[0];
    s_cnt[threadIdx.x] = min(rg[1], 64);
    s_slot[threadIdx.x] = ri.slot;
    s_pos[threadIdx.x] = ri.pos;
  }
  __syncthreads();
  {
    const int i = threadIdx.x >> 6, k = threadIdx.x & 63;
    if (i < nr && k < s_cnt[i]) {
      const int slot = s_slot[i];
      const size_t oi = (size_t)slot * steer.max_ops + s_first[i] + k;
      evie_op op = steer.ops[oi];
      const int g = steer.op_gate[oi];
      if (g >= 0) {  // steering.rs:190-199: closed -> skip; opened in this call -> from the trigger row at/after its layer
        const size_t gi = (size_t)slot * steer.max_gates + g;
        const bool on = steer.open[gi] && (layer < steer.gates[gi].last_layer || s_pos[i] >= steer.from[gi]);
        if (!on) op.mode = 0;
      }
      s_ops[i][k] = op;
    }
  }
  __syncthreads();
  if (!active) return;
#pragma unroll
  for (int i = 0; i < RPC; i++) {
    if (i >= nr) break;
    const int r = r0 + i;
    float a[4] = {swiglu_act(g4[i].x, u4[i].x), swiglu_act(g4[i].y, u4[i].y), swiglu_act(g4[i].z, u4[i].z),
                  swiglu_act(g4[i].w, u4[i].w)};
    const int cnt = s_cnt[i];
    for (int k = 0; k < cnt; k++) {  // steering.rs:189-208, in the slot's order
      const evie_op op = s_ops[i][k];
      const int e = op.neuron - j0;
      if (e < 0 || e > 3) continue;
      if (op.mode == 1) a[e] += op.value;
      else if (op.mode == 2) a[e] *= op.value;
      else if (op.mode == 3) a[e] = op.value;
    }
    store_split4(X2, xplane, (size_t)r * n + j0, make_float4(a[0], a[1], a[2], a[3]));
    if (frames) {
      const uint32_t packed = (uint32_t)(uint8_t)compand(a[0] / sc.x) | ((uint32_t)(uint8_t)compand(a[1] / sc.y) << 8) |
                              ((uint32_t)(uint8_t)compand(a[2] / sc.z) << 16) |
                              ((uint32_t)(uint8_t)compand(a[3] / sc.w) << 24);
      *reinterpret_cast<uint32_t*>(frames + ((size_t)r * L + layer) * n + j0) = packed;
    }
    if (maxbuf && s_pos[i] > 0)
#pragma unroll
      for (int e = 0; e < 4; e++) atomicMax(maxbuf + (size_t)layer * n + j0 + e, __float_as_uint(fabsf(a[e])));
  }
}
constexpr int kSwigluRows = 4;


// steering.rs:164-187 for one segment (= one sequence and its slot's plan). Each thread owns rows: the gates whose
// first detector layer is this one restart at 0, then the layer's detector terms are added in plan order
// (p += w * a, each step rounded as the reference's f32 arithmetic). Then, per gate deciding here, the score is the
// last row's sum and a closed gate latches at the first row whose sum exceeds the threshold.
__global__ void __launch_bounds__(256) gate_detect_kernel(YView y, int ldy, const SegInfo* __restrict__ segs,
                                                          int layer, int n, int L, GateTables t) {
  pdl_trigger();
  pdl_wait();
  __shared__ int s_min[8];
  const SegInfo sg = segs[blockIdx.x];
  const int sl = sg.slot;
  const int ng = t.n_gates[sl];
  if (ng == 0) return;
  const GateSpec* gs = t.gates + (size_t)sl * t.max_gates;
  const DetSpec* ds = t.dets + (size_t)sl * t.max_dets;
  const int d0 = t.det_range[((size_t)sl * L + layer) * 2];
  const int nd = t.det_range[((size_t)sl * L + layer) * 2 + 1];
  for (int i = threadIdx.x; i < sg.count; i += blockDim.x) {
    const int r = sg.start + i;
    float* p = t.partial + (size_t)r * t.max_gates;
    for (int g = 0; g < ng; g++)
      if (gs[g].first_layer == layer) p[g] = 0.0f;
    const size_t yr = (size_t)r * ldy;
    for (int k = 0; k < nd; k++) {
      const DetSpec d = ds[d0 + k];
      const float a = swiglu_act(y.at(yr + d.neuron), y.at(yr + n + d.neuron));
      p[d.gate] = __fadd_rn(p[d.gate], __fmul_rn(d.weight, a));
    }
  }
  __syncthreads();
  for (int g = 0; g < ng; g++) {
    const GateSpec spec = gs[g];
    if (spec.last_layer != layer) continue;
    const size_t gi = (size_t)sl * t.max_gates + g;
    const bool was_open = t.open[gi] != 0;
    int first = INT_MAX;  // rows are visited in increasing order, so a thread's first hit is its minimum
    if (!was_open)
      for (int i = threadIdx.x; i < sg.count; i += blockDim.x)
        if (t.partial[(size_t)(sg.start + i) * t.max_gates + g] > spec.threshold) {
          first = i;
          break;
        }
    first = __reduce_min_sync(0xffffffffu, first);
    if ((threadIdx.x & 31) == 0) s_min[threadIdx.x >> 5] = first;
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int w = 1; w < (int)(blockDim.x >> 5); w++) first = min(first, s_min[w]);
      t.score[gi] = t.partial[(size_t)(sg.start + sg.count - 1) * t.max_gates + g];
      if (was_open) {
        t.from[gi] = INT_MIN;
      } else if (first != INT_MAX) {
        t.open[gi] = 1;
        t.from[gi] = sg.pos0 + first;
      }
    }
    __syncthreads();
  }
}

__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t i) {
  uint32_t u = __float_as_uint(v == 0.0f ? 0.0f : v);  // -0 and +0 tie, as the reference compares them
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)u << 32) | (0xFFFFFFFFu - i);  // larger value first, then lower index
}

// kernels.rs:642-662 with k = 1 (sampling.rs:60-62): the first index of the maximum logit.
__global__ void __launch_bounds__(256) logits_argmax_kernel(YView L2, int nseg, int V,
                                                            float* __restrict__ logits,
                                                            unsigned long long* __restrict__ best) {
  pdl_trigger();
  pdl_wait();
  __shared__ unsigned long long red[8];
  const int s = blockIdx.y;
  unsigned long long key = 0;
  const int i0 = blockIdx.x * 1024 + threadIdx.x;
#pragma unroll
  for (int e = 0; e < 4; e++) {
    const int i = i0 + e * 256;
    if (i < V) {
      const float v = L2.at((size_t)s * V + i);
      if (logits) logits[(size_t)s * V + i] = v;
      const unsigned long long k = argmax_key(v, (uint32_t)i);
      key = k > key ? k : key;
    }
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    const unsigned long long o = __shfl_xor_sync(0xffffffffu, key, off);
    key = o > key ? o : key;
  }
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = key;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long k = red[0];
    for (int w = 1; w < 8; w++) k = red[w] > k ? red[w] : k;
    atomicMax(best + s, k);
  }
}

__global__ void argmax_finish_kernel(unsigned long long* best, uint32_t* next_tokens, int nseg) {
  pdl_trigger();
  pdl_wait();
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s >= nseg) return;
  next_tokens[s] = 0xFFFFFFFFu - (uint32_t)(best[s] & 0xFFFFFFFFull);
  best[s] = 0;
}

__global__ void advance_rows_kernel(RowInfo* rows, int nseq, const uint32_t* next) {
  pdl_trigger();
  pdl_wait();
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s >= nseq) return;
  rows[s].pos += 1;
  rows[s].token = (int)next[s];
}

}  // namespace

// Threads for the row-norm kernels: decode-sized calls (R <= 128) one float4 per thread up to 1024 threads, two
// beyond; many-row calls two float4 per thread above 320 threads. Measured per 4B call: the prefill add+norm at 320
// threads 13.0 against 16.5 ms at 640, while the decode step's 63 launches took 0.69 against 0.56 ms at 320.
static int norm_threads(int d, int R) {
  const int n4 = d / 4;
  const int t = n4 <= (R > 128 ? 320 : 1024) ? n4 : (n4 + 1) / 2;
  return (t + 31) / 32 * 32;
}

evie_status k_advance_rows(RowInfo* rows, int nseq, const uint32_t* next, cudaStream_t st) {
  EVIE_CUDA_TRY(launch_k(advance_rows_kernel, dim3((nseq + 127) / 128), dim3(128), 0, st, rows, nseq, next));
  EVIE_CHECK_LAUNCH("advance_rows_kernel");
  return EVIE_OK;
}

evie_status k_embed_norm(const RowInfo* rows, int R, const __nv_bfloat16* embed, float* x, const float* gain,
                         float eps, int d, __nv_bfloat16* X2, uint32_t* seen, int seen_words, cudaStream_t st) {
  if (R == 0) return EVIE_OK;
  EVIE_CUDA_TRY(launch_k(embed_norm_kernel, dim3(R), dim3(kNormThreads), 0, st, rows, embed, x, gain, eps, d, X2, (size_t)R * d, seen, seen_words));
  EVIE_CHECK_LAUNCH("embed_norm_kernel");
  return EVIE_OK;
}

evie_status k_add_norm(float* x, YView y, int ldy, int R, const float* gain, float eps, int d,
                       __nv_bfloat16* X2, uint16_t* resid, int cap_layer, int L, cudaStream_t st) {
  if (R == 0) return EVIE_OK;
  EVIE_CUDA_TRY(launch_k(add_norm_kernel, dim3(R), dim3(norm_threads(d, R)), 0, st, x, y, ldy, gain, eps, d, X2, (size_t)R * d, resid, cap_layer, L));
  EVIE_CHECK_LAUNCH("add_norm_kernel");
  return EVIE_OK;
}

evie_status k_add_final(float* x, YView y, int ldy, int R, const RowInfo* rows, const SegInfo* segs,
                        int nseg, const float* gain, float eps, int d, __nv_bfloat16* X2, uint16_t* resid,
                        int cap_layer, int L, cudaStream_t st) {
  if (R == 0) return EVIE_OK;
  EVIE_CUDA_TRY(launch_k(add_final_kernel, dim3(R), dim3(norm_threads(d, R)), 0, st, x, y, ldy, rows, segs, nseg, gain, eps, d, X2, resid, cap_layer,
                                                  L));
  EVIE_CHECK_LAUNCH("add_final_kernel");
  return EVIE_OK;
}

evie_status k_conv_silu_norm(YView y, int ldy, int R, const RowInfo* rows, const SegInfo* segs,
                             float* conv_state, size_t cs_slot, const float* conv_w, const ModelShape& s,
                             float* act, cudaStream_t st, bool update_window, int nseg, int max_seg_rows,
                             bool split_qk) {
  if (R == 0) return EVIE_OK;
  if (split_qk && !(max_seg_rows > 1 && s.K == 4 && !update_window && s.dk == 128))
    return fail(EVIE_ERR_ARG, "conv: split q/k output needs the 4-tap multi-row form with 128-wide key heads");
  const auto a16 = [](const void* p) { return ((uintptr_t)p & 15u) == 0; };
  const bool vec4 = s.K == 4 && s.conv_dim % 128 == 0 && ldy % 4 == 0 && y.plane % 4 == 0 && cs_slot % 4 == 0 &&
                    a16(y.p) && a16(conv_state) && a16(conv_w) && a16(act);
  if (max_seg_rows > 1 && vec4 && !update_window) {
    dim3 grid((s.conv_dim + 511) / 512, nseg, (max_seg_rows + kConvRows - 1) / kConvRows);
    auto* kern = y.n == 1 ? conv_rows4_kernel<true> : conv_rows4_kernel<false>;
    EVIE_CUDA_TRY(launch_k(kern, grid, dim3(128), 0, st, y, ldy, segs, conv_state, cs_slot, conv_w,
                           s.conv_dim, s.hk, 1.0f / sqrtf((float)s.dk), act, split_qk));
    EVIE_CHECK_LAUNCH("conv_rows4_kernel");
    return EVIE_OK;
  }
  if (max_seg_rows > 1 && s.K == 4 && !update_window) {
    dim3 grid(s.conv_dim / 128, nseg, (max_seg_rows + kConvRows - 1) / kConvRows);
    EVIE_CUDA_TRY(launch_k(conv_rows_kernel<4>, dim3(grid), dim3(128), 0, st, y, ldy, segs, conv_state, cs_slot, conv_w, s.conv_dim, s.hk,
                                              1.0f / sqrtf((float)s.dk), act, split_qk));
    EVIE_CHECK_LAUNCH("conv_rows_kernel");
    return EVIE_OK;
  }
  if (update_window && vec4) {
    dim3 grid((s.conv_dim + 511) / 512, R);
    EVIE_CUDA_TRY(launch_k(conv_decode4_kernel, dim3(grid), dim3(128), 0, st, y, ldy, rows, segs, conv_state, cs_slot, conv_w, s.conv_dim, s.hk,
                                              1.0f / sqrtf((float)s.dk), act));
    EVIE_CHECK_LAUNCH("conv_decode4_kernel");
    return EVIE_OK;
  }
  dim3 grid(s.conv_dim / 128, R);
  EVIE_CUDA_TRY(launch_k(conv_silu_norm_kernel, dim3(grid), dim3(128), 0, st, y, ldy, rows, segs, conv_state, cs_slot, conv_w, s.K,
                                              s.conv_dim, s.hk, 1.0f / sqrtf((float)s.dk), act, update_window));
  EVIE_CHECK_LAUNCH("conv_silu_norm_kernel");
  return EVIE_OK;
}

evie_status k_conv_state_update(YView y, int ldy, int R, const SegInfo* segs, int nseg, float* conv_state,
                                size_t cs_slot, const ModelShape& s, cudaStream_t st) {
  if (nseg == 0) return EVIE_OK;
  dim3 grid((s.conv_dim + 255) / 256, nseg);
  EVIE_CUDA_TRY(launch_k(conv_state_update_kernel, dim3(grid), dim3(256), 0, st, y, ldy, segs, conv_state, cs_slot, s.K,
                                                 s.conv_dim));
  EVIE_CHECK_LAUNCH("conv_state_update_kernel");
  return EVIE_OK;
}

evie_status k_gdn_mixer(const float* act, YView y, int ldy, int R, const SegInfo* segs, int nseg,
                        float* rec_state, size_t rs_slot, const float* neg_a, const float* dt_bias,
                        const float* norm_w, const ModelShape& s, __nv_bfloat16* X2, cudaStream_t st) {
  if (nseg == 0) return EVIE_OK;
  dim3 grid(s.hv, nseg);
  if (R > nseg) {  // some segment has several rows: the warp-local sequential kernel
    constexpr int kSmemSeq = (5 * kSeqChunk * 128 + 2 * kSeqChunk) * 4;
    EVIE_TRY(max_dynamic_smem((const void*)gdn_mixer_seq_kernel, kSmemSeq));
    EVIE_CUDA_TRY(launch_k(gdn_mixer_seq_kernel, dim3(grid), dim3(kMixThreads), kSmemSeq, st, act, y, ldy, segs, rec_state, rs_slot, neg_a, dt_bias,
                                                              norm_w, s.conv_dim, s.key_dim, s.vd, s.hv, s.hv / s.hk,
                                                              s.eps, X2, (size_t)R * s.vd));
    EVIE_CHECK_LAUNCH("gdn_mixer_seq_kernel");
    return EVIE_OK;
  }
  // decode: the persistent kernel (state of the next unit prefetched), unless EVIE_MIXER_PER_HEAD=1 keeps one CTA
  // per (segment, head)
  static const bool per_head = [] {
    const char* e = getenv("EVIE_MIXER_PER_HEAD");
    return e && e[0] == '1';
  }();
  // the staged inputs are bulk copies: 16-byte aligned rows and planes
  const bool staged = ldy % 4 == 0 && y.plane % 4 == 0 && s.conv_dim % 4 == 0 && ((uintptr_t)y.p & 15u) == 0 &&
                      ((uintptr_t)act & 15u) == 0 && y.n >= 1 && y.n <= YView::kMaxPlanes;
  if (!per_head && staged) {
    unsigned int* counter = device_timeout_counter();
    if (!counter) return fail(EVIE_ERR_CUDA, "device timeout counter unavailable");
    const int units = nseg * s.hv;
    const int ctas = std::min(units, 2 * sm_count());
    const int smem = kMixStateBytes + 2 * mix_stage_floats(y.n) * 4;
    EVIE_TRY(max_dynamic_smem((const void*)gdn_mixer_persist_kernel, smem));
    EVIE_CUDA_TRY(launch_k(gdn_mixer_persist_kernel, dim3(ctas), dim3(kMixThreads), smem, st, act, y, ldy,
                           segs, nseg, rec_state, rs_slot, neg_a, dt_bias, norm_w, s.conv_dim, s.key_dim, s.vd, s.hv,
                           s.hv / s.hk, s.eps, X2, (size_t)R * s.vd, counter));
    EVIE_CHECK_LAUNCH("gdn_mixer_persist_kernel");
    return EVIE_OK;
  }
  EVIE_CUDA_TRY(launch_k(gdn_mixer_kernel, dim3(grid), dim3(kMixThreads), 0, st, act, y, ldy, segs, rec_state, rs_slot, neg_a,
                                                 dt_bias, norm_w, s.conv_dim, s.key_dim, s.vd, s.hv, s.hv / s.hk, s.eps,
                                                 X2, (size_t)R * s.vd));
  EVIE_CHECK_LAUNCH("gdn_mixer_kernel");
  return EVIE_OK;
}

evie_status k_gdn_gated_norm(const float* act, YView y, int ldy, int R, const float* norm_w, const ModelShape& s,
                             __nv_bfloat16* X2, cudaStream_t st) {
  if (R == 0) return EVIE_OK;
  if (s.dv != 128) return fail(EVIE_ERR_ARG, "gated norm: value heads must be 128 wide");
  const long pairs = (long)R * s.hv;
  EVIE_CUDA_TRY(launch_k(gdn_gated_norm_kernel, dim3((unsigned)((pairs + 7) / 8)), dim3(256), 0, st, act, y, ldy, R,
                         s.conv_dim, s.key_dim, s.hv, norm_w, s.eps, X2, (size_t)R * s.vd, s.vd));
  EVIE_CHECK_LAUNCH("gdn_gated_norm_kernel");
  return EVIE_OK;
}

template <typename KV>
evie_status k_attn_prep(YView y, int ldy, int R, const RowInfo* rows, const float* q_norm,
                        const float* k_norm, const float* inv_freq, const ModelShape& s, float* q_rot, KV* kc,
                        KV* vc, const int* page_table, int pages_per_slot, int page_size, cudaStream_t st) {
  if (R == 0) return EVIE_OK;
  static const bool cta_form = [] {
    const char* e = getenv("EVIE_ATTN_PREP_CTA");
    return e && e[0] == '1';
  }();
  const auto a16 = [](const void* p) { return ((uintptr_t)p & 15u) == 0; };
  if constexpr (sizeof(KV) == 2) {
    if (!cta_form && s.hd == 256 && s.rot == 64 && ldy % 4 == 0 && y.plane % 4 == 0 && a16(y.p) && a16(q_rot) &&
        a16(kc) && a16(vc) && a16(q_norm) && a16(k_norm)) {
      const long warps = (long)R * (s.nh + s.nkv);
      EVIE_CUDA_TRY(launch_k(attn_prep_warp_kernel, dim3((unsigned)((warps + 7) / 8)), dim3(256), 0, st, y, ldy, R,
                             rows, q_norm, k_norm, inv_freq, s.nh, s.nkv, s.eps, q_rot, kc, vc, page_table,
                             pages_per_slot, page_size));
      EVIE_CHECK_LAUNCH("attn_prep_warp_kernel");
      return EVIE_OK;
    }
  }
  dim3 grid(s.nh + s.nkv, R);
  EVIE_CUDA_TRY(launch_k(attn_prep_kernel<KV>, dim3(grid), dim3(256), 0, st, y, ldy, rows, q_norm, k_norm, inv_freq, s.nh, s.nkv,
                                             s.hd, s.rot, s.eps, q_rot, kc, vc, page_table, pages_per_slot, page_size));
  EVIE_CHECK_LAUNCH("attn_prep_kernel");
  return EVIE_OK;
}
template evie_status k_attn_prep<__nv_bfloat16>(YView, int, int, const RowInfo*, const float*, const float*,
                                                const float*, const ModelShape&, float*, __nv_bfloat16*,
                                                __nv_bfloat16*, const int*, int, int, cudaStream_t);
template evie_status k_attn_prep<float>(YView, int, int, const RowInfo*, const float*, const float*,
                                        const float*, const ModelShape&, float*, float*, float*, const int*, int, int,
                                        cudaStream_t);

evie_status k_swiglu(YView y, int ldy, int R, const RowInfo* rows, int layer, const ModelShape& s,
                     SteerTables steer, const float* scale, int8_t* frames, uint32_t* maxbuf, __nv_bfloat16* X2,
                     cudaStream_t st) {
  if (R == 0) return EVIE_OK;
  // Many-row calls (prefill) take kSwigluRows rows per CTA unless EVIE_SWIGLU_ROWS=1; decode-sized calls keep one
  // row per CTA (more CTAs for few rows).
  static const int rpc = [] {
    const char* e = getenv("EVIE_SWIGLU_ROWS");
    return e && e[0] == '1' ? 1 : kSwigluRows;
  }();
  if (R > 128 && rpc > 1) {
    dim3 grid((s.n + 1023) / 1024, (R + kSwigluRows - 1) / kSwigluRows);
    auto* kern = y.n == 1 ? swiglu_rows_kernel<kSwigluRows, true> : swiglu_rows_kernel<kSwigluRows, false>;
    EVIE_CUDA_TRY(launch_k(kern, grid, dim3(256), 0, st, y, ldy, rows, R, layer, s.n, s.L, steer, scale, frames,
                           maxbuf, X2, (size_t)R * s.n));
    EVIE_CHECK_LAUNCH("swiglu_rows_kernel");
    return EVIE_OK;
  }
  dim3 grid((s.n + 1023) / 1024, R);
  EVIE_CUDA_TRY(launch_k(swiglu_kernel, dim3(grid), dim3(256), 0, st, y, ldy, rows, layer, s.n, s.L, steer, scale, frames, maxbuf,
                                      X2, (size_t)R * s.n));
  EVIE_CHECK_LAUNCH("swiglu_kernel");
  return EVIE_OK;
}

evie_status k_gate_detect(YView y, int ldy, const SegInfo* segs, int nseg, int layer, const ModelShape& s,
                          GateTables t, cudaStream_t st) {
  if (nseg == 0) return EVIE_OK;
  EVIE_CUDA_TRY(launch_k(gate_detect_kernel, dim3(nseg), dim3(256), 0, st, y, ldy, segs, layer, s.n, s.L, t));
  EVIE_CHECK_LAUNCH("gate_detect_kernel");
  return EVIE_OK;
}

evie_status k_logits_argmax(YView L2, int nseg, int V, float* logits, unsigned long long* best,
                            uint32_t* next_tokens, cudaStream_t st) {
  if (nseg == 0) return EVIE_OK;
  dim3 grid((V + 1023) / 1024, nseg);
  EVIE_CUDA_TRY(launch_k(logits_argmax_kernel, dim3(grid), dim3(256), 0, st, L2, nseg, V, logits, best));
  EVIE_CHECK_LAUNCH("logits_argmax_kernel");
  EVIE_CUDA_TRY(launch_k(argmax_finish_kernel, dim3((nseg + 127) / 128), dim3(128), 0, st, best, next_tokens, nseg));
  EVIE_CHECK_LAUNCH("argmax_finish_kernel");
  return EVIE_OK;
}

}  // namespace evie
