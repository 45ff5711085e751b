// Gated DeltaNet recurrent decode step (one token per head) for sm_100a.
//
// Semantics follow evie-core's recur_body (crates/evie-core/src/model.rs:501-524):
//   kv = S^T k;  delta = (v - decay * kv) * beta;  S <- decay * S + k delta^T;  o = S^T q  (o from the updated S)
// with decay = exp(g). The state S of a head is [dk][dv] fp32, row i = key index.
//
// Design (HBM-bound: 128 KiB of state traffic per head against ~7 flop/B of work):
//   * the columns of S evolve independently (delta_j only needs column j), so one CTA owns one head and
//     COLS = 32 of its dv columns: 4 CTAs per head, B*H*4 independent CTAs of 128 threads;
//   * a thread holds 8 rows x 4 columns of its slice in registers: the state is read exactly once and
//     written exactly once, with 128-byte coalesced float4 accesses (4 rows x 128 B per warp instruction);
//   * the two reductions over the key index (S^T k and S^T q) use warp shuffles across the 4 row groups
//     of a warp, then a 4-warp shared-memory stage.
#include "common.h"
#include "gdn_chunk.h"
#include "gdn_decode.h"

namespace evie {

namespace {

constexpr int kDK = 128, kDV = 128;
constexpr int kCols = 32;                  // dv columns per CTA
constexpr int kThreads = 128;
constexpr int kColLanes = kCols / 4;       // float4 lanes across the columns (8)
constexpr int kRowGroups = kThreads / kColLanes;  // 16
constexpr int kRowsPerThread = kDK / kRowGroups;  // 8
constexpr int kWarps = kThreads / 32;

template <typename T>
__device__ __forceinline__ float ld1(const T* p);
template <>
__device__ __forceinline__ float ld1<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }

template <typename T>
__global__ void __launch_bounds__(kThreads) gdn_decode_step_kernel(const T* __restrict__ q, const T* __restrict__ k,
                                                                   const T* __restrict__ v,
                                                                   const float* __restrict__ g,
                                                                   const float* __restrict__ beta,
                                                                   float* __restrict__ S, float* __restrict__ o) {
  const int head = blockIdx.x / (kDV / kCols);
  const int col0 = (blockIdx.x % (kDV / kCols)) * kCols;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int cl = tid % kColLanes, rg = tid / kColLanes;

  __shared__ float sq[kDK], sk[kDK];
  __shared__ float4 red_kv[kWarps][kColLanes], red_o[kWarps][kColLanes];

  float* Sh = S + (size_t)head * kDK * kDV + col0 + cl * 4;
  float4 s[kRowsPerThread];
#pragma unroll
  for (int r = 0; r < kRowsPerThread; r++) s[r] = ld_stream4(Sh + (size_t)(rg + r * kRowGroups) * kDV);

  sq[tid] = ld1(q + (size_t)head * kDK + tid);
  sk[tid] = ld1(k + (size_t)head * kDK + tid);
  const float decay = expf(g[head]);
  const float b = beta[head];
  float vv[4];
#pragma unroll
  for (int j = 0; j < 4; j++) vv[j] = ld1(v + (size_t)head * kDV + col0 + cl * 4 + j);
  __syncthreads();

  // kv = S^T k over this thread's rows, then across the row groups.
  float4 kv = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int r = 0; r < kRowsPerThread; r++) {
    const float kr = sk[rg + r * kRowGroups];
    kv.x += s[r].x * kr; kv.y += s[r].y * kr; kv.z += s[r].z * kr; kv.w += s[r].w * kr;
  }
#pragma unroll
  for (int off = kColLanes; off < 32; off <<= 1) {
    kv.x += __shfl_xor_sync(0xffffffffu, kv.x, off);
    kv.y += __shfl_xor_sync(0xffffffffu, kv.y, off);
    kv.z += __shfl_xor_sync(0xffffffffu, kv.z, off);
    kv.w += __shfl_xor_sync(0xffffffffu, kv.w, off);
  }
  if (lane < kColLanes) red_kv[warp][cl] = kv;
  __syncthreads();
  kv = red_kv[0][cl];
#pragma unroll
  for (int w = 1; w < kWarps; w++) {
    const float4 t = red_kv[w][cl];
    kv.x += t.x; kv.y += t.y; kv.z += t.z; kv.w += t.w;
  }
  const float d0 = (vv[0] - decay * kv.x) * b, d1 = (vv[1] - decay * kv.y) * b;
  const float d2 = (vv[2] - decay * kv.z) * b, d3 = (vv[3] - decay * kv.w) * b;

  // State update (written back once) and o = S_new^T q.
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int r = 0; r < kRowsPerThread; r++) {
    const int row = rg + r * kRowGroups;
    const float kr = sk[row], qr = sq[row];
    float4 n;
    n.x = s[r].x * decay + kr * d0; n.y = s[r].y * decay + kr * d1;
    n.z = s[r].z * decay + kr * d2; n.w = s[r].w * decay + kr * d3;
    st_stream4(Sh + (size_t)row * kDV, n);
    acc.x += n.x * qr; acc.y += n.y * qr; acc.z += n.z * qr; acc.w += n.w * qr;
  }
#pragma unroll
  for (int off = kColLanes; off < 32; off <<= 1) {
    acc.x += __shfl_xor_sync(0xffffffffu, acc.x, off);
    acc.y += __shfl_xor_sync(0xffffffffu, acc.y, off);
    acc.z += __shfl_xor_sync(0xffffffffu, acc.z, off);
    acc.w += __shfl_xor_sync(0xffffffffu, acc.w, off);
  }
  if (lane < kColLanes) red_o[warp][cl] = acc;
  __syncthreads();
  if (tid < kColLanes) {
    float4 t = red_o[0][cl];
#pragma unroll
    for (int w = 1; w < kWarps; w++) {
      const float4 u = red_o[w][cl];
      t.x += u.x; t.y += u.y; t.z += u.z; t.w += u.w;
    }
    *reinterpret_cast<float4*>(o + (size_t)head * kDV + col0 + cl * 4) = t;
  }
}

// Token-sequential prefill: the same step applied to T tokens in order with the state slice resident in
// registers, so the state is read once and written once per call. q,k,v: [B][T][H][d] bf16; g, beta:
// [B][T][H]; o: [B][T][H][dv] bf16. The next token's inputs are prefetched into registers during each step.
__global__ void __launch_bounds__(kThreads) gdn_prefill_seq_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k, const __nv_bfloat16* __restrict__ v,
    const float* __restrict__ g, const float* __restrict__ beta, float* __restrict__ S, __nv_bfloat16* __restrict__ o,
    int T, int H) {
  const int bh = blockIdx.x / (kDV / kCols);
  const int b = bh / H, h = bh % H;
  const int col0 = (blockIdx.x % (kDV / kCols)) * kCols;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int cl = tid % kColLanes, rg = tid / kColLanes;

  __shared__ float sq[2][kDK], sk[2][kDK];
  __shared__ float4 red_kv[2][kWarps][kColLanes], red_o[2][kWarps][kColLanes];

  float* Sh = S + (size_t)bh * kDK * kDV + col0 + cl * 4;
  float4 s[kRowsPerThread];
#pragma unroll
  for (int r = 0; r < kRowsPerThread; r++) s[r] = ld_stream4(Sh + (size_t)(rg + r * kRowGroups) * kDV);

  auto row_of = [&](int t) { return ((size_t)b * T + t) * H + h; };
  // prefetch registers for token t
  float pq = 0.f, pk = 0.f, pg = 0.f, pb = 0.f;
  float pv[4] = {0.f, 0.f, 0.f, 0.f};
  auto fetch = [&](int t) {
    const size_t row = row_of(t);
    pq = __bfloat162float(q[row * kDK + tid]);
    pk = __bfloat162float(k[row * kDK + tid]);
    pg = g[row];
    pb = beta[row];
#pragma unroll
    for (int j = 0; j < 4; j++) pv[j] = __bfloat162float(v[row * kDV + col0 + cl * 4 + j]);
  };
  if (T > 0) fetch(0);
  for (int t = 0; t < T; t++) {
    const int buf = t & 1;
    sq[buf][tid] = pq;
    sk[buf][tid] = pk;
    const float decay = expf(pg), bt = pb;
    const float v0 = pv[0], v1 = pv[1], v2 = pv[2], v3 = pv[3];
    if (t + 1 < T) fetch(t + 1);
    __syncthreads();
    float4 kv = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int r = 0; r < kRowsPerThread; r++) {
      const float kr = sk[buf][rg + r * kRowGroups];
      kv.x += s[r].x * kr; kv.y += s[r].y * kr; kv.z += s[r].z * kr; kv.w += s[r].w * kr;
    }
#pragma unroll
    for (int off = kColLanes; off < 32; off <<= 1) {
      kv.x += __shfl_xor_sync(0xffffffffu, kv.x, off);
      kv.y += __shfl_xor_sync(0xffffffffu, kv.y, off);
      kv.z += __shfl_xor_sync(0xffffffffu, kv.z, off);
      kv.w += __shfl_xor_sync(0xffffffffu, kv.w, off);
    }
    if (lane < kColLanes) red_kv[buf][warp][cl] = kv;
    __syncthreads();
    kv = red_kv[buf][0][cl];
#pragma unroll
    for (int w = 1; w < kWarps; w++) {
      const float4 u = red_kv[buf][w][cl];
      kv.x += u.x; kv.y += u.y; kv.z += u.z; kv.w += u.w;
    }
    const float d0 = (v0 - decay * kv.x) * bt, d1 = (v1 - decay * kv.y) * bt;
    const float d2 = (v2 - decay * kv.z) * bt, d3 = (v3 - decay * kv.w) * bt;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int r = 0; r < kRowsPerThread; r++) {
      const int row = rg + r * kRowGroups;
      const float kr = sk[buf][row], qr = sq[buf][row];
      s[r].x = s[r].x * decay + kr * d0; s[r].y = s[r].y * decay + kr * d1;
      s[r].z = s[r].z * decay + kr * d2; s[r].w = s[r].w * decay + kr * d3;
      acc.x += s[r].x * qr; acc.y += s[r].y * qr; acc.z += s[r].z * qr; acc.w += s[r].w * qr;
    }
#pragma unroll
    for (int off = kColLanes; off < 32; off <<= 1) {
      acc.x += __shfl_xor_sync(0xffffffffu, acc.x, off);
      acc.y += __shfl_xor_sync(0xffffffffu, acc.y, off);
      acc.z += __shfl_xor_sync(0xffffffffu, acc.z, off);
      acc.w += __shfl_xor_sync(0xffffffffu, acc.w, off);
    }
    if (lane < kColLanes) red_o[buf][warp][cl] = acc;
    __syncthreads();
    if (tid < kColLanes) {
      float4 u = red_o[buf][0][cl];
#pragma unroll
      for (int w = 1; w < kWarps; w++) {
        const float4 x = red_o[buf][w][cl];
        u.x += x.x; u.y += x.y; u.z += x.z; u.w += x.w;
      }
      __nv_bfloat162 lo = __floats2bfloat162_rn(u.x, u.y), hi = __floats2bfloat162_rn(u.z, u.w);
      uint2 pack;
      pack.x = *reinterpret_cast<uint32_t*>(&lo);
      pack.y = *reinterpret_cast<uint32_t*>(&hi);
      *reinterpret_cast<uint2*>(o + row_of(t) * kDV + col0 + cl * 4) = pack;
    }
  }
#pragma unroll
  for (int r = 0; r < kRowsPerThread; r++) st_stream4(Sh + (size_t)(rg + r * kRowGroups) * kDV, s[r]);
}

}  // namespace

evie_status launch_gdn_decode_step_bf16(const void* q, const void* k, const void* v, const float* g,
                                        const float* beta, float* state, float* o, int heads, cudaStream_t st) {
  if (heads == 0) return EVIE_OK;
  gdn_decode_step_kernel<__nv_bfloat16><<<heads * (kDV / kCols), kThreads, 0, st>>>(
      (const __nv_bfloat16*)q, (const __nv_bfloat16*)k, (const __nv_bfloat16*)v, g, beta, state, o);
  EVIE_CHECK_LAUNCH("gdn_decode_step_kernel");
  return EVIE_OK;
}

evie_status launch_gdn_prefill_seq_bf16(const void* q, const void* k, const void* v, const float* g,
                                        const float* beta, float* state, void* o, int B, int T, int H,
                                        cudaStream_t st) {
  if ((long)B * H == 0) return EVIE_OK;
  gdn_prefill_seq_kernel<<<B * H * (kDV / kCols), kThreads, 0, st>>>(
      (const __nv_bfloat16*)q, (const __nv_bfloat16*)k, (const __nv_bfloat16*)v, g, beta, state,
      (__nv_bfloat16*)o, T, H);
  EVIE_CHECK_LAUNCH("gdn_prefill_seq_kernel");
  return EVIE_OK;
}

}  // namespace evie

extern "C" evie_status evie_gdn_decode_step(const void* q, const void* k, const void* v, const float* g,
                                            const float* beta, float* state, float* o, int B, int H, int dk, int dv,
                                            void* stream) {
  EVIE_ARG(dk == 128 && dv == 128, "evie_gdn_decode_step: dk = dv = 128 required (got %d, %d)", dk, dv);
  EVIE_ARG(B >= 0 && H >= 0, "evie_gdn_decode_step: negative batch or heads");
  EVIE_ARG(q && k && v && g && beta && state && o || (long)B * H == 0, "evie_gdn_decode_step: null pointer");
  EVIE_ARG(((uintptr_t)state & 15) == 0 && ((uintptr_t)o & 15) == 0,
           "evie_gdn_decode_step: state and o must be 16-byte aligned");
  EVIE_ARG((long)B * H <= (1L << 26), "evie_gdn_decode_step: too many heads");
  return evie::launch_gdn_decode_step_bf16(q, k, v, g, beta, state, o, B * H, (cudaStream_t)stream);
}

extern "C" evie_status evie_gdn_chunk_prefill(const void* q, const void* k, const void* v, const float* g,
                                              const float* beta, float* state, void* o, int B, int T, int H, int dk,
                                              int dv, int chunk, void* stream) {
  EVIE_ARG(dk == 128 && dv == 128, "evie_gdn_chunk_prefill: dk = dv = 128 required (got %d, %d)", dk, dv);
  EVIE_ARG(chunk == 64, "evie_gdn_chunk_prefill: chunk must be 64 (got %d)", chunk);
  EVIE_ARG(B >= 0 && T >= 0 && H >= 0, "evie_gdn_chunk_prefill: negative size");
  EVIE_ARG((long)B * H * T == 0 || (q && k && v && g && beta && state && o), "evie_gdn_chunk_prefill: null pointer");
  EVIE_ARG((((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)state) & 15) == 0 && ((uintptr_t)o & 1) == 0,
           "evie_gdn_chunk_prefill: q, k, v and state must be 16-byte aligned, o 2-byte aligned");
  EVIE_ARG((long)B * H <= (1L << 31) - 1 && (long)B * T * H <= (1L << 40),
           "evie_gdn_chunk_prefill: too many heads or tokens");
  return evie::launch_gdn_chunk_prefill_bf16(q, k, v, g, beta, state, o, B, T, H, (cudaStream_t)stream);
}

extern "C" evie_status evie_gdn_prefill_tokenwise(const void* q, const void* k, const void* v, const float* g,
                                                  const float* beta, float* state, void* o, int B, int T, int H,
                                                  int dk, int dv, void* stream) {
  EVIE_ARG(dk == 128 && dv == 128, "evie_gdn_prefill_tokenwise: dk = dv = 128 required (got %d, %d)", dk, dv);
  EVIE_ARG(B >= 0 && T >= 0 && H >= 0, "evie_gdn_prefill_tokenwise: negative size");
  EVIE_ARG((long)B * H * T == 0 || (q && k && v && g && beta && state && o),
           "evie_gdn_prefill_tokenwise: null pointer");
  EVIE_ARG(((uintptr_t)state & 15) == 0 && ((uintptr_t)o & 7) == 0,
           "evie_gdn_prefill_tokenwise: state must be 16-byte and o 8-byte aligned");
  return evie::launch_gdn_prefill_seq_bf16(q, k, v, g, beta, state, o, B, T, H, (cudaStream_t)stream);
}
