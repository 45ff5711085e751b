// Gated GQA softmax attention, decode (one query row per sequence), over a paged bf16 KV cache, for sm_100a.
//
// Semantics follow the attention core of evie-core's Model::attention (crates/evie-core/src/model.rs:445-464):
//   scores_j = scale * q . k_j (j < ctx);  p = softmax(scores);  o = sum_j p_j v_j;  o *= sigmoid(gate)
// for every query head h, with KV head h / (Hq / Hkv) (model.rs:447).
//
// Design (HBM-bound: every K/V byte is read exactly once; ~4 flop per byte at GQA group 4):
//   * one CTA per (sequence b, KV head, split of kSplit tokens) serves all GROUP query heads of that KV head, so
//     K/V are streamed once, not GROUP times;
//   * a warp reads a token's 512-byte K (or V) row with one 16-byte load per lane (8 head dims per lane) —
//     fully coalesced, and kTokIter rows are in flight per lane before any use;
//   * q.k partial dots for kTokIter tokens x GROUP heads (= 32 values) are finished with one 31-shuffle
//     reduce-scatter, leaving one score per lane;
//   * the softmax of the split is exact (two passes over the scores held in shared memory); P.V accumulates
//     GROUP x 8 values per lane and is reduced across warps in shared memory;
//   * splits are merged in-kernel: every CTA publishes (m, l, O) for its split, takes a ticket with atomicAdd,
//     and the CTA that takes the last ticket combines them (no spin-wait, no second launch). A sequence that fits
//     one split writes its output directly.
#include <cstdlib>
#include <map>
#include <mutex>

#include "common.h"
#include "gdn_chunk.h"
#include "gqa_decode.h"
#include "model_kernels.h"
#include "mma_sync.h"
#include "tc.h"
#include "tmap.h"

namespace evie {

namespace {

constexpr int kHD = 256;
constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kSplit = 512;                   // tokens per CTA
constexpr int kTokPerWarp = kSplit / kWarps;  // 64
constexpr float kLog2e = 1.4426950408889634f;

// One lane's 8 consecutive head dims of a K or V row.
template <typename KV>
struct KVRow;
template <>
struct KVRow<__nv_bfloat16> {
  using Raw = uint4;
  __device__ __forceinline__ static void load(Raw& r, const __nv_bfloat16* p) {
    r = p ? *reinterpret_cast<const uint4*>(p) : make_uint4(0, 0, 0, 0);
  }
  __device__ __forceinline__ static void widen(const Raw& r, float* f) { bf16x8_to_f32(r, f); }
};
template <>
struct KVRow<float> {
  struct Raw {
    float4 a, b;
  };
  __device__ __forceinline__ static void load(Raw& r, const float* p) {
    if (p) {
      r.a = *reinterpret_cast<const float4*>(p);
      r.b = *reinterpret_cast<const float4*>(p + 4);
    } else {
      r.a = r.b = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  __device__ __forceinline__ static void widen(const Raw& r, float* f) {
    f[0] = r.a.x; f[1] = r.a.y; f[2] = r.a.z; f[3] = r.a.w; f[4] = r.b.x; f[5] = r.b.y; f[6] = r.b.z; f[7] = r.b.w;
  }
};

// Inputs/outputs of the isolated op: bf16 q and gate logits [B][Hq][hd], f32 out, caller's page table.
struct IsoIO {
  const __nv_bfloat16* q;
  const __nv_bfloat16* gate_logits;
  float* out;
  const int32_t* page_table;
  const int32_t* ctx_lens;
  int Hq, max_pages;
  __device__ __forceinline__ int ctx_of(int b) const { return ctx_lens[b]; }
  __device__ __forceinline__ const int32_t* page_row(int b) const { return page_table + (size_t)b * max_pages; }
  __device__ __forceinline__ void load_q(int b, int h, int lane, float* f) const { load_q8(b, h, lane * 8, f); }
  __device__ __forceinline__ void load_q8(int b, int h, int d0, float* f) const {
    bf16x8_to_f32(*reinterpret_cast<const uint4*>(q + ((size_t)b * Hq + h) * kHD + d0), f);
  }
  __device__ __forceinline__ float gate(int b, int h, int d) const {
    return __bfloat162float(gate_logits[((size_t)b * Hq + h) * kHD + d]);
  }
  __device__ __forceinline__ void store(int b, int h, int d, float v) const { out[((size_t)b * Hq + h) * kHD + d] = v; }
};

// Inputs/outputs inside the model: one query per row (ctx = pos + 1), f32 rotated q [R][nh][hd], gate logits
// from the q projection planes (per head [q | gate]), output written as the split operand of o_proj.
struct ModelIO {
  const float* q_rot;
  YView y;
  int ldy;
  __nv_bfloat16* X2;
  size_t xplane;
  const RowInfo* rows;
  const int* page_table;
  int pages_per_slot, Hq;
  __device__ __forceinline__ int ctx_of(int b) const { return rows[b].pos + 1; }
  __device__ __forceinline__ const int32_t* page_row(int b) const {
    return page_table + (size_t)rows[b].slot * pages_per_slot;
  }
  __device__ __forceinline__ void load_q(int b, int h, int lane, float* f) const { load_q8(b, h, lane * 8, f); }
  __device__ __forceinline__ void load_q8(int b, int h, int d0, float* f) const {
    const float4* p = reinterpret_cast<const float4*>(q_rot + ((size_t)b * Hq + h) * kHD + d0);
    const float4 a = p[0], c = p[1];
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = c.x; f[5] = c.y; f[6] = c.z; f[7] = c.w;
  }
  __device__ __forceinline__ float gate(int b, int h, int d) const {
    return y.at((size_t)b * ldy + (size_t)h * 2 * kHD + kHD + d);
  }
  __device__ __forceinline__ void store(int b, int h, int d, float v) const {
    store_split(X2, xplane, (size_t)b * Hq * kHD + (size_t)h * kHD + d, v);
  }
};

struct Scratch {
  float* o;        // [B][Hkv][max_splits][GROUP][HD] unnormalised split outputs
  float* ml;       // [B][Hkv][max_splits][GROUP][2]  split max (log2 domain) and sum
  int* tickets;    // [B][Hkv]
  int max_splits;
};

template <int GROUP, typename KV, class IO>
__global__ void __launch_bounds__(kThreads, 2)
    gqa_decode_kernel(IO io, const KV* __restrict__ kp, const KV* __restrict__ vp, int Hkv, int page_size,
                      int max_pages, float scale, Scratch scr) {
  pdl_trigger();
  pdl_wait();
  constexpr int kTokIter = 32 / GROUP;  // tokens per reduce-scatter round
  const int split = blockIdx.x;
  const int kvh = blockIdx.y;
  const int b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ctx = min(io.ctx_of(b), max_pages * page_size);
  const int n_splits = (ctx + kSplit - 1) / kSplit;
  const int t0 = split * kSplit;

  const int h0 = kvh * GROUP;  // first query head of this KV head
  if (ctx <= 0) {
    if (split == 0)
      for (int i = tid; i < GROUP * kHD; i += kThreads) io.store(b, h0 + i / kHD, i % kHD, 0.0f);
    return;
  }
  if (split >= n_splits) return;

  __shared__ float s_p[kSplit][GROUP];       // scores, then probabilities (token-major for broadcast reads)
  __shared__ float s_red[kWarps][GROUP][kHD];
  __shared__ float s_stat[kWarps][GROUP];
  __shared__ float s_m[GROUP], s_l[GROUP];
  __shared__ int s_last;

  // q for this KV head's query heads, 8 dims per lane, pre-scaled into the log2 domain.
  float qr[GROUP][8];
  {
    const float f = scale * kLog2e;
#pragma unroll
    for (int h = 0; h < GROUP; h++) {
      io.load_q(b, h0 + h, lane, qr[h]);
#pragma unroll
      for (int d = 0; d < 8; d++) qr[h][d] *= f;
    }
  }
  const int32_t* pt = io.page_row(b);
  auto row_ptr = [&](const KV* pages, int j) {
    const int page = pt[j / page_size];
    return pages + (((size_t)page * Hkv + kvh) * page_size + (j % page_size)) * kHD + lane * 8;
  };

  // ---- scores
  const int wt0 = t0 + warp * kTokPerWarp;
  for (int it = 0; it < kTokPerWarp; it += kTokIter) {
    typename KVRow<KV>::Raw kr[kTokIter];
#pragma unroll
    for (int t = 0; t < kTokIter; t++) {
      const int j = wt0 + it + t;
      KVRow<KV>::load(kr[t], j < ctx ? row_ptr(kp, j) : nullptr);
    }
    float vals[32];
#pragma unroll
    for (int t = 0; t < kTokIter; t++) {
      float kf[8];
      KVRow<KV>::widen(kr[t], kf);
#pragma unroll
      for (int h = 0; h < GROUP; h++) {
        float a = 0.f;
#pragma unroll
        for (int d = 0; d < 8; d++) a = fmaf(qr[h][d], kf[d], a);
        vals[t * GROUP + h] = a;
      }
    }
    // reduce-scatter: afterwards lane l holds the full sum of value index l
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
      const bool upper = (lane & off) != 0;
#pragma unroll
      for (int i = 0; i < off; i++) {
        const float send = upper ? vals[i] : vals[i + off];
        const float keep = upper ? vals[i + off] : vals[i];
        vals[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
      }
    }
    const int tl = it + lane / GROUP;  // token within the warp's range
    const int j = wt0 + tl;
    s_p[warp * kTokPerWarp + tl][lane % GROUP] = j < ctx ? vals[0] : -INFINITY;
  }
  __syncthreads();

  // ---- softmax over the split (max, exp2, sum), per query head
  {
    float mx[GROUP];
#pragma unroll
    for (int h = 0; h < GROUP; h++) mx[h] = -INFINITY;
    for (int t = tid; t < kSplit; t += kThreads)
#pragma unroll
      for (int h = 0; h < GROUP; h++) mx[h] = fmaxf(mx[h], s_p[t][h]);
#pragma unroll
    for (int h = 0; h < GROUP; h++) {
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], off));
      if (lane == 0) s_stat[warp][h] = mx[h];
    }
    __syncthreads();
    if (tid < GROUP) {
      float m = s_stat[0][tid];
      for (int w = 1; w < kWarps; w++) m = fmaxf(m, s_stat[w][tid]);
      s_m[tid] = m;
    }
    __syncthreads();
    float sm[GROUP];
#pragma unroll
    for (int h = 0; h < GROUP; h++) sm[h] = 0.f;
    for (int t = tid; t < kSplit; t += kThreads)
#pragma unroll
      for (int h = 0; h < GROUP; h++) {
        const float p = exp2f(s_p[t][h] - s_m[h]);
        s_p[t][h] = p;
        sm[h] += p;
      }
#pragma unroll
    for (int h = 0; h < GROUP; h++) {
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) sm[h] += __shfl_xor_sync(0xffffffffu, sm[h], off);
    }
    __syncthreads();  // everyone has read s_stat (max) before it is reused for sums
    if (lane == 0)
#pragma unroll
      for (int h = 0; h < GROUP; h++) s_stat[warp][h] = sm[h];
    __syncthreads();
    if (tid < GROUP) {
      float l = 0.f;
      for (int w = 0; w < kWarps; w++) l += s_stat[w][tid];
      s_l[tid] = l;
    }
  }

  // ---- P.V
  float acc[GROUP][8];
#pragma unroll
  for (int h = 0; h < GROUP; h++)
#pragma unroll
    for (int d = 0; d < 8; d++) acc[h][d] = 0.f;
  constexpr int kVIter = 8;
  for (int it = 0; it < kTokPerWarp; it += kVIter) {
    typename KVRow<KV>::Raw vr[kVIter];
#pragma unroll
    for (int t = 0; t < kVIter; t++) {
      const int j = wt0 + it + t;
      KVRow<KV>::load(vr[t], j < ctx ? row_ptr(vp, j) : nullptr);
    }
#pragma unroll
    for (int t = 0; t < kVIter; t++) {
      float vf[8];
      KVRow<KV>::widen(vr[t], vf);
      const int tl = warp * kTokPerWarp + it + t;
#pragma unroll
      for (int h = 0; h < GROUP; h++) {
        const float p = s_p[tl][h];
#pragma unroll
        for (int d = 0; d < 8; d++) acc[h][d] = fmaf(p, vf[d], acc[h][d]);
      }
    }
  }
#pragma unroll
  for (int h = 0; h < GROUP; h++) {
    float4* dst = reinterpret_cast<float4*>(&s_red[warp][h][lane * 8]);
    dst[0] = make_float4(acc[h][0], acc[h][1], acc[h][2], acc[h][3]);
    dst[1] = make_float4(acc[h][4], acc[h][5], acc[h][6], acc[h][7]);
  }
  __syncthreads();

  // ---- publish or finish
  constexpr int kOutPerThread = GROUP * kHD / kThreads;
  float osum[kOutPerThread];
#pragma unroll
  for (int i = 0; i < kOutPerThread; i++) {
    const int e = tid + i * kThreads;
    const int h = e / kHD, d = e % kHD;
    float a = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; w++) a += s_red[w][h][d];
    osum[i] = a;
  }
  if (n_splits == 1) {
#pragma unroll
    for (int i = 0; i < kOutPerThread; i++) {
      const int e = tid + i * kThreads;
      const int h = e / kHD, d = e % kHD;
      io.store(b, h0 + h, d, osum[i] / s_l[h] * sigmoidf_(io.gate(b, h0 + h, d)));
    }
    return;
  }
  const size_t bh = (size_t)b * Hkv + kvh;
  float* po = scr.o + (bh * scr.max_splits + split) * GROUP * kHD;
#pragma unroll
  for (int i = 0; i < kOutPerThread; i++) __stcg(po + tid + i * kThreads, osum[i]);
  if (tid < GROUP) {
    float* pml = scr.ml + ((bh * scr.max_splits + split) * GROUP + tid) * 2;
    __stcg(pml, s_m[tid]);
    __stcg(pml + 1, s_l[tid]);
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = atomicAdd(scr.tickets + bh, 1) == n_splits - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();

  // Last CTA of this (b, KV head): merge the splits. Per-split weights first (reuse s_p as scratch).
  float* s_w = &s_p[0][0];  // [GROUP][n_splits]  (n_splits <= kSplit)
  if (tid < GROUP) {
    const float* ml = scr.ml + (bh * scr.max_splits) * GROUP * 2;
    float M = -INFINITY;
    for (int s = 0; s < n_splits; s++) M = fmaxf(M, __ldcg(ml + ((size_t)s * GROUP + tid) * 2));
    float L = 0.f;
    for (int s = 0; s < n_splits; s++) {
      const float w = exp2f(__ldcg(ml + ((size_t)s * GROUP + tid) * 2) - M);
      s_w[tid * n_splits + s] = w;
      L += w * __ldcg(ml + ((size_t)s * GROUP + tid) * 2 + 1);
    }
    for (int s = 0; s < n_splits; s++) s_w[tid * n_splits + s] /= L;
  }
  __syncthreads();
  const float* pob = scr.o + bh * scr.max_splits * GROUP * kHD;
#pragma unroll
  for (int i = 0; i < kOutPerThread; i++) {
    const int e = tid + i * kThreads;
    const int h = e / kHD, d = e % kHD;
    float a = 0.f;
    for (int s = 0; s < n_splits; s++) a += s_w[h * n_splits + s] * __ldcg(pob + (size_t)s * GROUP * kHD + e);
    io.store(b, h0 + h, d, a * sigmoidf_(io.gate(b, h0 + h, d)));
  }
  if (tid == 0) scr.tickets[bh] = 0;  // ready for the next call
}


// ---------------------------------------------------------------------------------------------------------------
// Tensor-core variant for bf16 KV and GQA group 4 (every Qwen3.5 size): scores and P.V on mma.sync m16n8k16, with
// K and V loaded straight from HBM into the MMA operand registers by 16-byte loads. The 8 columns of each MMA are the
// 4 query heads x {hi, lo}: q (and later p) is split into two bf16 halves (x = hi + lo, 16 significant bits), so the
// products match an fp32 computation on the bf16 K/V to ~2^-16 while no MMA column is padding.
//   QK:  S^T[16 tokens][8] += K[16 tokens][16 dims] . Q^T[16 dims][8]     (16 MMAs per 16 tokens)
//   PV:  O^T[16 dims][8]   += V^T[16 dims][16 tokens] . P^T[16 tokens][8] (16 MMAs per 16 tokens)
// Head dims are permuted inside each MMA so that a lane's operand registers come from contiguous 16-byte runs:
//   QK k-block 2p+e, slots {2c,2c+1 | 2c+8,2c+9} <-> dims 32p + 8c + 4e + {0,1 | 2,3} (c = lane % 4);
//   PV half h, m-tile i, rows {g | g+8} <-> dims {128h + 16g + i | 128h + 16g + 8 + i}  (g = lane / 4),
//   so a lane's two 16-byte V loads of a token fill one 32-byte sector and each half reads whole sectors.
// One CTA = 8 warps x 64 tokens = one 512-token split of one (sequence, KV head); the softmax is exact per warp
// (two passes over its 64 scores held in registers), warps are merged in shared memory, splits as before.
constexpr int kMmaTiles = kTokPerWarp / 16;  // 4 tiles of 16 tokens per warp

template <class IO>
__global__ void __launch_bounds__(kThreads, 2)
    gqa_decode_mma_kernel(IO io, const __nv_bfloat16* __restrict__ kp, const __nv_bfloat16* __restrict__ vp, int Hkv,
                          int page_size, int max_pages, float scale, Scratch scr) {
  pdl_trigger();
  pdl_wait();
  constexpr int GROUP = 4;
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, c = lane & 3;
  const int ctx = min(io.ctx_of(b), max_pages * page_size);
  const int n_splits = (ctx + kSplit - 1) / kSplit;
  const int h0 = kvh * GROUP;
  if (ctx <= 0) {
    if (split == 0)
      for (int i = tid; i < GROUP * kHD; i += kThreads) io.store(b, h0 + i / kHD, i % kHD, 0.0f);
    return;
  }
  if (split >= n_splits) return;

  __shared__ __align__(16) __nv_bfloat16 sP[kWarps][8][16];
  __shared__ float sO[kWarps][GROUP][kHD];
  __shared__ float sM[kWarps][GROUP], sL[kWarps][GROUP];
  __shared__ float s_w[kWarps][GROUP];
  __shared__ float s_fin[GROUP][2];
  __shared__ int s_last;

  // Q^T fragments: column n = g is head g % 4, half g / 4 (0 = hi, 1 = lo), pre-scaled into the log2 domain.
  uint32_t qb0[16], qb1[16];
  {
    const int head = h0 + (g & 3);
    const bool lo = g >= 4;
    const float f = scale * kLog2e;
#pragma unroll
    for (int p = 0; p < 8; p++) {
      float v[8];
      io.load_q8(b, head, 32 * p + 8 * c, v);
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const float x = v[j] * f;
        v[j] = lo ? x - bf16_round(x) : x;
      }
#pragma unroll
      for (int e = 0; e < 2; e++) {
        qb0[2 * p + e] = pack_bf16x2(v[4 * e + 0], v[4 * e + 1]);
        qb1[2 * p + e] = pack_bf16x2(v[4 * e + 2], v[4 * e + 3]);
      }
    }
  }
  const int32_t* pt = io.page_row(b);
  auto row = [&](const __nv_bfloat16* pages, int j) {
    const int page = pt[j / page_size];
    return pages + (((size_t)page * Hkv + kvh) * page_size + (j % page_size)) * kHD;
  };
  const int wt0 = split * kSplit + warp * kTokPerWarp;

  // ---- scores: lane holds heads hh, hh+1 (hh = 2 (c & 1)) for tokens g and g+8 of each tile
  float sc[kMmaTiles][4];
#pragma unroll
  for (int t = 0; t < kMmaTiles; t++) {
    const int jA = wt0 + 16 * t + g, jB = jA + 8;
    const __nv_bfloat16* pa = jA < ctx ? row(kp, jA) : nullptr;
    const __nv_bfloat16* pb = jB < ctx ? row(kp, jB) : nullptr;
    uint4 ka[8], kb[8];
#pragma unroll
    for (int p = 0; p < 8; p++) {
      ka[p] = pa ? ldg_stream128(pa + 32 * p + 8 * c) : make_uint4(0, 0, 0, 0);
      kb[p] = pb ? ldg_stream128(pb + 32 * p + 8 * c) : make_uint4(0, 0, 0, 0);
    }
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int p = 0; p < 8; p++)
#pragma unroll
      for (int e = 0; e < 2; e++)
        mma_bf16_16816(acc, word_of(ka[p], 2 * e), word_of(kb[p], 2 * e), word_of(ka[p], 2 * e + 1),
                       word_of(kb[p], 2 * e + 1), qb0[2 * p + e], qb1[2 * p + e]);
#pragma unroll
    for (int i = 0; i < 4; i++) acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], 2);  // hi + lo columns
    sc[t][0] = jA < ctx ? acc[0] : -INFINITY;
    sc[t][1] = jA < ctx ? acc[1] : -INFINITY;
    sc[t][2] = jB < ctx ? acc[2] : -INFINITY;
    sc[t][3] = jB < ctx ? acc[3] : -INFINITY;
  }
  // ---- warp softmax statistics per head (lanes with equal c hold the same heads)
  float m0 = -INFINITY, m1 = -INFINITY;
#pragma unroll
  for (int t = 0; t < kMmaTiles; t++) {
    m0 = fmaxf(m0, fmaxf(sc[t][0], sc[t][2]));
    m1 = fmaxf(m1, fmaxf(sc[t][1], sc[t][3]));
  }
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, off));
    m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, off));
  }
  const float b0m = m0 == -INFINITY ? 0.f : m0, b1m = m1 == -INFINITY ? 0.f : m1;
  float l0 = 0.f, l1 = 0.f;
#pragma unroll
  for (int t = 0; t < kMmaTiles; t++) {
    sc[t][0] = exp2f(sc[t][0] - b0m);
    sc[t][1] = exp2f(sc[t][1] - b1m);
    sc[t][2] = exp2f(sc[t][2] - b0m);
    sc[t][3] = exp2f(sc[t][3] - b1m);
    l0 += sc[t][0] + sc[t][2];
    l1 += sc[t][1] + sc[t][3];
  }
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, off);
    l1 += __shfl_xor_sync(0xffffffffu, l1, off);
  }
  const int hh = 2 * (c & 1);
  if (g == 0 && c < 2) {
    sM[warp][hh] = m0;
    sM[warp][hh + 1] = m1;
    sL[warp][hh] = l0;
    sL[warp][hh + 1] = l1;
  }

  // ---- P.V in two halves of the head dims (32 accumulators per lane each)
#pragma unroll 1
  for (int half = 0; half < 2; half++) {
    float o[8][4];
#pragma unroll
    for (int i = 0; i < 8; i++) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
#pragma unroll
    for (int t = 0; t < kMmaTiles; t++) {
      const int base = wt0 + 16 * t;
      __syncwarp();
      {  // P^T into shared memory as [h'][token]: lanes c < 2 write the hi halves, c >= 2 the lo halves
        const int r0 = hh + (c >= 2 ? 4 : 0);
        float pv[4] = {sc[t][0], sc[t][1], sc[t][2], sc[t][3]};
        if (c >= 2)
#pragma unroll
          for (int i = 0; i < 4; i++) pv[i] -= bf16_round(pv[i]);
        sP[warp][r0][g] = __float2bfloat16_rn(pv[0]);
        sP[warp][r0 + 1][g] = __float2bfloat16_rn(pv[1]);
        sP[warp][r0][g + 8] = __float2bfloat16_rn(pv[2]);
        sP[warp][r0 + 1][g + 8] = __float2bfloat16_rn(pv[3]);
      }
      __syncwarp();
      const uint32_t pb0 = *reinterpret_cast<const uint32_t*>(&sP[warp][g][2 * c]);
      const uint32_t pb1 = *reinterpret_cast<const uint32_t*>(&sP[warp][g][2 * c + 8]);
      uint4 v[4][2];
#pragma unroll
      for (int tk = 0; tk < 4; tk++) {
        const int j = base + 2 * c + (tk & 1) + 8 * (tk >> 1);
        const __nv_bfloat16* pv = j < ctx ? row(vp, j) : nullptr;
#pragma unroll
        for (int r = 0; r < 2; r++)
          v[tk][r] = pv ? ldg_stream128(pv + 128 * half + 16 * g + 8 * r) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int i = 0; i < 8; i++) {
        const int wi = i >> 1;
        const uint32_t sel = (i & 1) ? 0x7632u : 0x5410u;
        const uint32_t a0 = __byte_perm(word_of(v[0][0], wi), word_of(v[1][0], wi), sel);
        const uint32_t a1 = __byte_perm(word_of(v[0][1], wi), word_of(v[1][1], wi), sel);
        const uint32_t a2 = __byte_perm(word_of(v[2][0], wi), word_of(v[3][0], wi), sel);
        const uint32_t a3 = __byte_perm(word_of(v[2][1], wi), word_of(v[3][1], wi), sel);
        mma_bf16_16816(o[i], a0, a1, a2, a3, pb0, pb1);
      }
    }
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
      for (int k = 0; k < 4; k++) o[i][k] += __shfl_xor_sync(0xffffffffu, o[i][k], 2);  // hi + lo columns
    if (c < 2) {
#pragma unroll
      for (int i = 0; i < 8; i++) {
        const int d0 = 128 * half + 16 * g + i, d1 = d0 + 8;
        sO[warp][hh][d0] = o[i][0];
        sO[warp][hh + 1][d0] = o[i][1];
        sO[warp][hh][d1] = o[i][2];
        sO[warp][hh + 1][d1] = o[i][3];
      }
    }
  }
  __syncthreads();

  // ---- merge the 8 warps of this split
  if (tid < GROUP) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; w++) M = fmaxf(M, sM[w][tid]);
    float L = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; w++) {
      const float wt = sM[w][tid] == -INFINITY ? 0.f : exp2f(sM[w][tid] - M);
      s_w[w][tid] = wt;
      L += wt * sL[w][tid];
    }
    s_fin[tid][0] = M;
    s_fin[tid][1] = L;
  }
  __syncthreads();
  constexpr int kOutPerThread = GROUP * kHD / kThreads;
  float osum[kOutPerThread];
#pragma unroll
  for (int i = 0; i < kOutPerThread; i++) {
    const int e = tid + i * kThreads;
    const int h = e / kHD, d = e % kHD;
    float a = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; w++) a += s_w[w][h] * sO[w][h][d];
    osum[i] = a;
  }
  if (n_splits == 1) {
#pragma unroll
    for (int i = 0; i < kOutPerThread; i++) {
      const int e = tid + i * kThreads;
      const int h = e / kHD, d = e % kHD;
      io.store(b, h0 + h, d, osum[i] / s_fin[h][1] * sigmoidf_(io.gate(b, h0 + h, d)));
    }
    return;
  }
  const size_t bh = (size_t)b * Hkv + kvh;
  float* po = scr.o + (bh * scr.max_splits + split) * GROUP * kHD;
#pragma unroll
  for (int i = 0; i < kOutPerThread; i++) __stcg(po + tid + i * kThreads, osum[i]);
  if (tid < GROUP) {
    float* pml = scr.ml + ((bh * scr.max_splits + split) * GROUP + tid) * 2;
    __stcg(pml, s_fin[tid][0]);
    __stcg(pml + 1, s_fin[tid][1]);
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = atomicAdd(scr.tickets + bh, 1) == n_splits - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  float* s_sw = &sO[0][0][0];  // [GROUP][n_splits] merge weights (n_splits <= 512 fits in sO)
  if (tid < GROUP) {
    const float* ml = scr.ml + (bh * scr.max_splits) * GROUP * 2;
    float M = -INFINITY;
    for (int s2 = 0; s2 < n_splits; s2++) M = fmaxf(M, __ldcg(ml + ((size_t)s2 * GROUP + tid) * 2));
    float L = 0.f;
    for (int s2 = 0; s2 < n_splits; s2++) {
      const float w = exp2f(__ldcg(ml + ((size_t)s2 * GROUP + tid) * 2) - M);
      s_sw[tid * n_splits + s2] = w;
      L += w * __ldcg(ml + ((size_t)s2 * GROUP + tid) * 2 + 1);
    }
    for (int s2 = 0; s2 < n_splits; s2++) s_sw[tid * n_splits + s2] /= L;
  }
  __syncthreads();
  const float* pob = scr.o + bh * scr.max_splits * GROUP * kHD;
#pragma unroll
  for (int i = 0; i < kOutPerThread; i++) {
    const int e = tid + i * kThreads;
    const int h = e / kHD, d = e % kHD;
    float a = 0.f;
    for (int s2 = 0; s2 < n_splits; s2++) a += s_sw[h * n_splits + s2] * __ldcg(pob + (size_t)s2 * GROUP * kHD + e);
    io.store(b, h0 + h, d, a * sigmoidf_(io.gate(b, h0 + h, d)));
  }
  if (tid == 0) scr.tickets[bh] = 0;
}

// The same tensor-core kernel with K and V streamed into shared memory by bulk copies. Each warp owns 64 tokens of
// the split, i.e. 4 K tiles and 4 V tiles of 16 tokens; a 16-token tile of one KV head is one contiguous 8 KB run of
// a page, so it arrives by one cp.async.bulk completing on the warp's mbarrier. The warp keeps three tiles in flight
// in a private 3-stage ring and refills a stage as soon as it has read it, so its next loads overlap the MMAs,
// the softmax and the P.V of the current tile (the register-fed kernel above has one tile in flight per warp and
// none while it computes). Tiles past the context are neither copied nor read; rows past the context inside the
// last tile are masked as before. 192 KB of ring per CTA (which also holds the warps' P.V results at the end): one
// CTA of 8 warps per SM.
constexpr int kTileBytes = 16 * kHD * 2;                  // 8 KB
constexpr int kStages = 3;                                // tiles in flight per warp
constexpr int kWarpRing = kStages * kTileBytes;           // 24 KB
constexpr int kRingBytes = kWarps * kWarpRing;            // 192 KB

template <class IO>
__global__ void __launch_bounds__(kThreads, 1)
    gqa_decode_bulk_kernel(IO io, const __nv_bfloat16* __restrict__ kp, const __nv_bfloat16* __restrict__ vp,
                           int Hkv, int page_size, int max_pages, float scale, Scratch scr,
                           unsigned int* timeouts) {
  pdl_trigger();
  pdl_wait();
  constexpr int GROUP = 4;
  extern __shared__ __align__(128) uint8_t ring_all[];
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, c = lane & 3;
  const int ctx = min(io.ctx_of(b), max_pages * page_size);
  const int n_splits = (ctx + kSplit - 1) / kSplit;
  const int h0 = kvh * GROUP;
  if (ctx <= 0) {
    if (split == 0)
      for (int i = tid; i < GROUP * kHD; i += kThreads) io.store(b, h0 + i / kHD, i % kHD, 0.0f);
    return;
  }
  if (split >= n_splits) return;

  __shared__ __align__(16) __nv_bfloat16 sP[kWarps][8][16];
  // a warp's [GROUP][kHD] P.V result goes into its own ring once its last tile has been read
  auto sO = [&](int w, int h) { return reinterpret_cast<float*>(ring_all + w * kWarpRing) + h * kHD; };
  __shared__ float sM[kWarps][GROUP], sL[kWarps][GROUP];
  __shared__ float s_w[kWarps][GROUP];
  __shared__ float s_fin[GROUP][2];
  __shared__ int s_last;
  __shared__ __align__(8) uint64_t s_bar[kWarps][kStages];

  const int32_t* pt = io.page_row(b);
  auto row = [&](const __nv_bfloat16* pages, int j) {
    const int page = pt[j / page_size];
    return pages + (((size_t)page * Hkv + kvh) * page_size + (j % page_size)) * kHD;
  };
  const int wt0 = split * kSplit + warp * kTokPerWarp;
  // valid tiles of this warp: the first nt K tiles, then the first nt V tiles (n = 0 .. 2 nt - 1)
  const int nt = min(kMmaTiles, max(0, (ctx - wt0 + 15) / 16));
  uint8_t* ring = ring_all + warp * kWarpRing;
  uint64_t* bar = s_bar[warp];
  if (lane == 0) {
    for (int i = 0; i < kStages; i++) tc::mbar_init(&bar[i], 1);
    tc::fence_barrier_init();
  }
  __syncwarp();
  bool ok = true;
  int issued = 0, consumed = 0;
  auto issue = [&](int n) {  // tile n into stage n % kStages (lane 0; the warp has finished reading that stage)
    if (!ok) return;
    const bool isv = n >= nt;
    const int base = wt0 + 16 * (isv ? n - nt : n);
    const int rows = min(16, ctx - base);
    if (lane == 0) {
      tc::fence_proxy_async();
      tc::mbar_arrive_expect_tx(&bar[n % kStages], (uint32_t)rows * kHD * 2);
      tc::bulk_load(ring + (n % kStages) * kTileBytes, row(isv ? vp : kp, base), (uint32_t)rows * kHD * 2,
                    &bar[n % kStages]);
    }
    issued = n + 1;
  };
  auto take = [&](int n) -> const uint8_t* {  // wait for tile n; its stage
    if (ok && !tc::mbar_wait(&bar[n % kStages], (n / kStages) & 1)) ok = false;
    if (ok) consumed = n + 1;
    return ring + (n % kStages) * kTileBytes;
  };
  for (int n = 0; n < kStages && n < 2 * nt; n++) issue(n);

  // Q^T fragments: column n = g is head g % 4, half g / 4 (0 = hi, 1 = lo), pre-scaled into the log2 domain.
  uint32_t qb0[16], qb1[16];
  {
    const int head = h0 + (g & 3);
    const bool lo = g >= 4;
    const float f = scale * kLog2e;
#pragma unroll
    for (int p = 0; p < 8; p++) {
      float v[8];
      io.load_q8(b, head, 32 * p + 8 * c, v);
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const float x = v[j] * f;
        v[j] = lo ? x - bf16_round(x) : x;
      }
#pragma unroll
      for (int e = 0; e < 2; e++) {
        qb0[2 * p + e] = pack_bf16x2(v[4 * e + 0], v[4 * e + 1]);
        qb1[2 * p + e] = pack_bf16x2(v[4 * e + 2], v[4 * e + 3]);
      }
    }
  }

  // ---- scores: lane holds heads hh, hh+1 (hh = 2 (c & 1)) for tokens g and g+8 of each tile
  float sc[kMmaTiles][4];
#pragma unroll
  for (int t = 0; t < kMmaTiles; t++) {
    const int jA = wt0 + 16 * t + g, jB = jA + 8;
    if (t < nt) {
      const uint8_t* tile = take(t);
      const bool va = jA < ctx, vb = jB < ctx;
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int p = 0; p < 8; p++) {
        const uint4 ka = va ? *reinterpret_cast<const uint4*>(tile + g * 512 + (32 * p + 8 * c) * 2)
                            : make_uint4(0, 0, 0, 0);
        const uint4 kb = vb ? *reinterpret_cast<const uint4*>(tile + (g + 8) * 512 + (32 * p + 8 * c) * 2)
                            : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int e = 0; e < 2; e++)
          mma_bf16_16816(acc, word_of(ka, 2 * e), word_of(kb, 2 * e), word_of(ka, 2 * e + 1), word_of(kb, 2 * e + 1),
                         qb0[2 * p + e], qb1[2 * p + e]);
      }
      __syncwarp();
      if (t + kStages < 2 * nt) issue(t + kStages);
#pragma unroll
      for (int i = 0; i < 4; i++) acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], 2);  // hi + lo columns
      sc[t][0] = va ? acc[0] : -INFINITY;
      sc[t][1] = va ? acc[1] : -INFINITY;
      sc[t][2] = vb ? acc[2] : -INFINITY;
      sc[t][3] = vb ? acc[3] : -INFINITY;
    } else {
      sc[t][0] = sc[t][1] = sc[t][2] = sc[t][3] = -INFINITY;
    }
  }
  // ---- warp softmax statistics per head (lanes with equal c hold the same heads)
  float m0 = -INFINITY, m1 = -INFINITY;
#pragma unroll
  for (int t = 0; t < kMmaTiles; t++) {
    m0 = fmaxf(m0, fmaxf(sc[t][0], sc[t][2]));
    m1 = fmaxf(m1, fmaxf(sc[t][1], sc[t][3]));
  }
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, off));
    m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, off));
  }
  const float b0m = m0 == -INFINITY ? 0.f : m0, b1m = m1 == -INFINITY ? 0.f : m1;
  float l0 = 0.f, l1 = 0.f;
#pragma unroll
  for (int t = 0; t < kMmaTiles; t++) {
    sc[t][0] = exp2f(sc[t][0] - b0m);
    sc[t][1] = exp2f(sc[t][1] - b1m);
    sc[t][2] = exp2f(sc[t][2] - b0m);
    sc[t][3] = exp2f(sc[t][3] - b1m);
    l0 += sc[t][0] + sc[t][2];
    l1 += sc[t][1] + sc[t][3];
  }
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, off);
    l1 += __shfl_xor_sync(0xffffffffu, l1, off);
  }
  const int hh = 2 * (c & 1);
  if (g == 0 && c < 2) {
    sM[warp][hh] = m0;
    sM[warp][hh + 1] = m1;
    sL[warp][hh] = l0;
    sL[warp][hh + 1] = l1;
  }

  // ---- P.V: both halves of the head dims per tile (the tile is read from shared memory once per half)
  float o[2][8][4];
#pragma unroll
  for (int h = 0; h < 2; h++)
#pragma unroll
    for (int i = 0; i < 8; i++) o[h][i][0] = o[h][i][1] = o[h][i][2] = o[h][i][3] = 0.f;
#pragma unroll 1
  for (int t = 0; t < nt; t++) {
    const int base = wt0 + 16 * t;
    __syncwarp();
    {  // P^T into shared memory as [h'][token]: lanes c < 2 write the hi halves, c >= 2 the lo halves
      const int r0 = hh + (c >= 2 ? 4 : 0);
      float pv[4] = {sc[0][0], sc[0][1], sc[0][2], sc[0][3]};
#pragma unroll
      for (int tt = 1; tt < kMmaTiles; tt++)
        if (tt == t) pv[0] = sc[tt][0], pv[1] = sc[tt][1], pv[2] = sc[tt][2], pv[3] = sc[tt][3];
      if (c >= 2)
#pragma unroll
        for (int i = 0; i < 4; i++) pv[i] -= bf16_round(pv[i]);
      sP[warp][r0][g] = __float2bfloat16_rn(pv[0]);
      sP[warp][r0 + 1][g] = __float2bfloat16_rn(pv[1]);
      sP[warp][r0][g + 8] = __float2bfloat16_rn(pv[2]);
      sP[warp][r0 + 1][g + 8] = __float2bfloat16_rn(pv[3]);
    }
    __syncwarp();
    const uint32_t pb0 = *reinterpret_cast<const uint32_t*>(&sP[warp][g][2 * c]);
    const uint32_t pb1 = *reinterpret_cast<const uint32_t*>(&sP[warp][g][2 * c + 8]);
    const uint8_t* tile = take(nt + t);
#pragma unroll
    for (int half = 0; half < 2; half++) {
      uint4 v[4][2];
#pragma unroll
      for (int tk = 0; tk < 4; tk++) {
        const int jl = 2 * c + (tk & 1) + 8 * (tk >> 1);
#pragma unroll
        for (int r = 0; r < 2; r++)
          v[tk][r] = base + jl < ctx
                         ? *reinterpret_cast<const uint4*>(tile + jl * 512 + (128 * half + 16 * g + 8 * r) * 2)
                         : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int i = 0; i < 8; i++) {
        const int wi = i >> 1;
        const uint32_t sel = (i & 1) ? 0x7632u : 0x5410u;
        const uint32_t a0 = __byte_perm(word_of(v[0][0], wi), word_of(v[1][0], wi), sel);
        const uint32_t a1 = __byte_perm(word_of(v[0][1], wi), word_of(v[1][1], wi), sel);
        const uint32_t a2 = __byte_perm(word_of(v[2][0], wi), word_of(v[3][0], wi), sel);
        const uint32_t a3 = __byte_perm(word_of(v[2][1], wi), word_of(v[3][1], wi), sel);
        mma_bf16_16816(o[half][i], a0, a1, a2, a3, pb0, pb1);
      }
    }
    __syncwarp();
    if (nt + t + kStages < 2 * nt) issue(nt + t + kStages);
  }
  // Every copy this warp issued has been waited for (consumed == issued). After a give-up the warp waits for the
  // outstanding ones once more, again bounded by kWaitNs; if that wait gives up too, a copy may still land in the
  // ring while the warp writes sO below or after the CTA exits, and this split's outputs are undefined (the call
  // already reports EVIE_ERR_TIMEOUT through the device counter).
  ok = __all_sync(0xffffffffu, ok);
  if (!ok) {
    for (int n = consumed; n < issued; n++) tc::mbar_wait(&bar[n % kStages], (n / kStages) & 1);
    if (lane == 0) atomicAdd(timeouts, 1u);
  }
#pragma unroll
  for (int half = 0; half < 2; half++) {
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
      for (int k = 0; k < 4; k++) o[half][i][k] += __shfl_xor_sync(0xffffffffu, o[half][i][k], 2);  // hi + lo
    if (c < 2) {
#pragma unroll
      for (int i = 0; i < 8; i++) {
        const int d0 = 128 * half + 16 * g + i, d1 = d0 + 8;
        sO(warp, hh)[d0] = o[half][i][0];
        sO(warp, hh + 1)[d0] = o[half][i][1];
        sO(warp, hh)[d1] = o[half][i][2];
        sO(warp, hh + 1)[d1] = o[half][i][3];
      }
    }
  }
  __syncthreads();

  // ---- merge the 8 warps of this split
  if (tid < GROUP) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; w++) M = fmaxf(M, sM[w][tid]);
    float L = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; w++) {
      const float wt = sM[w][tid] == -INFINITY ? 0.f : exp2f(sM[w][tid] - M);
      s_w[w][tid] = wt;
      L += wt * sL[w][tid];
    }
    s_fin[tid][0] = M;
    s_fin[tid][1] = L;
  }
  __syncthreads();
  constexpr int kOutPerThread = GROUP * kHD / kThreads;
  float osum[kOutPerThread];
#pragma unroll
  for (int i = 0; i < kOutPerThread; i++) {
    const int e = tid + i * kThreads;
    const int h = e / kHD, d = e % kHD;
    float a = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; w++) a += s_w[w][h] * sO(w, h)[d];
    osum[i] = a;
  }
  if (n_splits == 1) {
#pragma unroll
    for (int i = 0; i < kOutPerThread; i++) {
      const int e = tid + i * kThreads;
      const int h = e / kHD, d = e % kHD;
      io.store(b, h0 + h, d, osum[i] / s_fin[h][1] * sigmoidf_(io.gate(b, h0 + h, d)));
    }
    return;
  }
  const size_t bh = (size_t)b * Hkv + kvh;
  float* po = scr.o + (bh * scr.max_splits + split) * GROUP * kHD;
#pragma unroll
  for (int i = 0; i < kOutPerThread; i++) __stcg(po + tid + i * kThreads, osum[i]);
  if (tid < GROUP) {
    float* pml = scr.ml + ((bh * scr.max_splits + split) * GROUP + tid) * 2;
    __stcg(pml, s_fin[tid][0]);
    __stcg(pml + 1, s_fin[tid][1]);
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = atomicAdd(scr.tickets + bh, 1) == n_splits - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  float* s_sw = sO(0, 0);  // [GROUP][n_splits] merge weights (n_splits <= 512 fits in warp 0's ring)
  if (tid < GROUP) {
    const float* ml = scr.ml + (bh * scr.max_splits) * GROUP * 2;
    float M = -INFINITY;
    for (int s2 = 0; s2 < n_splits; s2++) M = fmaxf(M, __ldcg(ml + ((size_t)s2 * GROUP + tid) * 2));
    float L = 0.f;
    for (int s2 = 0; s2 < n_splits; s2++) {
      const float w = exp2f(__ldcg(ml + ((size_t)s2 * GROUP + tid) * 2) - M);
      s_sw[tid * n_splits + s2] = w;
      L += w * __ldcg(ml + ((size_t)s2 * GROUP + tid) * 2 + 1);
    }
    for (int s2 = 0; s2 < n_splits; s2++) s_sw[tid * n_splits + s2] /= L;
  }
  __syncthreads();
  const float* pob = scr.o + bh * scr.max_splits * GROUP * kHD;
#pragma unroll
  for (int i = 0; i < kOutPerThread; i++) {
    const int e = tid + i * kThreads;
    const int h = e / kHD, d = e % kHD;
    float a = 0.f;
    for (int s2 = 0; s2 < n_splits; s2++) a += s_sw[h * n_splits + s2] * __ldcg(pob + (size_t)s2 * GROUP * kHD + e);
    io.store(b, h0 + h, d, a * sigmoidf_(io.gate(b, h0 + h, d)));
  }
  if (tid == 0) scr.tickets[bh] = 0;
}

// ---------------------------------------------------------------------------------------------------------------
// The same tensor-core kernel with K and V tiles brought by TMA in the 128-byte swizzle. A 16-token tile is four
// boxes of 64 dims x 16 rows over the cache viewed as [pages x Hkv x page_size rows][256 dims]; in shared memory
// each box is 16 rows of 128 bytes whose 16-byte chunks are XORed with the row index (mod 8). The MMA operands are
// then read with ldmatrix: the 8 rows of each 8 x 8 matrix fall on 8 different chunks, so the fragment loads are
// free of bank conflicts (the bulk-copy ring above keeps rows 512 bytes apart: 2-way conflicts for K, 4-way for V),
// and V^T comes from ldmatrix.trans without byte permutes. Head dims are in natural order: QK k-block kb covers
// dims 16 kb .. 16 kb + 15, PV m-tile i dims 16 i .. 16 i + 15. Rows past the context in the last tile are loaded
// (the box is whole) and never used: their scores are masked, and their V values are zeroed in the registers before
// P V (they may hold anything, e.g. NaN). WARPS warps of kSplit / WARPS tokens per CTA; with 4 warps two CTAs share
// an SM, so one CTA's ring fills while the other streams.
template <int WARPS>
struct TmaCfg {
  static constexpr int kThreads = WARPS * 32;
  static constexpr int kTokW = kSplit / WARPS;  // tokens per warp
  static constexpr int kTiles = kTokW / 16;     // K tiles (and V tiles) per warp
  static constexpr int kStages = 3;
  static constexpr int kWarpRing = kStages * kTileBytes;
  static constexpr int kSmem = WARPS * kWarpRing + 1024;  // + slack to align the ring to 1024 bytes
  static_assert(kTiles <= 32, "one lane per tile for the row lookup");
};

// Shared address of the 16-byte chunk of dims d .. d + 7 (d % 8 == 0) in row r of a swizzled 16-row tile
__device__ __forceinline__ uint32_t sw_addr(uint32_t tile, int r, int d) {
  return tile + (uint32_t)(d >> 6) * 2048u + (uint32_t)r * 128u + ((uint32_t)(((d & 63) >> 3) ^ (r & 7)) << 4);
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

template <class IO, int WARPS>
__global__ void __launch_bounds__(WARPS * 32, 8 / WARPS)
    gqa_decode_tma_kernel(const __grid_constant__ CUtensorMap mk, const __grid_constant__ CUtensorMap mv, IO io,
                          int Hkv, int page_size, int max_pages, float scale, Scratch scr, unsigned int* timeouts) {
  using C = TmaCfg<WARPS>;
  pdl_trigger();
  pdl_wait();
  constexpr int GROUP = 4;
  extern __shared__ uint8_t tma_smem_raw[];
  uint8_t* ring_all = tma_smem_raw + ((1024u - (tc::smem_u32(tma_smem_raw) & 1023u)) & 1023u);
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, c = lane & 3;
  const int ctx = min(io.ctx_of(b), max_pages * page_size);
  const int n_splits = (ctx + kSplit - 1) / kSplit;
  const int h0 = kvh * GROUP;
  if (ctx <= 0) {
    if (split == 0)
      for (int i = tid; i < GROUP * kHD; i += C::kThreads) io.store(b, h0 + i / kHD, i % kHD, 0.0f);
    return;
  }
  if (split >= n_splits) return;

  __shared__ __align__(16) __nv_bfloat16 sP[WARPS][8][16];
  __shared__ __align__(16) float sQ[GROUP][kHD];
  auto sO = [&](int w, int h) { return reinterpret_cast<float*>(ring_all + w * C::kWarpRing) + h * kHD; };
  __shared__ float sM[WARPS][GROUP], sL[WARPS][GROUP];
  __shared__ float s_w[WARPS][GROUP];
  __shared__ float s_fin[GROUP][2];
  __shared__ int s_last;
  __shared__ __align__(8) uint64_t s_bar[WARPS][C::kStages];

  const int32_t* pt = io.page_row(b);
  const int wt0 = split * kSplit + warp * C::kTokW;
  const int nt = min(C::kTiles, max(0, (ctx - wt0 + 15) / 16));
  // lane t holds the cache row of tile t (K tile t and V tile t cover the same tokens)
  int my_row = 0;
  if (lane < nt) {
    const int j = wt0 + 16 * lane;
    my_row = (pt[j / page_size] * Hkv + kvh) * page_size + j % page_size;
  }
  uint8_t* ring = ring_all + warp * C::kWarpRing;
  const uint32_t ring_s = tc::smem_u32(ring);
  uint64_t* bar = s_bar[warp];
  if (lane == 0) {
    for (int i = 0; i < C::kStages; i++) tc::mbar_init(&bar[i], 1);
    tc::fence_barrier_init();
  }
  __syncwarp();
  const uint64_t evict_first = tc::l2_evict_first();
  bool ok = true;
  int issued = 0, consumed = 0;
  auto issue = [&](int n) {  // tile n into stage n % kStages (the warp has finished reading that stage)
    const bool isv = n >= nt;
    const int row = __shfl_sync(0xffffffffu, my_row, isv ? n - nt : n);
    if (!ok) return;
    if (lane == 0) {
      uint8_t* dst = ring + (n % C::kStages) * kTileBytes;
      tc::fence_proxy_async();
      tc::mbar_arrive_expect_tx(&bar[n % C::kStages], kTileBytes);
#pragma unroll
      for (int s = 0; s < 4; s++)
        tc::tma_load_2d_hint(dst + s * 2048, isv ? &mv : &mk, &bar[n % C::kStages], 64 * s, row, evict_first);
    }
    issued = n + 1;
  };
  auto take = [&](int n) -> uint32_t {  // wait for tile n; its stage's shared address
    if (ok && !tc::mbar_wait(&bar[n % C::kStages], (n / C::kStages) & 1)) ok = false;
    if (ok) consumed = n + 1;
    return ring_s + (n % C::kStages) * kTileBytes;
  };
  for (int n = 0; n < C::kStages && n < 2 * nt; n++) issue(n);

  // q of the 4 heads staged once per CTA, then Q^T fragments: column n = g is head g % 4, half g / 4 (0 = hi,
  // 1 = lo), pre-scaled into the log2 domain; k-block kb holds dims {16 kb + 2c, +1} and {16 kb + 8 + 2c, +1}.
  for (int i = tid; i < GROUP * kHD / 8; i += C::kThreads) io.load_q8(b, h0 + i / 32, (i % 32) * 8, &sQ[i / 32][(i % 32) * 8]);
  __syncthreads();
  uint32_t qf[16][2];
  {
    const float* qh = sQ[g & 3];
    const bool lo = g >= 4;
    const float f = scale * kLog2e;
    auto part = [&](float x) {
      x *= f;
      return lo ? x - bf16_round(x) : x;
    };
#pragma unroll
    for (int kb = 0; kb < 16; kb++) {
      qf[kb][0] = pack_bf16x2(part(qh[16 * kb + 2 * c]), part(qh[16 * kb + 2 * c + 1]));
      qf[kb][1] = pack_bf16x2(part(qh[16 * kb + 8 + 2 * c]), part(qh[16 * kb + 9 + 2 * c]));
    }
  }
  // ldmatrix row addresses: lane l gives row (l & 7) of matrix l >> 3
  const int mi = lane >> 3, rr = lane & 7;
  const int k_row = (mi & 1) * 8 + rr, k_dim = (mi >> 1) * 8;  // K: matrices (rows 0-7 | 8-15) x (dims +0 | +8)
  const int v_row = (mi >> 1) * 8 + rr, v_dim = (mi & 1) * 8;  // V: matrices (tokens 0-7 | 8-15) x (dims +0 | +8)

  // ---- scores: lane holds heads hh, hh+1 (hh = 2 (c & 1)) for tokens g and g+8 of each tile
  float sc[C::kTiles][4];
#pragma unroll
  for (int t = 0; t < C::kTiles; t++) {
    const int jA = wt0 + 16 * t + g, jB = jA + 8;
    if (t < nt) {
      const uint32_t tile = take(t);
      float acc0[4] = {0.f, 0.f, 0.f, 0.f}, acc1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int kb = 0; kb < 16; kb++) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4(sw_addr(tile, k_row, 16 * kb + k_dim), a0, a1, a2, a3);
        mma_bf16_16816((kb & 1) ? acc1 : acc0, a0, a1, a2, a3, qf[kb][0], qf[kb][1]);
      }
      __syncwarp();
      if (t + C::kStages < 2 * nt) issue(t + C::kStages);
      float acc[4];
#pragma unroll
      for (int i = 0; i < 4; i++) {
        acc[i] = acc0[i] + acc1[i];
        acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], 2);  // hi + lo columns
      }
      sc[t][0] = jA < ctx ? acc[0] : -INFINITY;
      sc[t][1] = jA < ctx ? acc[1] : -INFINITY;
      sc[t][2] = jB < ctx ? acc[2] : -INFINITY;
      sc[t][3] = jB < ctx ? acc[3] : -INFINITY;
    } else {
      sc[t][0] = sc[t][1] = sc[t][2] = sc[t][3] = -INFINITY;
    }
  }
  // ---- warp softmax statistics per head (lanes with equal c hold the same heads)
  float m0 = -INFINITY, m1 = -INFINITY;
#pragma unroll
  for (int t = 0; t < C::kTiles; t++) {
    m0 = fmaxf(m0, fmaxf(sc[t][0], sc[t][2]));
    m1 = fmaxf(m1, fmaxf(sc[t][1], sc[t][3]));
  }
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, off));
    m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, off));
  }
  const float b0m = m0 == -INFINITY ? 0.f : m0, b1m = m1 == -INFINITY ? 0.f : m1;
  float l0 = 0.f, l1 = 0.f;
#pragma unroll
  for (int t = 0; t < C::kTiles; t++) {
    sc[t][0] = exp2f(sc[t][0] - b0m);
    sc[t][1] = exp2f(sc[t][1] - b1m);
    sc[t][2] = exp2f(sc[t][2] - b0m);
    sc[t][3] = exp2f(sc[t][3] - b1m);
    l0 += sc[t][0] + sc[t][2];
    l1 += sc[t][1] + sc[t][3];
  }
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, off);
    l1 += __shfl_xor_sync(0xffffffffu, l1, off);
  }
  const int hh = 2 * (c & 1);
  if (g == 0 && c < 2) {
    sM[warp][hh] = m0;
    sM[warp][hh + 1] = m1;
    sL[warp][hh] = l0;
    sL[warp][hh + 1] = l1;
  }

  // ---- P.V over the 16 m-tiles of 16 head dims
  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; i++) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
#pragma unroll 1
  for (int t = 0; t < nt; t++) {
    const int base = wt0 + 16 * t;
    __syncwarp();
    {  // P^T into shared memory as [h'][token]: lanes c < 2 write the hi halves, c >= 2 the lo halves
      const int r0 = hh + (c >= 2 ? 4 : 0);
      float pv[4] = {sc[0][0], sc[0][1], sc[0][2], sc[0][3]};
#pragma unroll
      for (int tt = 1; tt < C::kTiles; tt++)
        if (tt == t) pv[0] = sc[tt][0], pv[1] = sc[tt][1], pv[2] = sc[tt][2], pv[3] = sc[tt][3];
      if (c >= 2)
#pragma unroll
        for (int i = 0; i < 4; i++) pv[i] -= bf16_round(pv[i]);
      sP[warp][r0][g] = __float2bfloat16_rn(pv[0]);
      sP[warp][r0 + 1][g] = __float2bfloat16_rn(pv[1]);
      sP[warp][r0][g + 8] = __float2bfloat16_rn(pv[2]);
      sP[warp][r0 + 1][g + 8] = __float2bfloat16_rn(pv[3]);
    }
    __syncwarp();
    const uint32_t pb0 = *reinterpret_cast<const uint32_t*>(&sP[warp][g][2 * c]);
    const uint32_t pb1 = *reinterpret_cast<const uint32_t*>(&sP[warp][g][2 * c + 8]);
    // V rows past the context: tokens 2c, 2c+1 (low, high half of a0 and a1) and 2c+8, 2c+9 (a2, a3)
    const int left = ctx - base;  // >= 1
    const uint32_t m01 = (2 * c < left ? 0x0000FFFFu : 0u) | (2 * c + 1 < left ? 0xFFFF0000u : 0u);
    const uint32_t m23 = (2 * c + 8 < left ? 0x0000FFFFu : 0u) | (2 * c + 9 < left ? 0xFFFF0000u : 0u);
    const uint32_t tile = take(nt + t);
#pragma unroll
    for (int i = 0; i < 16; i++) {
      uint32_t a0, a1, a2, a3;
      ldsm_x4_t(sw_addr(tile, v_row, 16 * i + v_dim), a0, a1, a2, a3);
      mma_bf16_16816(o[i], a0 & m01, a1 & m01, a2 & m23, a3 & m23, pb0, pb1);
    }
    __syncwarp();
    if (nt + t + C::kStages < 2 * nt) issue(nt + t + C::kStages);
  }
  // Every copy this warp issued has been waited for (consumed == issued). After a give-up the warp waits for the
  // outstanding ones once more, again bounded by kWaitNs; if that wait gives up too, a copy may still land in the
  // ring while the warp writes sO below or after the CTA exits, and this split's outputs are undefined (the call
  // already reports EVIE_ERR_TIMEOUT through the device counter).
  ok = __all_sync(0xffffffffu, ok);
  if (!ok) {
    for (int n = consumed; n < issued; n++) tc::mbar_wait(&bar[n % C::kStages], (n / C::kStages) & 1);
    if (lane == 0) atomicAdd(timeouts, 1u);
  }
#pragma unroll
  for (int i = 0; i < 16; i++)
#pragma unroll
    for (int k = 0; k < 4; k++) o[i][k] += __shfl_xor_sync(0xffffffffu, o[i][k], 2);  // hi + lo
  if (c < 2) {
#pragma unroll
    for (int i = 0; i < 16; i++) {
      const int d0 = 16 * i + g, d1 = d0 + 8;
      sO(warp, hh)[d0] = o[i][0];
      sO(warp, hh + 1)[d0] = o[i][1];
      sO(warp, hh)[d1] = o[i][2];
      sO(warp, hh + 1)[d1] = o[i][3];
    }
  }
  __syncthreads();

  // ---- merge the warps of this split
  if (tid < GROUP) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < WARPS; w++) M = fmaxf(M, sM[w][tid]);
    float L = 0.f;
#pragma unroll
    for (int w = 0; w < WARPS; w++) {
      const float wt = sM[w][tid] == -INFINITY ? 0.f : exp2f(sM[w][tid] - M);
      s_w[w][tid] = wt;
      L += wt * sL[w][tid];
    }
    s_fin[tid][0] = M;
    s_fin[tid][1] = L;
  }
  __syncthreads();
  constexpr int kOutPerThread = GROUP * kHD / C::kThreads;
  float osum[kOutPerThread];
#pragma unroll
  for (int i = 0; i < kOutPerThread; i++) {
    const int e = tid + i * C::kThreads;
    const int h = e / kHD, d = e % kHD;
    float a = 0.f;
#pragma unroll
    for (int w = 0; w < WARPS; w++) a += s_w[w][h] * sO(w, h)[d];
    osum[i] = a;
  }
  if (n_splits == 1) {
#pragma unroll
    for (int i = 0; i < kOutPerThread; i++) {
      const int e = tid + i * C::kThreads;
      const int h = e / kHD, d = e % kHD;
      io.store(b, h0 + h, d, osum[i] / s_fin[h][1] * sigmoidf_(io.gate(b, h0 + h, d)));
    }
    return;
  }
  const size_t bh = (size_t)b * Hkv + kvh;
  float* po = scr.o + (bh * scr.max_splits + split) * GROUP * kHD;
#pragma unroll
  for (int i = 0; i < kOutPerThread; i++) __stcg(po + tid + i * C::kThreads, osum[i]);
  if (tid < GROUP) {
    float* pml = scr.ml + ((bh * scr.max_splits + split) * GROUP + tid) * 2;
    __stcg(pml, s_fin[tid][0]);
    __stcg(pml + 1, s_fin[tid][1]);
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = atomicAdd(scr.tickets + bh, 1) == n_splits - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  float* s_sw = sO(0, 0);  // [GROUP][n_splits] merge weights (n_splits <= 512 fits in warp 0's ring)
  if (tid < GROUP) {
    const float* ml = scr.ml + (bh * scr.max_splits) * GROUP * 2;
    float M = -INFINITY;
    for (int s2 = 0; s2 < n_splits; s2++) M = fmaxf(M, __ldcg(ml + ((size_t)s2 * GROUP + tid) * 2));
    float L = 0.f;
    for (int s2 = 0; s2 < n_splits; s2++) {
      const float w = exp2f(__ldcg(ml + ((size_t)s2 * GROUP + tid) * 2) - M);
      s_sw[tid * n_splits + s2] = w;
      L += w * __ldcg(ml + ((size_t)s2 * GROUP + tid) * 2 + 1);
    }
    for (int s2 = 0; s2 < n_splits; s2++) s_sw[tid * n_splits + s2] /= L;
  }
  __syncthreads();
  const float* pob = scr.o + bh * scr.max_splits * GROUP * kHD;
#pragma unroll
  for (int i = 0; i < kOutPerThread; i++) {
    const int e = tid + i * C::kThreads;
    const int h = e / kHD, d = e % kHD;
    float a = 0.f;
    for (int s2 = 0; s2 < n_splits; s2++) a += s_sw[h * n_splits + s2] * __ldcg(pob + (size_t)s2 * GROUP * kHD + e);
    io.store(b, h0 + h, d, a * sigmoidf_(io.gate(b, h0 + h, d)));
  }
  if (tid == 0) scr.tickets[bh] = 0;
}


// The paged cache [pages][Hkv][page_size][256] bf16 as a 2-D tensor (dim, page row), box 64 dims x 16 rows, 128-byte
// swizzle. The row extent is not known to the isolated op, so the map spans the largest row count a TMA coordinate
// can address; the page table bounds the rows read, as it bounds the other kernels' loads.
evie_status kv_tile_map(CUtensorMap* m, const void* base) {
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return fail(EVIE_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  const cuuint64_t dims[2] = {(cuuint64_t)kHD, (cuuint64_t)INT32_MAX};
  const cuuint64_t strides[1] = {(cuuint64_t)kHD * 2};
  const cuuint32_t box[2] = {64, 16};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(EVIE_ERR_CUDA, "cuTensorMapEncodeTiled (KV tiles) failed (%d)", (int)r);
  return EVIE_OK;
}

// Split scratch per (device, stream), grown on demand and kept for the process lifetime, so that calls on
// different streams never share tickets or partials.
struct DeviceScratch {
  void* base = nullptr;
  size_t bytes = 0;
};
std::mutex g_scratch_mu;
std::map<std::pair<int, cudaStream_t>, DeviceScratch> g_scratch;

evie_status get_scratch(int B, int Hkv, int group, int max_splits, Scratch* s, cudaStream_t st) {
  int dev = 0;
  EVIE_CUDA_TRY(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  const size_t n_o = (size_t)B * Hkv * max_splits * group * kHD;
  const size_t n_ml = (size_t)B * Hkv * max_splits * group * 2;
  const size_t n_t = (size_t)B * Hkv;
  const size_t need = (n_o + n_ml) * sizeof(float) + n_t * sizeof(int) + 256;
  DeviceScratch& d = g_scratch[{dev, st}];
  if (d.bytes < need) {
    if (d.base) {
      EVIE_CUDA_TRY(cudaStreamSynchronize(st));
      EVIE_CUDA_TRY(cudaFree(d.base));
      d.base = nullptr;
      d.bytes = 0;
    }
    if (cudaMalloc(&d.base, need) != cudaSuccess) {
      cudaGetLastError();
      return fail(EVIE_ERR_OOM, "evie_gqa_decode_paged: cannot allocate %zu bytes of split scratch", need);
    }
    EVIE_CUDA_TRY(cudaMemsetAsync(d.base, 0, need, st));  // tickets start at zero; each merge resets its own
    d.bytes = need;
  }
  char* p = (char*)d.base;
  s->tickets = (int*)p;
  p += (n_t * sizeof(int) + 255) / 256 * 256;
  s->ml = (float*)p;
  p += n_ml * sizeof(float);
  s->o = (float*)p;
  s->max_splits = max_splits;
  return EVIE_OK;
}


// EVIE_GQA_CUDA_CORES=1 selects the CUDA-core kernel for bf16 KV too (kept as the cross-check of the MMA path).
bool mma_disabled() {
  static const bool off = [] {
    const char* e = getenv("EVIE_GQA_CUDA_CORES");
    return e && e[0] == '1';
  }();
  return off;
}

// EVIE_GQA_BULK=0 keeps the register-fed tensor-core kernel instead of the shared-memory ring ones (same results).
bool bulk_enabled() {
  static const bool on = [] {
    const char* e = getenv("EVIE_GQA_BULK");
    return !(e && e[0] == '0');
  }();
  return on;
}

// Warps per CTA of the TMA kernel: 4 (two CTAs per SM, the default) or 8; EVIE_GQA_TMA=0 keeps the bulk-copy ring.
int tma_warps() {
  static const int w = [] {
    const char* e = getenv("EVIE_GQA_TMA");
    if (!e) return 4;
    const int v = atoi(e);
    return v == 0 || v == 8 ? v : 4;
  }();
  return w;
}

template <class IO, int WARPS>
evie_status launch_tma(const IO& io, const __nv_bfloat16* kp, const __nv_bfloat16* vp, dim3 grid, int Hkv,
                       int page_size, int max_pages, float scale, const Scratch& scr, unsigned int* counter,
                       cudaStream_t st) {
  using C = TmaCfg<WARPS>;
  if (page_size % 16 != 0) return fail(EVIE_ERR_ARG, "decode attention: page size must be a multiple of 16");
  if (((uintptr_t)kp | (uintptr_t)vp) & 15) return fail(EVIE_ERR_ARG, "decode attention: KV pages 16-byte aligned");
  CUtensorMap mk, mv;
  EVIE_TRY(kv_tile_map(&mk, kp));
  EVIE_TRY(kv_tile_map(&mv, vp));
  EVIE_TRY(max_dynamic_smem((const void*)gqa_decode_tma_kernel<IO, WARPS>, C::kSmem));
  EVIE_CUDA_TRY(launch_k(gqa_decode_tma_kernel<IO, WARPS>, grid, dim3(C::kThreads), C::kSmem, st, mk, mv, io, Hkv,
                         page_size, max_pages, scale, scr, counter));
  EVIE_CHECK_LAUNCH("gqa_decode_tma_kernel");
  return EVIE_OK;
}

template <typename KV, class IO>
evie_status launch_gqa(const IO& io, const KV* kp, const KV* vp, int B, int Hq, int Hkv, int page_size, int max_pages,
                       int max_ctx, float scale, const Scratch& scr, cudaStream_t st) {
  const int group = Hq / Hkv;
  const int max_splits = (max_ctx + kSplit - 1) / kSplit;
  dim3 grid(max_splits > 0 ? max_splits : 1, Hkv, B);
  if constexpr (sizeof(KV) == 2) {
    if (group == 4 && !mma_disabled()) {
      if (bulk_enabled()) {
        unsigned int* counter = device_timeout_counter();
        if (!counter) return fail(EVIE_ERR_CUDA, "device timeout counter unavailable");
        if (tma_warps() == 4) return launch_tma<IO, 4>(io, kp, vp, grid, Hkv, page_size, max_pages, scale, scr, counter, st);
        if (tma_warps() == 8) return launch_tma<IO, 8>(io, kp, vp, grid, Hkv, page_size, max_pages, scale, scr, counter, st);
        EVIE_TRY(max_dynamic_smem((const void*)gqa_decode_bulk_kernel<IO>, kRingBytes));
        EVIE_CUDA_TRY(launch_k(gqa_decode_bulk_kernel<IO>, dim3(grid), dim3(kThreads), kRingBytes, st, io, kp, vp, Hkv, page_size, max_pages, scale,
                                                                        scr, counter));
        EVIE_CHECK_LAUNCH("gqa_decode_bulk_kernel");
        return EVIE_OK;
      }
      EVIE_CUDA_TRY(launch_k(gqa_decode_mma_kernel<IO>, dim3(grid), dim3(kThreads), 0, st, io, kp, vp, Hkv, page_size, max_pages, scale, scr));
      EVIE_CHECK_LAUNCH("gqa_decode_mma_kernel");
      return EVIE_OK;
    }
  }
  switch (group) {
    case 2: EVIE_CUDA_TRY(launch_k(gqa_decode_kernel<2, KV, IO>, dim3(grid), dim3(kThreads), 0, st, io, kp, vp, Hkv, page_size, max_pages, scale, scr)); break;
    case 4: EVIE_CUDA_TRY(launch_k(gqa_decode_kernel<4, KV, IO>, dim3(grid), dim3(kThreads), 0, st, io, kp, vp, Hkv, page_size, max_pages, scale, scr)); break;
    default: return fail(EVIE_ERR_ARG, "GQA group %d not supported (2, 4)", group);
  }
  EVIE_CHECK_LAUNCH("gqa_decode_kernel");
  return EVIE_OK;
}

}  // namespace

size_t gqa_scratch_bytes(int rows, int Hkv, int group, int max_ctx) {
  const size_t max_splits = (size_t)(max_ctx + kSplit - 1) / kSplit;
  const size_t n_o = (size_t)rows * Hkv * max_splits * group * kHD;
  const size_t n_ml = (size_t)rows * Hkv * max_splits * group * 2;
  const size_t n_t = (size_t)rows * Hkv;
  return (n_t * sizeof(int) + 255) / 256 * 256 + (n_ml + n_o) * sizeof(float) + 256;
}

evie_status launch_gqa_decode_bf16(const void* q, const void* gate, const void* kp, const void* vp,
                                   const int32_t* page_table, const int32_t* ctx_lens, float* out, int B, int Hq,
                                   int Hkv, int page_size, int max_pages, float scale, cudaStream_t st) {
  const int group = Hq / Hkv;
  const long max_tokens = (long)max_pages * page_size;
  const int max_splits = (int)((max_tokens + kSplit - 1) / kSplit);
  if (B == 0 || max_splits == 0) {
    if (B > 0) {  // no context at all: outputs are zero
      EVIE_CUDA_TRY(cudaMemsetAsync(out, 0, sizeof(float) * (size_t)B * Hq * kHD, st));
    }
    return EVIE_OK;
  }
  Scratch scr;
  evie_status rc = get_scratch(B, Hkv, group, max_splits, &scr, st);
  if (rc != EVIE_OK) return rc;
  IsoIO io{(const __nv_bfloat16*)q, (const __nv_bfloat16*)gate, out, page_table, ctx_lens, Hq, max_pages};
  return launch_gqa<__nv_bfloat16>(io, (const __nv_bfloat16*)kp, (const __nv_bfloat16*)vp, B, Hq, Hkv, page_size,
                                   max_pages, (int)max_tokens, scale, scr, st);
}

// ---------------------------------------------------------------------------------------------------------------
// Allocation-free variant of the isolated op (evie_gqa_decode_paged_noalloc).
//
// Some callers cannot let a library allocate device memory for them: serving engines that reserve nearly all of the
// GPU's memory for their own caching allocator at start-up (a later cudaMalloc then fails, or carves memory out of
// a pool they manage), and callers on a latency-critical path where cudaMalloc / cudaFree would synchronise the
// device. For them the split scratch comes from this fixed array, compiled into the library: every GPU that loads
// the library holds these bytes until the process exits.
constexpr size_t kNoAllocScratchBytes = 32u << 20;
static __device__ __align__(256) unsigned char g_gqa_noalloc_scratch[kNoAllocScratchBytes];

// In host code `g_gqa_noalloc_scratch` only names the symbol; it is not a device address, and a kernel given it would
// fault (or silently use the wrong memory where the GPU can reach host memory). The device address is looked up once
// per device, with that device current, on the first call there.
std::mutex g_noalloc_mu;
void* g_noalloc_addr[kMaxDevices] = {};

evie_status noalloc_scratch(void** out) {
  int dev = 0;
  EVIE_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices)
    return fail(EVIE_ERR_ARG, "evie_gqa_decode_paged_noalloc: device %d out of range (0..%d)", dev, kMaxDevices - 1);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_addr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_gqa_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return fail(EVIE_ERR_CUDA, "evie_gqa_decode_paged_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    g_noalloc_addr[dev] = p;
  }
  *out = g_noalloc_addr[dev];
  return EVIE_OK;
}

evie_status launch_gqa_decode_bf16_noalloc(const void* q, const void* gate, const void* kp, const void* vp,
                                           const int32_t* page_table, const int32_t* ctx_lens, float* out, int B,
                                           int Hq, int Hkv, int page_size, int max_pages, float scale,
                                           cudaStream_t st) {
  const int group = Hq / Hkv;
  const long max_tokens = (long)max_pages * page_size;
  const int max_splits = (int)((max_tokens + kSplit - 1) / kSplit);
  if (B == 0 || max_splits == 0) {
    if (B > 0) EVIE_CUDA_TRY(cudaMemsetAsync(out, 0, sizeof(float) * (size_t)B * Hq * kHD, st));
    return EVIE_OK;
  }
  // Same partition as the allocating path: tickets, then per-split (max, sum), then per-split outputs.
  const size_t n_t = (size_t)B * Hkv;
  const size_t t_bytes = (n_t * sizeof(int) + 255) / 256 * 256;
  const size_t n_ml = (size_t)B * Hkv * max_splits * group * 2;
  const size_t n_o = (size_t)B * Hkv * max_splits * group * kHD;
  const size_t need = t_bytes + (n_ml + n_o) * sizeof(float);
  if (need > kNoAllocScratchBytes)
    return fail(EVIE_ERR_ARG,
                "evie_gqa_decode_paged_noalloc: these sizes need %zu bytes of split scratch, more than its fixed %zu "
                "(sizes with B x Hkv x ceil(max_pages x page_size / 512) at most %zu always fit); use "
                "evie_gqa_decode_paged",
                need, kNoAllocScratchBytes,
                (kNoAllocScratchBytes - 255) / (sizeof(int) + (size_t)group * (kHD + 2) * sizeof(float)));
  void* base = nullptr;
  evie_status rc = noalloc_scratch(&base);
  if (rc != EVIE_OK) return rc;
  // The array keeps the previous call's contents; the tickets must start at zero.
  EVIE_CUDA_TRY(cudaMemsetAsync(base, 0, t_bytes, st));
  Scratch scr;
  char* p = (char*)base;
  scr.tickets = (int*)p;
  p += t_bytes;
  scr.ml = (float*)p;
  p += n_ml * sizeof(float);
  scr.o = (float*)p;
  scr.max_splits = max_splits;
  IsoIO io{(const __nv_bfloat16*)q, (const __nv_bfloat16*)gate, out, page_table, ctx_lens, Hq, max_pages};
  return launch_gqa<__nv_bfloat16>(io, (const __nv_bfloat16*)kp, (const __nv_bfloat16*)vp, B, Hq, Hkv, page_size,
                                   max_pages, (int)max_tokens, scale, scr, st);
}

template <typename KV>
evie_status launch_gqa_model(const float* q_rot, YView y, int ldy, __nv_bfloat16* X2,
                             size_t xplane, const RowInfo* rows, int R, const int* page_table, int pages_per_slot,
                             const KV* kc, const KV* vc, int Hq, int Hkv, int page_size, int max_ctx, float scale,
                             void* scratch, int ticket_rows, cudaStream_t st) {
  if (R == 0) return EVIE_OK;
  const int group = Hq / Hkv;
  const int max_splits = (max_ctx + kSplit - 1) / kSplit;
  Scratch scr;
  char* p = (char*)scratch;
  scr.tickets = (int*)p;  // fixed-size region: tickets of unused rows stay zero across calls
  p += ((size_t)ticket_rows * Hkv * sizeof(int) + 255) / 256 * 256;
  scr.ml = (float*)p;
  p += (size_t)R * Hkv * max_splits * group * 2 * sizeof(float);
  scr.o = (float*)p;
  scr.max_splits = max_splits;
  ModelIO io{q_rot, y, ldy, X2, xplane, rows, page_table, pages_per_slot, Hq};
  return launch_gqa<KV>(io, kc, vc, R, Hq, Hkv, page_size, pages_per_slot, max_ctx, scale, scr, st);
}
template evie_status launch_gqa_model<__nv_bfloat16>(const float*, YView, int, __nv_bfloat16*, size_t,
                                                     const RowInfo*, int, const int*, int, const __nv_bfloat16*,
                                                     const __nv_bfloat16*, int, int, int, int, float, void*, int,
                                                     cudaStream_t);
template evie_status launch_gqa_model<float>(const float*, YView, int, __nv_bfloat16*, size_t,
                                             const RowInfo*, int, const int*, int, const float*, const float*, int, int,
                                             int, int, float, void*, int, cudaStream_t);

}  // namespace evie

extern "C" evie_status evie_gqa_decode_paged(const void* q, const void* gate, const void* k_pages, const void* v_pages,
                                             const int32_t* page_table, const int32_t* ctx_lens, float* out, int B,
                                             int Hq, int Hkv, int hd, int page_size, int max_pages, float scale,
                                             void* stream) {
  EVIE_ARG(hd == 256, "evie_gqa_decode_paged: head_dim 256 required (got %d)", hd);
  EVIE_ARG(B >= 0 && Hkv > 0 && Hq > 0 && Hq % Hkv == 0, "evie_gqa_decode_paged: bad head counts %d/%d", Hq, Hkv);
  const int group = Hq / Hkv;
  EVIE_ARG(group == 2 || group == 4, "evie_gqa_decode_paged: GQA group %d unsupported (2 or 4)", group);
  EVIE_ARG(page_size > 0 && page_size % 64 == 0, "evie_gqa_decode_paged: page_size must be a multiple of 64");
  EVIE_ARG(max_pages >= 0 && (long)max_pages * page_size <= evie::kGqaMaxContext,
           "evie_gqa_decode_paged: max_pages * page_size exceeds %ld tokens", (long)evie::kGqaMaxContext);
  EVIE_ARG(B <= 65535 && Hkv <= 65535, "evie_gqa_decode_paged: grid too large");
  EVIE_ARG(B == 0 || (q && gate && k_pages && v_pages && page_table && ctx_lens && out),
           "evie_gqa_decode_paged: null pointer");
  EVIE_ARG((((uintptr_t)q | (uintptr_t)k_pages | (uintptr_t)v_pages) & 15) == 0,
           "evie_gqa_decode_paged: q and the KV pages must be 16-byte aligned");
  return evie::launch_gqa_decode_bf16(q, gate, k_pages, v_pages, page_table, ctx_lens, out, B, Hq, Hkv, page_size,
                                      max_pages, scale, (cudaStream_t)stream);
}

// No counterpart in the reference: the allocation-free form of evie_gqa_decode_paged (see the header).
extern "C" evie_status evie_gqa_decode_paged_noalloc(const void* q, const void* gate, const void* k_pages,
                                                     const void* v_pages, const int32_t* page_table,
                                                     const int32_t* ctx_lens, float* out, int B, int Hq, int Hkv,
                                                     int hd, int page_size, int max_pages, float scale, void* stream) {
  EVIE_ARG(hd == 256, "evie_gqa_decode_paged_noalloc: head_dim 256 required (got %d)", hd);
  EVIE_ARG(B >= 0 && Hkv > 0 && Hq > 0 && Hq % Hkv == 0, "evie_gqa_decode_paged_noalloc: bad head counts %d/%d", Hq,
           Hkv);
  const int group = Hq / Hkv;
  EVIE_ARG(group == 2 || group == 4, "evie_gqa_decode_paged_noalloc: GQA group %d unsupported (2 or 4)", group);
  EVIE_ARG(page_size > 0 && page_size % 64 == 0, "evie_gqa_decode_paged_noalloc: page_size must be a multiple of 64");
  EVIE_ARG(max_pages >= 0 && (long)max_pages * page_size <= evie::kGqaMaxContext,
           "evie_gqa_decode_paged_noalloc: max_pages * page_size exceeds %ld tokens", (long)evie::kGqaMaxContext);
  EVIE_ARG(B <= 65535 && Hkv <= 65535, "evie_gqa_decode_paged_noalloc: grid too large");
  EVIE_ARG(B == 0 || (q && gate && k_pages && v_pages && page_table && ctx_lens && out),
           "evie_gqa_decode_paged_noalloc: null pointer");
  EVIE_ARG((((uintptr_t)q | (uintptr_t)k_pages | (uintptr_t)v_pages) & 15) == 0,
           "evie_gqa_decode_paged_noalloc: q and the KV pages must be 16-byte aligned");
  return evie::launch_gqa_decode_bf16_noalloc(q, gate, k_pages, v_pages, page_table, ctx_lens, out, B, Hq, Hkv,
                                              page_size, max_pages, scale, (cudaStream_t)stream);
}
