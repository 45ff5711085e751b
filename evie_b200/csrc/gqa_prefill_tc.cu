// Gated GQA softmax attention for prefill rows on sm_100a tensor cores (tcgen05 MMA, TMEM accumulators, TMA).
//
// Semantics are the attention core of Model::attention (crates/evie-core/src/model.rs:445-464): for query row r at
// position pos_r and query head h (KV head h / 4),
//   o = softmax(scale * q . k_j, j <= pos_r) V * sigmoid(gate),
// over the paged bf16 KV cache the rows' keys and values were appended to. The WGSL twin is attn_scores / attn_out
// (gpu/kernels.wgsl:508-589).
//
// Work layout. One CTA per (block of 32 consecutive rows of one sequence, KV head): the MMA's M = 128 rows are the
// (query head of the group, row) pairs, m = 32 head + row, so TMEM lane quarter q holds head q of the group and lane
// l row l. K and V stream through shared memory in 64-token tiles, each read once per block of 32 rows x 4 heads.
//   S   = Q K^T          M = 128, N = 64 tokens, K = 256 dims: Q is f32 in the model, so it is held as two bf16
//                        planes (hi = bf16(q s), lo = bf16(q s - hi), s = scale log2 e) and S = Q_hi K^T + Q_lo K^T;
//                        S is double-buffered in TMEM, so the next tile's scores overlap this tile's softmax.
//   P   = exp2(S - m)    the softmax warps (one thread per (head, row)) read S with tcgen05.ld, mask tokens past
//                        the row's position, and write P as bf16 hi + lo planes into TMEM, the A operand of
//   O  += P V            M = 128, N = 256 dims, K = 64 tokens (A from TMEM, V as the MN-major B operand), O in TMEM.
// The running max m is raised only when a tile's maximum exceeds it by more than 8 (a factor 256 in P): O and the
// running sum are then rescaled by exp2(m_old - m_new) in TMEM; otherwise P is taken against the old m (at most 256,
// exact in the hi + lo planes). The final O / l is the same quotient either way.
// The last tile's V rows past the block's last position are zeroed in shared memory before P V reads them (the
// cache there may hold anything); its K rows need no zeroing (their scores are masked).
//
// Buffers: K single (its next copy waits for this tile's S MMAs, which are issued a tile ahead), V and P double,
// so the softmax of tile j + 1 overlaps P V of tile j and only a rescale of O waits for it.
//
// Roles (224 threads): warp 0 lane 0 issues the K and V tile copies; warp 1 owns tensor memory and lane 0 issues
// the S MMAs; warp 6 lane 0 issues the P V MMAs (a second issuing thread, so they never queue behind a wait for the
// next K tile); warps 2-5 run the softmax and the epilogue (O / l x sigmoid(gate), staged through shared memory so
// that the stores are coalesced). Every mbarrier wait is bounded (2 s); a thread that gives up stops, the CTA drains its
// copies and MMAs (bounded again), frees TMEM and counts the give-up for the host.
#include <cudaTypedefs.h>

#include <map>
#include <mutex>
#include <vector>

#include "gdn_chunk.h"
#include "gqa_decode.h"
#include "model_kernels.h"
#include "tc.h"
#include "tmap.h"

namespace evie {

namespace {

constexpr int kHD = 256;
constexpr int kGroup = 4;
constexpr int kRows = 32;     // query rows per CTA (x 4 heads = M 128)
constexpr int kTok = 64;      // tokens per K / V tile
constexpr int kThreads = 224;  // warp 0 copies, warp 1 S MMAs (and TMEM), warps 2-5 softmax, warp 6 P V MMAs
constexpr int kSoftThreads = 128;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescale = 8.0f;  // log2 of the largest P value allowed before the running max is raised

// Shared memory (offsets from a 1024-aligned base)
constexpr uint32_t kQPlane = 65536;                  // 4 dim blocks x 128 rows x 128 B
constexpr uint32_t kOffQH = 0, kOffQL = kQPlane;
constexpr uint32_t kOffK = 2 * kQPlane;              // 4 dim blocks x 64 tokens x 128 B
constexpr uint32_t kOffV = kOffK + 32768;            // two buffers of 32 KB
constexpr uint32_t kOffBar = kOffV + 65536;
constexpr uint32_t kSmem = kOffBar + 256 + 1024;
static_assert(kSmem <= 232448, "shared memory");
constexpr int kStageStride = 260;                    // floats per staged output row (1040 B: conflict-free float4)
static_assert(128 * kStageStride * 4 <= (int)kOffBar, "output staging must fit below the barriers");

// TMEM columns: O, two S buffers, two P buffers (hi plane then lo plane, 32 columns each)
constexpr uint32_t kColO = 0, kColS = 256, kColP = 384;

// mbarriers; the double-buffered ones have one barrier per buffer, so that a wait never aliases a later phase
enum {
  B_KFULL = 0, B_KFREE, B_VF0, B_VF1, B_S0, B_S1, B_SF0, B_SF1, B_PF0, B_PF1, B_PV0, B_PV1, B_DRAIN, B_DRAIN2,
  kNumBars
};

__device__ __forceinline__ uint32_t swz(int r, int c) { return (uint32_t)r * 128u + ((uint32_t)(c ^ (r & 7)) << 4); }

__device__ __forceinline__ uint32_t pack_rn(float a, float b) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);  // a in the low half
  return *reinterpret_cast<const uint32_t*>(&v);
}

// The model: queries f32 [R][Hq][256]; gate logits in the attention input projection (YView); output into the
// o_proj operand planes.
struct ModelIO {
  const float* q;
  YView y;
  int ldy;
  __nv_bfloat16* X2;
  size_t xplane;
  int Hq;
  __device__ __forceinline__ const float* qrow(int row, int head) const { return q + ((size_t)row * Hq + head) * kHD; }
  __device__ __forceinline__ float gate(int row, int head, int d) const {
    return y.at((size_t)row * ldy + (size_t)head * 2 * kHD + kHD + d);
  }
  __device__ __forceinline__ void store(int row, int head, int d, float v) const {
    store_split(X2, xplane, ((size_t)row * Hq + head) * kHD + d, v);
  }
};
// The isolated op: q, gate logits and out f32 [R][Hq][256].
struct IsoIO {
  const float* q;
  const float* g;
  float* out;
  int Hq;
  __device__ __forceinline__ const float* qrow(int row, int head) const { return q + ((size_t)row * Hq + head) * kHD; }
  __device__ __forceinline__ float gate(int row, int head, int d) const {
    return g[((size_t)row * Hq + head) * kHD + d];
  }
  __device__ __forceinline__ void store(int row, int head, int d, float v) const {
    out[((size_t)row * Hq + head) * kHD + d] = v;
  }
};

template <class IO>
__global__ void __launch_bounds__(kThreads, 1)
    gqa_prefill_tc_kernel(const __grid_constant__ CUtensorMap mk, const __grid_constant__ CUtensorMap mv, const IO io,
                          const SegInfo* __restrict__ segs, const int* __restrict__ page_table, int pages_per_slot,
                          int Hkv, int page_size, float qscale, unsigned int* timeouts) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = smem_raw + ((1024u - (tc::smem_u32(smem_raw) & 1023u)) & 1023u);
  const int kvh = blockIdx.z;
  const SegInfo sg = segs[blockIdx.y];
  // Row blocks in reverse: CTAs are dispatched x fastest, and a block's causal work grows with its rows, so the
  // longest blocks of each (segment, KV head) start first and the last CTAs of the launch are short ones.
  const int r_first = (gridDim.x - 1 - blockIdx.x) * kRows;
  if (r_first >= sg.count) return;  // the whole CTA: before any barrier or TMEM allocation
  const int nr = min(kRows, sg.count - r_first);
  const int row0 = sg.start + r_first;
  const int pos_first = sg.pos0 + r_first;
  const int pmax = pos_first + nr - 1;
  const int ntiles = pmax / kTok + 1;
  const int* pt = page_table + (size_t)sg.slot * pages_per_slot;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + kOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + kNumBars);
  __shared__ int s_fail;

  if (tid == 0) {
    for (int i = 0; i < kNumBars; i++)
      tc::mbar_init(&bar[i], (i == B_SF0 || i == B_SF1 || i == B_PF0 || i == B_PF1) ? kSoftThreads : 1);
    s_fail = 0;
    tc::fence_barrier_init();
    tc::prefetch_tmap(&mk);
    tc::prefetch_tmap(&mv);
  }
  if (warp == 1) tc::tmem_alloc(tmem_slot, 512);

  // ---- Q: rows m = 32 head + row (head of the group), 256 dims, scaled by scale log2 e, split into bf16 hi + lo,
  // K-major 128-byte-swizzled tiles of 64 dims. Rows past the block are zero. Eight 8-dim units per thread are
  // loaded before any is converted, so their global loads overlap.
  constexpr int kQUnits = 128 * 32;
  for (int u0 = tid; u0 < kQUnits; u0 += 8 * kThreads) {
    float x[8][8];
#pragma unroll
    for (int k = 0; k < 8; k++) {
      const int u = u0 + k * kThreads, m = u >> 5, k16 = u & 31, hq = m >> 5, r = m & 31;
      if (u < kQUnits && r < nr) {
        const float* qp = io.qrow(row0 + r, kvh * kGroup + hq) + 8 * k16;
        const float4 a = *reinterpret_cast<const float4*>(qp);
        const float4 b = *reinterpret_cast<const float4*>(qp + 4);
        x[k][0] = a.x; x[k][1] = a.y; x[k][2] = a.z; x[k][3] = a.w;
        x[k][4] = b.x; x[k][5] = b.y; x[k][6] = b.z; x[k][7] = b.w;
      } else {
#pragma unroll
        for (int i = 0; i < 8; i++) x[k][i] = 0.f;
      }
    }
#pragma unroll
    for (int k = 0; k < 8; k++) {
      const int u = u0 + k * kThreads, m = u >> 5, k16 = u & 31;
      if (u >= kQUnits) break;
      uint32_t hi[4], lo[4];
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const float v0 = x[k][2 * i] * qscale, v1 = x[k][2 * i + 1] * qscale;
        const float h0 = __bfloat162float(__float2bfloat16_rn(v0)), h1 = __bfloat162float(__float2bfloat16_rn(v1));
        hi[i] = pack_rn(h0, h1);
        lo[i] = pack_rn(v0 - h0, v1 - h1);
      }
      const uint32_t off = (uint32_t)(k16 >> 3) * 16384u + swz(m, k16 & 7);
      *reinterpret_cast<uint4*>(sm + kOffQH + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
      *reinterpret_cast<uint4*>(sm + kOffQL + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    }
  }
  tc::fence_proxy_async();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;
  int kfills = 0, vfills[2] = {0, 0};  // producer: copies armed

  if (warp == 0) {
    if (lane == 0) {
      // ---- K (one buffer) and V (two buffers) tile copies
      for (int j = 0; j < ntiles && ok; j++) {
        const int tok0 = j * kTok;
        const int krow = (pt[tok0 / page_size] * Hkv + kvh) * page_size + tok0 % page_size;
        if (j >= 1 && !tc::mbar_wait(&bar[B_KFREE], (j - 1) & 1)) { ok = false; break; }
        tc::mbar_arrive_expect_tx(&bar[B_KFULL], 32768);
        kfills++;
        for (int c = 0; c < 4; c++) tc::tma_load_2d(sm + kOffK + c * 8192, &mk, &bar[B_KFULL], c * 64, krow);
        const int vb = j & 1;  // V buffer of tile j was read by P V of tile j - 2
        if (j >= 2 && !tc::mbar_wait(&bar[B_PV0 + vb], ((j - 2) >> 1) & 1)) { ok = false; break; }
        tc::mbar_arrive_expect_tx(&bar[B_VF0 + vb], 32768);
        vfills[vb]++;
        for (int c = 0; c < 4; c++)
          tc::tma_load_2d(sm + kOffV + vb * 32768 + c * 8192, &mv, &bar[B_VF0 + vb], c * 64, krow);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- S MMAs, running ahead of the softmax as far as the S buffers and the K copies allow
      constexpr uint32_t idS = tc::idesc(1, 1, 128, kTok);
      const uint64_t dQH = tc::sdesc_k_sw128(sm + kOffQH), dQL = tc::sdesc_k_sw128(sm + kOffQL);
      const uint64_t dK = tc::sdesc_k_sw128(sm + kOffK);
      for (int j = 0; j < ntiles; j++) {
        if (!tc::mbar_wait(&bar[B_KFULL], j & 1)) { ok = false; break; }
        if (j >= 2 && !tc::mbar_wait(&bar[B_SF0 + (j & 1)], ((j - 2) >> 1) & 1)) { ok = false; break; }
        tc::fence_after_sync();
        const uint32_t d = tmem + kColS + (uint32_t)(j & 1) * kTok;
        int n = 0;
#pragma unroll
        for (int c = 0; c < 4; c++)
#pragma unroll
          for (int kk = 0; kk < 4; kk++) {
            const uint32_t a = (c * 16384 + kk * 32) >> 4, b = (c * 8192 + kk * 32) >> 4;
            tc::mma_f16(d, dQH + a, dK + b, idS, n++ > 0);
            tc::mma_f16(d, dQL + a, dK + b, idS, 1u);
          }
        tc::mma_commit(&bar[B_KFREE]);
        tc::mma_commit(&bar[B_S0 + (j & 1)]);
      }
      tc::mma_commit(&bar[B_DRAIN]);
      if (!tc::mbar_wait(&bar[B_DRAIN], 0)) ok = false;
    }
  } else if (warp == 6) {
    if (lane == 0) {
      // ---- P V MMAs (another issuing thread: they never wait behind a K copy)
      constexpr uint32_t idO = tc::idesc(1, 1, 128, kHD, false, true);
      const uint64_t dV = tc::sdesc_mn_sw128(sm + kOffV, 8192, 1024);
      for (int j = 0; j < ntiles; j++) {
        const int b = j & 1;
        if (!tc::mbar_wait(&bar[B_PF0 + b], (j >> 1) & 1) || !tc::mbar_wait(&bar[B_VF0 + b], (j >> 1) & 1)) {
          ok = false;
          break;
        }
        tc::fence_after_sync();
        const uint32_t ph = tmem + kColP + (uint32_t)b * 64, pl = ph + 32;
        const uint64_t dvb = dV + ((uint32_t)(b * 32768) >> 4);
#pragma unroll
        for (int kk = 0; kk < kTok / 16; kk++) {
          tc::mma_f16_ts(tmem + kColO, ph + kk * 8, dvb + ((kk * 2048) >> 4), idO, (j > 0 || kk > 0));
          tc::mma_f16_ts(tmem + kColO, pl + kk * 8, dvb + ((kk * 2048) >> 4), idO, 1u);
        }
        tc::mma_commit(&bar[B_PV0 + b]);
      }
      tc::mma_commit(&bar[B_DRAIN2]);
      if (!tc::mbar_wait(&bar[B_DRAIN2], 0)) ok = false;
    }
  } else if (warp < 6) {
    // ---- softmax: thread = (head q of the group, row `lane`) in TMEM lane quarter q
    const int q = warp & 3;
    const uint32_t tl = tmem + ((uint32_t)(q * 32) << 16);
    const int pr = min(pos_first + lane, pmax);  // rows past the block take the last position (outputs unused)
    float m_run = -INFINITY, l = 0.f;
    for (int j = 0; j < ntiles; j++) {
      const int b = j & 1;
      if (!tc::mbar_wait(&bar[B_S0 + b], (j >> 1) & 1)) { ok = false; break; }
      tc::fence_after_sync();
      float s[kTok];
      tc::tmem_ld32(tl + kColS + b * kTok, s);
      tc::tmem_ld32(tl + kColS + b * kTok + 32, s + 32);
      tc::fence_before_sync();
      tc::mbar_arrive(&bar[B_SF0 + b]);  // S buffer free for tile j + 2
      float mt = -INFINITY;
#pragma unroll
      for (int i = 0; i < kTok; i++) {
        if (j * kTok + i > pr) s[i] = -INFINITY;
        mt = fmaxf(mt, s[i]);
      }
      const bool raise = mt > m_run + kRescale;
      float alpha = 1.f;
      if (raise) {
        alpha = exp2f(m_run - mt);  // 0 on the first tile
        m_run = mt;
        l *= alpha;
      }
      if (j >= 1 && __any_sync(0xffffffffu, raise)) {
        // rescale this warp's O rows once P V of the previous tile has landed (warp-wide TMEM access)
        if (!tc::mbar_wait(&bar[B_PV0 + (b ^ 1)], ((j - 1) >> 1) & 1)) { ok = false; break; }
        tc::fence_after_sync();
#pragma unroll 1
        for (int c0 = 0; c0 < kHD; c0 += 32) {
          float o[32];
          tc::tmem_ld32(tl + kColO + c0, o);
#pragma unroll
          for (int i = 0; i < 32; i++) o[i] *= alpha;
          tc::tmem_st32(tl + kColO + c0, o);
        }
      }
      uint32_t ph[kTok / 2], pl[kTok / 2];
#pragma unroll
      for (int i = 0; i < kTok / 2; i++) {
        const float p0 = exp2f(s[2 * i] - m_run), p1 = exp2f(s[2 * i + 1] - m_run);
        l += p0;
        l += p1;
        const float h0 = __bfloat162float(__float2bfloat16_rn(p0)), h1 = __bfloat162float(__float2bfloat16_rn(p1));
        ph[i] = pack_rn(h0, h1);
        pl[i] = pack_rn(p0 - h0, p1 - h1);
      }
      if (j >= 2) {  // P buffer b was read by P V of tile j - 2
        if (!tc::mbar_wait(&bar[B_PV0 + b], ((j - 2) >> 1) & 1)) { ok = false; break; }
        tc::fence_after_sync();
      }
      const uint32_t pcol = tl + kColP + (uint32_t)b * 64;
      tc::tmem_st16u(pcol, ph);
      tc::tmem_st16u(pcol + 16, ph + 16);
      tc::tmem_st16u(pcol + 32, pl);
      tc::tmem_st16u(pcol + 48, pl + 16);
      if (j == ntiles - 1) {  // zero the V rows past the block's last position (after their copy has landed)
        const int first_bad = pmax - j * kTok + 1;
        if (first_bad < kTok) {
          if (!tc::mbar_wait(&bar[B_VF0 + b], (j >> 1) & 1)) { ok = false; break; }
          const int units = (kTok - first_bad) * 4 * 8;  // rows x dim blocks x 16-byte units
          for (int u = tid - 64; u < units; u += kSoftThreads) {
            const int row = first_bad + u / 32, c = (u >> 3) & 3, k = u & 7;
            *reinterpret_cast<uint4*>(sm + kOffV + b * 32768 + c * 8192 + row * 128 + k * 16) = make_uint4(0, 0, 0, 0);
          }
          tc::fence_proxy_async();
        }
      }
      tc::tmem_st_wait();
      tc::fence_before_sync();
      tc::mbar_arrive(&bar[B_PF0 + b]);
    }
    // ---- epilogue: O / l, staged row-major through shared memory (the Q tiles and K, V are no longer read)
    if (ok && !tc::mbar_wait(&bar[B_PV0 + ((ntiles - 1) & 1)], ((ntiles - 1) >> 1) & 1)) ok = false;
    tc::fence_after_sync();
    const bool soft_ok = tc::group_sync_or(1, kSoftThreads, !ok) == false;
    if (soft_ok) {
      float* stage = reinterpret_cast<float*>(sm);
      const int m = q * 32 + lane;
      const float inv = 1.0f / l;
#pragma unroll 1
      for (int c0 = 0; c0 < kHD; c0 += 32) {
        float o[32];
        tc::tmem_ld32(tl + kColO + c0, o);
#pragma unroll
        for (int i = 0; i < 32; i += 4)
          *reinterpret_cast<float4*>(stage + m * kStageStride + c0 + i) =
              make_float4(o[i] * inv, o[i + 1] * inv, o[i + 2] * inv, o[i + 3] * inv);
      }
      tc::group_sync_or(1, kSoftThreads, false);
      // warp w writes rows m = w', w' + 4, ...: 256 contiguous dims of one (row, head) per pass; the gate logits
      // of four rows are loaded before any is used, so their latencies overlap
      const int sw = warp - 2;
#pragma unroll 1
      for (int mm0 = sw; mm0 < 128; mm0 += 16) {
        float gv[4][kHD / 32];
#pragma unroll
        for (int k = 0; k < 4; k++) {
          const int mm = mm0 + 4 * k, hq = mm >> 5, r = mm & 31;
#pragma unroll
          for (int i = 0; i < kHD / 32; i++)
            gv[k][i] = r < nr ? io.gate(row0 + r, kvh * kGroup + hq, lane + 32 * i) : 0.f;
        }
#pragma unroll
        for (int k = 0; k < 4; k++) {
          const int mm = mm0 + 4 * k, hq = mm >> 5, r = mm & 31;
          if (r >= nr) continue;
#pragma unroll
          for (int i = 0; i < kHD / 32; i++) {
            const int d = lane + 32 * i;
            io.store(row0 + r, kvh * kGroup + hq, d, stage[mm * kStageStride + d] * sigmoidf_(gv[k][i]));
          }
        }
      }
    } else {
      ok = false;
    }
  }

  if (!ok) atomicExch(&s_fail, 1);
  __syncthreads();
  if (s_fail) {
    if (!ok) atomicAdd(timeouts, 1u);
    if (tid == 0) {  // copies still in flight land before the CTA exits (bounded)
      if (kfills) tc::mbar_wait(&bar[B_KFULL], (kfills - 1) & 1);
      for (int b = 0; b < 2; b++)
        if (vfills[b]) tc::mbar_wait(&bar[B_VF0 + b], (vfills[b] - 1) & 1);
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (warp == 1) tc::tmem_dealloc(tmem, 512);
}


// The paged cache [pages][Hkv][page_size][256] bf16 as a 2-D tensor (dim, page row); box (64 dims, 64 rows),
// 128-byte swizzle: one box is one dim block of a 64-token tile.
evie_status cache_map(CUtensorMap* m, const void* base, long rows) {
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return fail(EVIE_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  const cuuint64_t dims[2] = {(cuuint64_t)kHD, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)kHD * 2};
  const cuuint32_t box[2] = {64, (cuuint32_t)kTok};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(EVIE_ERR_CUDA, "cuTensorMapEncodeTiled (KV cache) failed (%d)", (int)r);
  return EVIE_OK;
}

template <class IO>
evie_status launch(const IO& io, const SegInfo* segs, int nseg, int max_seg_rows, const int* page_table,
                   int pages_per_slot, const __nv_bfloat16* kc, const __nv_bfloat16* vc, long cache_rows, int Hkv,
                   int page_size, float scale, cudaStream_t st) {
  if (nseg == 0 || max_seg_rows == 0) return EVIE_OK;
  if (page_size % kTok != 0) return fail(EVIE_ERR_ARG, "prefill attention: page size must be a multiple of %d", kTok);
  if (((uintptr_t)kc | (uintptr_t)vc) & 15) return fail(EVIE_ERR_ARG, "prefill attention: KV pages 16-byte aligned");
  CUtensorMap mk, mv;
  EVIE_TRY(cache_map(&mk, kc, cache_rows));
  EVIE_TRY(cache_map(&mv, vc, cache_rows));
  unsigned int* counter = device_timeout_counter();
  if (!counter) return fail(EVIE_ERR_CUDA, "device timeout counter unavailable");
  auto* kern = gqa_prefill_tc_kernel<IO>;
  EVIE_TRY(max_dynamic_smem((const void*)kern, (int)kSmem));
  dim3 grid((max_seg_rows + kRows - 1) / kRows, nseg, Hkv);
  EVIE_CUDA_TRY(launch_k(kern, dim3(grid), dim3(kThreads), kSmem, st, mk, mv, io, segs, page_table, pages_per_slot, Hkv, page_size, scale * kLog2e,
                                      counter));
  EVIE_CHECK_LAUNCH("gqa_prefill_tc_kernel");
  return EVIE_OK;
}

// Per-(device, stream) device copy of the isolated op's segment table, grown on demand and kept.
struct SegBuf {
  SegInfo* p = nullptr;
  size_t n = 0;
};
std::mutex g_seg_mu;
std::map<std::pair<int, cudaStream_t>, SegBuf> g_segs;

}  // namespace

evie_status launch_gqa_prefill_tc_model(const float* q_rot, YView y, int ldy, __nv_bfloat16* X2, size_t xplane,
                                        const SegInfo* segs, int nseg, int max_seg_rows, const int* page_table,
                                        int pages_per_slot, const __nv_bfloat16* kc, const __nv_bfloat16* vc,
                                        long cache_rows, int Hq, int Hkv, int page_size, float scale,
                                        cudaStream_t st) {
  if (Hq != kGroup * Hkv) return fail(EVIE_ERR_ARG, "prefill attention: GQA group %d not supported (4)", Hq / Hkv);
  const ModelIO io{q_rot, y, ldy, X2, xplane, Hq};
  return launch(io, segs, nseg, max_seg_rows, page_table, pages_per_slot, kc, vc, cache_rows, Hkv, page_size, scale,
                st);
}

}  // namespace evie

extern "C" evie_status evie_gqa_prefill_paged(const float* q, const float* gate, const void* k_pages,
                                              const void* v_pages, int num_pages, const int32_t* page_table,
                                              int max_pages, const int32_t* seq_rows, const int32_t* seq_pos0,
                                              int n_seqs, float* out, int Hq, int Hkv, int hd, int page_size,
                                              float scale, void* stream) {
  using namespace evie;
  if (hd != kHD) return fail(EVIE_ERR_ARG, "evie_gqa_prefill_paged: head_dim 256 only, got %d", hd);
  if (Hkv <= 0 || Hq != kGroup * Hkv) return fail(EVIE_ERR_ARG, "evie_gqa_prefill_paged: Hq must be 4 x Hkv");
  if (n_seqs < 0 || num_pages <= 0 || max_pages <= 0) return fail(EVIE_ERR_ARG, "evie_gqa_prefill_paged: bad sizes");
  if (n_seqs == 0) return EVIE_OK;
  if (!q || !gate || !k_pages || !v_pages || !page_table || !seq_rows || !seq_pos0 || !out)
    return fail(EVIE_ERR_ARG, "evie_gqa_prefill_paged: null pointer");
  if (((uintptr_t)q | (uintptr_t)gate) & 15) return fail(EVIE_ERR_ARG, "evie_gqa_prefill_paged: q, gate 16-byte aligned");
  std::vector<SegInfo> h(n_seqs);
  int start = 0, max_rows = 0;
  for (int s = 0; s < n_seqs; s++) {
    if (seq_rows[s] < 0 || seq_pos0[s] < 0 || (long)seq_pos0[s] + seq_rows[s] > (long)max_pages * page_size)
      return fail(EVIE_ERR_ARG, "evie_gqa_prefill_paged: sequence %d does not fit its %d pages", s, max_pages);
    h[s] = SegInfo{s, start, seq_rows[s], seq_pos0[s]};
    start += seq_rows[s];
    max_rows = std::max(max_rows, seq_rows[s]);
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int dev = 0;
  EVIE_CUDA_TRY(cudaGetDevice(&dev));
  SegInfo* d = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_seg_mu);
    SegBuf& b = g_segs[{dev, st}];
    if (b.n < (size_t)n_seqs) {
      if (b.p) {
        EVIE_CUDA_TRY(cudaStreamSynchronize(st));
        cudaFree(b.p);
        b.p = nullptr;
        b.n = 0;
      }
      EVIE_CUDA_TRY(cudaMalloc(&b.p, sizeof(SegInfo) * n_seqs));
      b.n = n_seqs;
    }
    d = b.p;
  }
  EVIE_CUDA_TRY(cudaMemcpyAsync(d, h.data(), sizeof(SegInfo) * n_seqs, cudaMemcpyHostToDevice, st));
  // the copy must finish reading h before the function returns
  EVIE_CUDA_TRY(cudaStreamSynchronize(st));
  const IsoIO io{q, gate, out, Hq};
  return launch(io, d, n_seqs, max_rows, page_table, max_pages, static_cast<const __nv_bfloat16*>(k_pages),
                static_cast<const __nv_bfloat16*>(v_pages), (long)num_pages * Hkv * page_size, Hkv, page_size, scale,
                st);
}
