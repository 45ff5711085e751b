// Chunked Gated DeltaNet prefill on sm_100a tensor cores (tcgen05 MMA with TMEM accumulators, TMA tile loads).
//
// The recurrence is evie-core's token-sequential DeltaNet loop (crates/evie-core/src/model.rs:362-387, recur_body
// model.rs:501-541): per token, S <- exp(g) S + k (beta (v - exp(g) S^T k))^T and o = S^T q with the updated S.
// Grouped into chunks of C = 64 tokens it reads, for one head with S the [dk][dv] state entering the chunk,
// G_t = g_0 + ... + g_t (in-chunk cumulative log decay) and Gam_t = exp(G_t):
//   N[t][s] = beta_t (k_t . k_s) exp(G_t - G_s)          for s < t (strictly lower triangular)
//   T       = (I + N)^-1 diag(beta)                       (blocked forward substitution)
//   U       = T (V - diag(Gam) K S)                       (the chunk's delta rows, [C][dv])
//   O       = diag(Gam) Q S + P U,   P[t][s] = (q_t . k_s) exp(G_t - G_s) for s <= t, else 0
//   S'      = Gam_C S + K^T diag(exp(G_C - G_t)) U
// Only exponentials of differences G_t - G_s with s <= t appear (never exp(-G)), so nothing overflows for any
// chunk length or decay. Exponentials are taken as exp2 of log2-scaled sums.
//
// Precision. q, k, v are bf16 and enter the tensor core exactly (kind::f16, f32 accumulation). Every f32-valued
// operand (S, V - Gam K S, U, exp-weighted U, T, P) is split into bf16 planes hi + lo (x - hi - lo ~ 2^-17 |x|);
// a product with an exact bf16 partner takes two MMAs (hi, lo), a product of two split operands three
// (hi.hi + hi.lo + lo.hi). The result follows the f32 recurrence to ~1e-5 relative.
//
// Work layout. One CTA per (sequence, head), 512 threads in two groups of 8 warps, one CTA per SM (all 512 TMEM
// columns). Two warps share each TMEM lane quarter and split the columns between them.
//   * Chain warps 0-7 carry the state from chunk to chunk. Every S-dependent product is computed transposed, so
//     that M = 128 runs along dv: TMEM lane j is row dv = j of each accumulator; warp w handles lane quarter w % 4
//     and column half w / 4. Thread 0 issues their MMAs and all TMA loads.
//   * Prep warps 8-15 work one chunk ahead on what does not depend on S: the decay sums, [K;Q] K^T (thread 256
//     issues it), N, P and T. They hand a chunk over through two mbarriers, the decays first (BDE, which the
//     chain's output and state staging need) and then T and P (BTR, awaited just before the MMAs that read them).
//     They wait for the chain to release the buffers two chunks later (BCD).
// TMEM columns:
//   [0,128)   S^T f32 [dv][dk], holding Gam_C S entering each chunk's update
//   [128,256) the A operands of the chain's MMAs, bf16 pairs: S^T hi | S^T lo (64 + 64 columns) for S^T [K;Q]^T;
//             then R^T hi | R^T lo (32 + 32) for R^T T^T; then U^T hi | U^T lo | (E U)^T hi | (E U)^T lo
//             (32 each) for U^T P^T and (E U)^T K
//   [256,320) [K;Q] K^T (prep)            [320,448) (S^T [K;Q]^T): (K S)^T and (Q S)^T halves; (P U)^T reuses the
//   (K S)^T half                          [448,512) U^T f32
// Shared memory (1024-aligned offsets):
//   [0, 64K)       q/k tiles, two dk halves of 32 KB: [K0 | Q0 | Q1 | K1], 8 KB each, 128-byte swizzled K-major
//                  (TMA SW128). Chunk c uses K(c&1), Q(c&1); the stacks [K0;Q0] and [Q1;K1] are 128-row operands.
//   [64K, 80K)     v tile [64 t][128 dv] bf16, unswizzled
//   [80K, 112K)    T^T hi/lo, two buffers ([s][t]: the MN-major B operand of U^T = R^T T^T)
//   [112K, 144K)   P hi/lo, two buffers ([t][s] K-major, the B operand of (P U)^T = U^T P^T)
//   [144K, 160K)   f32 [64][64]: N^T above the diagonal; the solve's T11 and N21 T11 below it
//   [160K, +2048)  Gam, exp(G_C - G) (two buffers), G (log2 units), beta, the chain's Gam, mbarriers, TMEM base
//
// Every mbarrier wait is bounded (2 s of %globaltimer) and every group barrier ORs a failure flag, so both warp
// groups leave together. A wait that gives up bumps a device counter (read by evie_poll_device_errors); the CTA
// then drains its outstanding copies and MMAs (bounded again), frees its TMEM and returns.
//
// Model form (the forward pass's prefill, kModel = true). The model's q, k, v are f32 (conv + SiLU + L2 norm); bf16
// q and k move the 0.8B prefill logits by 0.13, so they enter the tensor core split, hi + lo, like every f32
// operand above: the conv kernel writes the two bf16 planes into the bytes of the q/k columns of its f32 output row
// ([2 planes][2 key_dim] bf16 is exactly 2 key_dim floats), and each K/Q tile is loaded in both planes (the lo plane
// 64 KB above the hi plane in shared memory). Every product with K or Q then takes one more MMA: [K;Q] K^T three
// (hi.hi + lo.hi + hi.lo), S^T [K;Q]^T and (E U)^T K three instead of two. V is read in f32 by the chain threads
// straight from the activation rows (the lane that needs V[t][dv] loads it, coalesced along dv, issued at the top of
// the chunk so that the loads overlap the first MMA), which frees the V tile's 16 KB; the output o[t][dv] is written
// in f32 over V[t][dv] by the same thread after it has read it, and the gated RMSNorm runs as a separate row kernel.
// Work items are (segment, value head); value head h reads key head h / ratio. A segment's last chunk loads up to
// 63 rows past its end (rows of the next segment; rows past the call's last row read as zero): they enter only
// through products with exact zeros (beta = 0 past the end zeroes their rows of N and their rows and columns of T,
// so their U rows are 0; the log decay is 0 there, so G and the state's decay stop at the last row; their V reads
// are skipped; their outputs are not stored), so finite neighbours cannot reach this segment's results.
#include <cudaTypedefs.h>

#include <mutex>

#include "common.h"
#include "gdn_chunk.h"
#include "model_kernels.h"
#include "tc.h"
#include "tmap.h"

namespace evie {

__device__ unsigned int g_tc_timeouts;

namespace {

constexpr int kC = 64;
constexpr int kD = 128;
constexpr int kThreads = 512;
constexpr int kGroup = 256;  // threads per warp group

constexpr uint32_t kKQHalf = 32768;
__device__ __forceinline__ uint32_t kslot(int p) { return p ? 24576u : 0u; }
__device__ __forceinline__ uint32_t qslot(int p) { return p ? 16384u : 8192u; }
__device__ __forceinline__ uint32_t stack_off(int p) { return p ? 16384u : 0u; }  // [K0;Q0] or [Q1;K1]
constexpr uint32_t kSmallBytes = 2048;
// Shared-memory map of the two forms. The model form keeps the lo plane of every K/Q tile 64 KB above its hi plane
// and has no V tile: [0, 128K) K/Q, then T^T, P, N^T and the small arrays as in the isolated form.
template <bool kModel>
struct Map {
  static constexpr uint32_t kPlane = kModel ? 65536u : 0u;  // hi -> lo plane of a K/Q tile
  static constexpr uint32_t kOffV = 65536;                   // isolated form only
  static constexpr uint32_t kOffTM = kModel ? 131072u : 81920u;  // buffers 16 KB apart, planes 8 KB apart
  static constexpr uint32_t kOffPM = kOffTM + 32768;            // buffers 16 KB apart, planes 8 KB apart
  static constexpr uint32_t kOffNT = kOffPM + 32768;
  static constexpr uint32_t kOffSmall = kOffNT + 16384;
  static constexpr uint32_t kSmemBytes = kOffSmall + kSmallBytes + 1024;  // + slack to align the base to 1024
  static_assert(kSmemBytes <= 232448, "shared memory map exceeds 227 KB");
  // MMA terms of the products with K or Q: [K;Q] K^T; S^T [K;Q]^T and (E U)^T K (S and E U are split)
  static constexpr int kPrepTerms = kModel ? 3 : 1;
  static constexpr int kChainTerms = kModel ? 3 : 2;
};

constexpr uint32_t kColS = 0, kColSH = 128, kColSL = 192, kColA = 256, kColKQS = 320, kColU = 448;
constexpr uint32_t kColRH = 128, kColRL = 160;                              // R^T, then U^T planes
constexpr uint32_t kColEH = 192, kColEL = 224;                              // (E U)^T planes

// mbarriers
enum { BK0 = 0, BK1, BQ0, BQ1, BV, BMC, BMP, BTR0, BTR1, BCD0, BCD1, BDE0, BDE1, kNumBars };
constexpr uint32_t kChainBar = 1, kPrepBar = 2;  // named barriers of the two warp groups (256 threads each)
constexpr float kLog2e = 1.4426950408889634f;

// Byte offset of 16-byte chunk `c` of row `r` in a K-major tile with 128-byte rows and the 128-byte swizzle.
__device__ __forceinline__ uint32_t swz(int r, int c) {
  return (uint32_t)r * 128u + ((uint32_t)(c ^ (r & 7)) << 4);
}


// 2n floats -> n words of bf16 hi = round(x) and n words of lo = round(x - hi) (round to nearest even, two values
// per conversion), pairs packed low-half-first (x - hi is exact: hi is within half a bf16 unit of x).
template <int N>
__device__ __forceinline__ void split_pairs(const float* x, uint32_t* hi, uint32_t* lo) {
#pragma unroll
  for (int i = 0; i < N; i++) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
    const float2 hf = __bfloat1622float2(h);
    const __nv_bfloat162 l = __floats2bfloat162_rn(x[2 * i] - hf.x, x[2 * i + 1] - hf.y);
    hi[i] = *reinterpret_cast<const uint32_t*>(&h);
    lo[i] = *reinterpret_cast<const uint32_t*>(&l);
  }
}

// 16 f32 (columns 16 q .. 16 q + 15) of row r of a split K-major SW128 tile: hi plane at `tile`, lo plane `plane`
// bytes further.
__device__ __forceinline__ void store_row16(uint8_t* tile, uint32_t plane, int r, int q, const float* x) {
#pragma unroll
  for (int c = 0; c < 2; c++) {
    uint32_t hi[4], lo[4];
    split_pairs<4>(x + 8 * c, hi, lo);
    *reinterpret_cast<uint4*>(tile + swz(r, 2 * q + c)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    *reinterpret_cast<uint4*>(tile + plane + swz(r, 2 * q + c)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
  }
}

// 2^x by the hardware approximation (relative error below 2^-22; results below 2^-126 flush to zero, which only
// drops decay factors that small).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// f32 -> bf16 bits, round to nearest even (finite inputs).
__device__ __forceinline__ uint16_t bf16_rne(float x) {
  const uint32_t u = __float_as_uint(x);
  return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

// Forward substitution on a 32x32 diagonal block of (I + N): x holds the right-hand side on entry and the solution
// on exit. NT[s][t] = N[base+t][base+s] is read as broadcast float4s (row base+s of the f32 N^T array).
__device__ __forceinline__ void forward32(const float* NT, int base, float* x) {
#pragma unroll
  for (int s = 0; s < 32; s++) {
    const float xs = x[s];
    const float* row = NT + (base + s) * kC + base;
#pragma unroll
    for (int t4 = ((s + 1) >> 2) << 2; t4 < 32; t4 += 4) {
      const float4 n = *reinterpret_cast<const float4*>(row + t4);
      if (t4 + 0 > s) x[t4 + 0] = fmaf(-n.x, xs, x[t4 + 0]);
      if (t4 + 1 > s) x[t4 + 1] = fmaf(-n.y, xs, x[t4 + 1]);
      if (t4 + 2 > s) x[t4 + 2] = fmaf(-n.z, xs, x[t4 + 2]);
      if (t4 + 3 > s) x[t4 + 3] = fmaf(-n.w, xs, x[t4 + 3]);
    }
  }
}

struct ChunkArgs {
  // isolated form: [B][T][H] log decays and betas, [B][H][128][128] states, [B][T][H][128] bf16 outputs
  const float* g;
  const float* beta;
  float* state;
  __nv_bfloat16* o;
  int T;
  int H;
  // model form
  const SegInfo* segs;
  YView y;               // the DeltaNet input projection: b and a logits of head h at columns conv_dim + vd + h, + hv
  int ldy;
  const float* neg_a;    // -exp(A_log) per value head
  const float* dt_bias;
  float* act;            // [R][conv_dim]: split q/k planes in the q/k columns, v in f32 (overwritten by o)
  float* rec_state;      // this layer's [hv][128][128] state of slot 0
  size_t rs_slot;        // element stride between slots
  int conv_dim, key_dim, vd, hv, ratio;
  unsigned int* timeouts;
};

template <bool kModel>
__global__ void __launch_bounds__(kThreads, 1)
    gdn_chunk_prefill_kernel(const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mk,
                             const __grid_constant__ CUtensorMap mv, const ChunkArgs a) {
  using L = Map<kModel>;
  pdl_trigger();
  pdl_wait();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = smem_raw + ((1024u - (tc::smem_u32(smem_raw) & 1023u)) & 1023u);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int q4 = warp & 3, hf = (warp >> 2) & 1;  // TMEM lane quarter, column half
  // Work item: (sequence b, head h) in the isolated form; (segment, value head h) in the model form, whose q and k
  // are key head kh = h / ratio's and whose rows start at row0 of the activation rows.
  const int bh = blockIdx.x;
  int b = 0, h, kh, T, row0 = 0;
  float* Sg;  // the head's [dk][dv] state
  if constexpr (kModel) {
    const SegInfo sg = a.segs[bh / a.hv];
    h = bh % a.hv;
    kh = h / a.ratio;
    T = sg.count;
    row0 = sg.start;
    Sg = a.rec_state + (size_t)sg.slot * a.rs_slot + (size_t)h * kD * kD;
  } else {
    b = bh / a.H;
    h = kh = bh % a.H;
    T = a.T;
    Sg = a.state + (size_t)bh * kD * kD;
  }
  const int H = a.H;
  const int nch = (T + kC - 1) / kC;

  float* GamB = reinterpret_cast<float*>(sm + L::kOffSmall);  // [2][64] exp(G_t)
  float* EcB = GamB + 128;                                  // [2][64] exp(G_63 - G_t)
  float* G2 = GamB + 256;                                   // [64] G_t * log2(e) (prep only)
  float* Bs = GamB + 320;                                   // [64] beta_t, 0 past the end of the sequence
  float* GamC = GamB + 384;                                 // [64] the chain's copy of exp(G_t)
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + L::kOffSmall + 1792);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + L::kOffSmall + 1792 + 8 * kNumBars);
  float* NT = reinterpret_cast<float*>(sm + L::kOffNT);

  if (warp == 0) tc::tmem_alloc(tmem_slot, 512);
  if (tid == 0) {
    for (int i = 0; i < kNumBars; i++)
      tc::mbar_init(&bar[i], (i == BTR0 || i == BTR1 || i == BCD0 || i == BCD1) ? kGroup
                             : (i == BDE0 || i == BDE1)                           ? 32
                                                                                  : 1);
    tc::fence_barrier_init();
    tc::prefetch_tmap(&mq);
    if constexpr (!kModel) {  // the model form reads q and k through one map and v by plain loads
      tc::prefetch_tmap(&mk);
      tc::prefetch_tmap(&mv);
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tl = tmem + ((uint32_t)(q4 * 32) << 16);  // this warp's quarter of the TMEM lanes
  // Shared-memory descriptors relative to `sm`: the start address is the low 14-bit field, so adding (offset >> 4)
  // to a base descriptor moves it (addresses stay below 256 KB).
  const uint64_t dK = tc::sdesc_k_sw128(sm);                     // K-major, 128-byte swizzle
  const uint64_t dMnK = tc::sdesc_mn_sw128(sm, kKQHalf, 1024);   // K^T operand (two 64-wide dk blocks)
  const uint64_t dMnT = tc::sdesc_mn_sw128(sm, 8192, 1024);      // T^T operand (one 64-wide block)
  bool ok = true;
  // Barriers with an operation in flight that the issuing thread has not seen complete, and that phase's parity.
  uint32_t pend = 0, ppar = 0;
  auto mark = [&](int i, uint32_t parity) {
    pend |= 1u << i;
    ppar = (ppar & ~(1u << i)) | (parity << i);
  };
  auto wait = [&](int i, uint32_t parity) {
    if (ok && !tc::mbar_wait(&bar[i], parity)) ok = false;
    if (ok && ((pend >> i) & 1u) && ((ppar >> i) & 1u) == parity) pend &= ~(1u << i);
  };

  if (warp < 8) {
    // =================================== chain warps ===================================
    const int dv = q4 * 32 + lane;
    auto issue_kq = [&](int c) {
      const int p = c & 1;
      tc::mbar_arrive_expect_tx(&bar[BK0 + p], kModel ? 32768 : 16384);
      tc::mbar_arrive_expect_tx(&bar[BQ0 + p], kModel ? 32768 : 16384);
      for (int hh = 0; hh < 2; hh++) {
        if constexpr (kModel) {
          // q/k columns of the activation rows as bf16 [row][plane][2 key_dim]: q of key head kh at kh * 128, its k
          // at key_dim + kh * 128
#pragma unroll
          for (int pl = 0; pl < 2; pl++) {
            uint8_t* dst = sm + pl * L::kPlane + hh * kKQHalf;
            tc::tma_load_3d(dst + kslot(p), &mq, &bar[BK0 + p], a.key_dim + kh * kD + hh * 64, pl, row0 + c * kC);
            tc::tma_load_3d(dst + qslot(p), &mq, &bar[BQ0 + p], kh * kD + hh * 64, pl, row0 + c * kC);
          }
        } else {
          tc::tma_load_4d(sm + hh * kKQHalf + kslot(p), &mk, &bar[BK0 + p], hh * 64, h, c * kC, b);
          tc::tma_load_4d(sm + hh * kKQHalf + qslot(p), &mq, &bar[BQ0 + p], hh * 64, h, c * kC, b);
        }
      }
      mark(BK0 + p, (c >> 1) & 1);
      mark(BQ0 + p, (c >> 1) & 1);
    };
    auto issue_v = [&](int c) {
      if constexpr (!kModel) {
        tc::mbar_arrive_expect_tx(&bar[BV], 16384);
        tc::tma_load_4d(sm + L::kOffV, &mv, &bar[BV], 0, h, c * kC, b);
        mark(BV, c & 1);
      }
    };
    if (tid == 0 && nch > 0) {
      issue_kq(0);
      if (nch > 1) issue_kq(1);
      issue_v(0);
    }
    // Model form: V[t][dv] (f32, in the activation rows) for t in [32 hf, 32 hf + 32) of the current chunk, 0 past
    // the segment; the same thread later writes o[t][dv] over it.
    float vr[kModel ? 32 : 1];
    const size_t vcol = kModel ? (size_t)2 * a.key_dim + (size_t)h * kD + dv : 0;
    auto load_v = [&](int c) {
      if constexpr (kModel) {
        const int t0 = c * kC + 32 * hf;
        const float* vp = a.act + (size_t)(row0 + t0) * a.conv_dim + vcol;
#pragma unroll
        for (int i = 0; i < 32; i++) vr[i] = t0 + i < T ? vp[(size_t)i * a.conv_dim] : 0.f;
      }
    };
    uint32_t nmc = 0;  // completions of the chain's MMA barrier seen
    constexpr uint32_t id64 = tc::idesc(1, 1, 128, 64);
    constexpr uint32_t id128 = tc::idesc(1, 1, 128, 128);
    constexpr uint32_t idS = tc::idesc(1, 1, 128, 128, false, true);
    constexpr uint32_t id64t = tc::idesc(1, 1, 128, 64, false, true);  // B operand MN-major (T^T rows)

    // S^T row dv, dk in [64 hf, 64 hf + 64): the split bf16 operand and Gam_C * S^T as the f32 accumulator (or,
    // after the last chunk, S out to global memory).
    auto stage_state = [&](bool from_global, bool last, float gc) {
#pragma unroll 1
      for (int k = 0; k < 2; k++) {
        const int dk0 = 64 * hf + 32 * k;
        float sv[32];
        if (from_global) {
#pragma unroll
          for (int i = 0; i < 32; i++) sv[i] = Sg[(size_t)(dk0 + i) * kD + dv];
        } else {
          tc::tmem_ld32(tl + kColS + dk0, sv);
        }
        if (last) {
#pragma unroll
          for (int i = 0; i < 32; i++) Sg[(size_t)(dk0 + i) * kD + dv] = sv[i];
          continue;
        }
        uint32_t hi[16], lo[16];
        split_pairs<16>(sv, hi, lo);
        tc::tmem_st16u(tl + kColSH + dk0 / 2, hi);
        tc::tmem_st16u(tl + kColSL + dk0 / 2, lo);
#pragma unroll
        for (int i = 0; i < 32; i++) sv[i] *= gc;
        tc::tmem_st32(tl + kColS + dk0, sv);
      }
      tc::tmem_st_wait();
    };

    if (nch > 0) {
      wait(BDE0, 0);  // chunk 0's decays
      if (ok) stage_state(true, false, GamB[63]);
    }
    tc::fence_before_sync();
    if (tc::group_sync_or(kChainBar, kGroup, !ok)) ok = false;
    tc::fence_after_sync();

#pragma unroll 1
    for (int c = 0; c < nch && ok; c++) {
      const int p = c & 1, t0 = c * kC;
      const float* Ec = EcB + 64 * p;
      if (tid < 64) GamC[tid] = GamB[64 * p + tid];  // the chain's own copy: buffer p is released before the outputs
      const uint32_t ks_col = kColKQS + (p ? 64u : 0u), qs_col = kColKQS + (p ? 0u : 64u);
      load_v(c);

      // ---- (K S)^T | (Q S)^T = S^T [stack]^T, A = S^T hi/lo from TMEM; terms (S hi, KQ hi), (S lo, KQ hi) and,
      // with split K/Q, (S hi, KQ lo)
      if (tid == 0) {
        wait(BK0 + p, (c >> 1) & 1);
        wait(BQ0 + p, (c >> 1) & 1);
        tc::fence_after_sync();
        if (ok) {
#pragma unroll
          for (int tm = 0; tm < L::kChainTerms; tm++)
#pragma unroll
            for (int s = 0; s < 8; s++)
              tc::mma_f16_ts(tmem + kColKQS, tmem + (tm == 1 ? kColSL : kColSH) + s * 8,
                             dK + (((s >> 2) * kKQHalf + stack_off(p) + (s & 3) * 32 + (tm == 2 ? L::kPlane : 0u)) >> 4),
                             id128, (tm | s) > 0);
          tc::mma_commit(&bar[BMC]);
          mark(BMC, nmc & 1);
        }
      }
      wait(BMC, nmc & 1);
      nmc++;
      if constexpr (!kModel) wait(BV, c & 1);
      if (tc::group_sync_or(kChainBar, kGroup, !ok)) { ok = false; break; }
      tc::fence_after_sync();

      // ---- R^T row dv, t in [32 hf, 32 hf + 32): V[t][dv] - Gam_t (K S)^T[dv][t], split into TMEM
      {
        const __nv_bfloat16* V = reinterpret_cast<const __nv_bfloat16*>(sm + L::kOffV);
        float r[32];
        tc::tmem_ld32(tl + ks_col + 32 * hf, r);
#pragma unroll
        for (int i = 0; i < 32; i++) {
          const int t = 32 * hf + i;
          float v;
          if constexpr (kModel) v = vr[i];
          else v = __bfloat162float(V[t * kD + dv]);
          r[i] = fmaf(-GamC[t], r[i], v);
        }
        uint32_t hi[16], lo[16];
        split_pairs<16>(r, hi, lo);
        tc::tmem_st16u(tl + kColRH + 16 * hf, hi);
        tc::tmem_st16u(tl + kColRL + 16 * hf, lo);
        tc::tmem_st_wait();
      }
      tc::fence_before_sync();
      if (tc::group_sync_or(kChainBar, kGroup, !ok)) { ok = false; break; }
      tc::fence_after_sync();

      // ---- U^T = R^T T^T (three passes; A from TMEM, B = T^T rows MN-major); T and P of this chunk from the prep
      wait(BTR0 + p, (c >> 1) & 1);
      if (tid == 0 && ok) {
        if (c + 1 < nch) issue_v(c + 1);  // V has been consumed
        const uint32_t tm = L::kOffTM + p * 16384;
        int n = 0;
#pragma unroll
        for (int pa = 0; pa < 2; pa++)
#pragma unroll
          for (int pb = 0; pb < 2; pb++) {
            if (pa & pb) continue;
#pragma unroll
            for (int s = 0; s < 4; s++, n++)
              tc::mma_f16_ts(tmem + kColU, tmem + (pa ? kColRL : kColRH) + s * 8,
                             dMnT + ((tm + pb * 8192 + s * 2048) >> 4), id64t, n > 0);
          }
        tc::mma_commit(&bar[BMC]);
        mark(BMC, nmc & 1);
      }
      wait(BMC, nmc & 1);
      nmc++;
      if (tc::group_sync_or(kChainBar, kGroup, !ok)) { ok = false; break; }
      tc::fence_after_sync();

      // ---- U^T and (exp(G_C - G_t) U)^T as split TMEM operands
      {
        float u[32];
        tc::tmem_ld32(tl + kColU + 32 * hf, u);
        uint32_t hi[16], lo[16];
        split_pairs<16>(u, hi, lo);
        tc::tmem_st16u(tl + kColRH + 16 * hf, hi);
        tc::tmem_st16u(tl + kColRL + 16 * hf, lo);
#pragma unroll
        for (int i = 0; i < 32; i++) u[i] *= Ec[32 * hf + i];
        split_pairs<16>(u, hi, lo);
        tc::tmem_st16u(tl + kColEH + 16 * hf, hi);
        tc::tmem_st16u(tl + kColEL + 16 * hf, lo);
        tc::tmem_st_wait();
      }
      tc::fence_before_sync();
      if (tc::group_sync_or(kChainBar, kGroup, !ok)) { ok = false; break; }
      tc::fence_after_sync();

      // ---- (P U)^T = U^T P^T (three passes, into the (K S)^T half); S^T += (E U)^T K (K as MN-major operand;
      // terms (E U hi, K hi), (E U lo, K hi) and, with split K, (E U hi, K lo))
      if (tid == 0) {
        const uint32_t pm = L::kOffPM + p * 16384;
        int n = 0;
#pragma unroll
        for (int pa = 0; pa < 2; pa++)
#pragma unroll
          for (int pb = 0; pb < 2; pb++) {
            if (pa & pb) continue;
#pragma unroll
            for (int s = 0; s < 4; s++, n++)
              tc::mma_f16_ts(tmem + ks_col, tmem + (pa ? kColRL : kColRH) + s * 8,
                             dK + ((pm + pb * 8192 + s * 32) >> 4), id64, n > 0);
          }
#pragma unroll
        for (int tm = 0; tm < L::kChainTerms; tm++)
#pragma unroll
          for (int s = 0; s < 4; s++)
            tc::mma_f16_ts(tmem + kColS, tmem + (tm == 1 ? kColEL : kColEH) + s * 8,
                           dMnK + ((kslot(p) + s * 2048 + (tm == 2 ? L::kPlane : 0u)) >> 4), idS, 1);
        tc::mma_commit(&bar[BMC]);
        mark(BMC, nmc & 1);
      }
      wait(BMC, nmc & 1);
      nmc++;
      // K/Q slot p was read by this chunk's MMAs (all complete) and by the prep's [stack] K^T of this chunk
      // (consumed before it handed over T): refill it now, so the load overlaps the rest of the prep's next chunk.
      if (tid == 0 && ok && c + 2 < nch) issue_kq(c + 2);
      tc::mbar_arrive(&bar[BCD0 + p]);  // T, P, Ec of this chunk are consumed: prep may refill buffer p
      const bool last = c + 1 == nch;
      // The output and the staging of the state need only the next chunk's decays (its T and P are awaited before
      // they are read), so this stage overlaps the prep's N, P and T of the next chunk.
      if (!last) wait(BDE0 + (p ^ 1), ((c + 1) >> 1) & 1);
      if (tc::group_sync_or(kChainBar, kGroup, !ok)) { ok = false; break; }
      tc::fence_after_sync();

      // ---- o_t = Gam_t (Q S)^T + (P U)^T for t in [32 hf, 32 hf + 32); the new state staged for the next chunk
      {
        const int nt = min(kC, T - t0);
        float ov[32], qs[32];
        tc::tmem_ld32x2(tl + ks_col + 32 * hf, tl + qs_col + 32 * hf, ov, qs);
        if constexpr (kModel) {
          float* og = a.act + (size_t)(row0 + t0) * a.conv_dim + vcol;  // over V[t][dv], which this thread read
#pragma unroll
          for (int i = 0; i < 32; i++) {
            const int t = 32 * hf + i;
            if (t < nt) og[(size_t)t * a.conv_dim] = fmaf(GamC[t], qs[i], ov[i]);
          }
        } else {
          __nv_bfloat16* og = a.o + (((size_t)b * T + t0) * H + h) * kD + dv;
#pragma unroll
          for (int i = 0; i < 32; i++) {
            const int t = 32 * hf + i;
            if (t < nt) reinterpret_cast<uint16_t*>(og)[(size_t)t * H * kD] = bf16_rne(fmaf(GamC[t], qs[i], ov[i]));
          }
        }
        stage_state(false, last, last ? 1.f : GamB[64 * (p ^ 1) + 63]);
      }
      tc::fence_before_sync();
      if (tc::group_sync_or(kChainBar, kGroup, !ok)) { ok = false; break; }
      tc::fence_after_sync();
    }
    if (!ok && tid == 0) {
      // Drain the copies and MMAs still in flight before shared memory and TMEM are released.
      for (int i = 0; i < kNumBars; i++)
        if ((pend >> i) & 1u) tc::mbar_wait(&bar[i], (ppar >> i) & 1u);
    }
  } else {
    // =================================== prep warps ===================================
    const int pt = tid - kGroup, pw = warp - 8;
    float gn0 = 0.f, gn1 = 0.f, bn0 = 0.f, bn1 = 0.f;  // warp 8: decay and beta of the next chunk, 2 tokens a lane
    auto fetch = [&](int c) {
      const int t = c * kC + 2 * lane;
      if constexpr (kModel) {
        // model.rs:374-375: log decay g = -exp(A_log) softplus(a + dt_bias), beta = sigmoid(b)
        const float na = a.neg_a[h], dtb = a.dt_bias[h];
        const size_t col = (size_t)a.conv_dim + a.vd + h, r = (size_t)(row0 + t) * a.ldy + col;
        gn0 = t < T ? na * softplus_(a.y.at(r + a.hv) + dtb) : 0.f;
        bn0 = t < T ? sigmoidf_(a.y.at(r)) : 0.f;
        gn1 = t + 1 < T ? na * softplus_(a.y.at(r + a.ldy + a.hv) + dtb) : 0.f;
        bn1 = t + 1 < T ? sigmoidf_(a.y.at(r + a.ldy)) : 0.f;
      } else {
        const size_t r = ((size_t)b * T + t) * H + h;
        gn0 = t < T ? __ldg(a.g + r) : 0.f;
        bn0 = t < T ? __ldg(a.beta + r) : 0.f;
        gn1 = t + 1 < T ? __ldg(a.g + r + H) : 0.f;
        bn1 = t + 1 < T ? __ldg(a.beta + r + H) : 0.f;
      }
    };
    if (pw == 0 && nch > 0) fetch(0);
    constexpr uint32_t idA = tc::idesc(1, 1, 128, 64);
    auto issue_a = [&](int c) {  // thread 256 issues [stack] K^T of chunk c into the A accumulator
      if (pt != 0) return;
      const int p = c & 1;
      wait(BK0 + p, (c >> 1) & 1);
      wait(BQ0 + p, (c >> 1) & 1);
      tc::fence_after_sync();
      if (!ok) return;
      // terms (stack hi, K hi) and, with split K/Q, (stack lo, K hi), (stack hi, K lo)
#pragma unroll
      for (int tm = 0; tm < L::kPrepTerms; tm++)
#pragma unroll
        for (int s = 0; s < 8; s++) {
          const uint32_t kb = (s >> 2) * kKQHalf + (s & 3) * 32;
          const uint32_t pa = tm == 1 ? L::kPlane : 0u, pb = tm == 2 ? L::kPlane : 0u;
          tc::mma_f16(tmem + kColA, dK + ((kb + stack_off(p) + pa) >> 4), dK + ((kb + kslot(p) + pb) >> 4), idA,
                      (tm | s) > 0);
        }
      tc::mma_commit(&bar[BMP]);
      mark(BMP, c & 1);
    };
    if (nch > 0) issue_a(0);

#pragma unroll 1
    for (int c = 0; c < nch && ok; c++) {
      const int p = c & 1;
      float* Gam = GamB + 64 * p;  // chunk c's decays, read by the chain
      float* Ec = EcB + 64 * p;
      uint8_t* TM = sm + L::kOffTM + p * 16384;
      uint8_t* PM = sm + L::kOffPM + p * 16384;
      if (c >= 2) wait(BCD0 + p, ((c >> 1) - 1) & 1);  // the chain is done with chunk c-2's buffers

      // ---- decay sums (log2 units) and beta; warp 8, two tokens a lane
      if (pw == 0) {
        const float a0 = gn0 * kLog2e, a1 = a0 + gn1 * kLog2e;
        float inc = a1;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
          const float y = __shfl_up_sync(0xffffffffu, inc, off);
          if (lane >= off) inc += y;
        }
        const float e0 = inc - a1 + a0, e1 = inc;
        const float lst = __shfl_sync(0xffffffffu, e1, 31);
        G2[2 * lane] = e0;
        G2[2 * lane + 1] = e1;
        Bs[2 * lane] = bn0;
        Bs[2 * lane + 1] = bn1;
        Gam[2 * lane] = ex2(e0);
        Gam[2 * lane + 1] = ex2(e1);
        Ec[2 * lane] = ex2(lst - e0);
        Ec[2 * lane + 1] = ex2(lst - e1);
        tc::mbar_arrive(&bar[BDE0 + p]);  // this chunk's decays are ready for the chain
        if (c + 1 < nch) fetch(c + 1);
      }

      // ---- [stack] K^T (issued at the end of the previous chunk's prep, or before the loop)
      wait(BMP, c & 1);
      if (tc::group_sync_or(kPrepBar, kGroup, !ok)) { ok = false; break; }
      tc::fence_after_sync();

      // ---- N (f32, transposed, above the diagonal of NT) and P (split): row r, s in [32 hf, 32 hf + 32)
      {
        const bool k_rows = (p == 0) == (q4 < 2);  // which lane half holds K K^T this chunk
        const int r = (q4 & 1) * 32 + lane;
        const float gr = G2[r], br = Bs[r];
        float row[32];
        tc::tmem_ld32(tl + kColA + 32 * hf, row);
        if (k_rows) {
#pragma unroll
          for (int i = 0; i < 32; i++) {
            const int s = 32 * hf + i;
            if (s < r) NT[s * kC + r] = br * row[i] * ex2(gr - G2[s]);
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; i++) {
            const int s = 32 * hf + i;
            row[i] = s <= r ? row[i] * ex2(gr - G2[s]) : 0.f;
          }
          store_row16(PM, 8192, r, 2 * hf, row);
          store_row16(PM, 8192, r, 2 * hf + 1, row + 16);
        }
      }
      tc::fence_proxy_async();
      tc::fence_before_sync();
      if (tc::group_sync_or(kPrepBar, kGroup, !ok)) { ok = false; break; }
      tc::fence_after_sync();

      // ---- T = (I + N)^-1 diag(beta) in 32-blocks: T11, T22 (diagonal solves), then T21 from N21 T11.
      // TM holds T^T: row s (128 bytes, swizzled) = column s of T, read by the MMA as an MN-major B operand.
      float t11[32];  // warp 8: column `lane` of T11, kept for the row write after T21
      if (pt < 64) {
        const int blk = pt >> 5, j = pt & 31, base = 32 * blk;
        float x[32];
#pragma unroll
        for (int t = 0; t < 32; t++) x[t] = t == j ? Bs[base + t] : 0.f;
        forward32(NT, base, x);
        if (blk == 0) {
#pragma unroll
          for (int t = 0; t < 32; t++) {
            if (t >= j) NT[t * kC + j] = x[t];  // T11, below the diagonal of NT
            t11[t] = x[t];
          }
        } else {
          float zero[16];
#pragma unroll
          for (int i = 0; i < 16; i++) zero[i] = 0.f;
          store_row16(TM, 8192, 32 + j, 0, zero);
          store_row16(TM, 8192, 32 + j, 1, zero);
          store_row16(TM, 8192, 32 + j, 2, x);
          store_row16(TM, 8192, 32 + j, 3, x + 16);
        }
      }
      if (tc::group_sync_or(kPrepBar, kGroup, !ok)) { ok = false; break; }
      {
        // Y = N21 T11: warp pw covers columns 4 pw .. 4 pw + 3, lane = row of the second block
        const int j0 = 4 * pw;
        float y[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 8
        for (int s = 0; s < 32; s++) {
          const float n = NT[s * kC + 32 + lane];
          const float4 tv = *reinterpret_cast<const float4*>(NT + s * kC + j0);
          if (s >= j0 + 0) y[0] = fmaf(n, tv.x, y[0]);
          if (s >= j0 + 1) y[1] = fmaf(n, tv.y, y[1]);
          if (s >= j0 + 2) y[2] = fmaf(n, tv.z, y[2]);
          if (s >= j0 + 3) y[3] = fmaf(n, tv.w, y[3]);
        }
        if (tc::group_sync_or(kPrepBar, kGroup, false)) { ok = false; break; }  // all reads of T11 rows done
        *reinterpret_cast<float4*>(NT + (32 + lane) * kC + j0) = make_float4(y[0], y[1], y[2], y[3]);
      }
      if (tc::group_sync_or(kPrepBar, kGroup, !ok)) { ok = false; break; }
      if (pt < 32) {
        // (I + N22) T21 = -N21 T11, column j = lane
        float x[32];
#pragma unroll
        for (int t = 0; t < 32; t++) x[t] = -NT[(32 + t) * kC + lane];
        forward32(NT, 32, x);
        store_row16(TM, 8192, lane, 0, t11);
        store_row16(TM, 8192, lane, 1, t11 + 16);
        store_row16(TM, 8192, lane, 2, x);
        store_row16(TM, 8192, lane, 3, x + 16);
      }
      tc::fence_proxy_async();
      tc::mbar_arrive(&bar[BTR0 + p]);  // T and P of chunk c are ready
      // The A accumulator was consumed by this chunk's N/P: start the next chunk's [stack] K^T now, so that it runs
      // while the buffers are awaited and the decays summed. (The chain loads its K/Q tiles once chunk c-1's MMAs
      // are complete, which needs only chunk c-1's hand-over: no wait here depends on the prep itself.)
      if (c + 1 < nch) issue_a(c + 1);
    }
    if (!ok && pt == 0 && ((pend >> BMP) & 1u)) tc::mbar_wait(&bar[BMP], (ppar >> BMP) & 1u);
  }

  if (!ok && (tid == 0 || tid == kGroup)) atomicAdd(a.timeouts, 1u);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (warp == 0) tc::tmem_dealloc(tmem, 512);
}


// [B][T][H][128] bf16 viewed as a 4-D tensor (d, head, token, sequence); box = (box_d, 1, 64, 1).
evie_status token_major_map(CUtensorMap* m, const void* base, int B, int T, int H, uint32_t box_d,
                            CUtensorMapSwizzle swizzle) {
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return fail(EVIE_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  const cuuint64_t dims[4] = {(cuuint64_t)kD, (cuuint64_t)H, (cuuint64_t)T, (cuuint64_t)B};
  const cuuint64_t strides[3] = {(cuuint64_t)kD * 2, (cuuint64_t)H * kD * 2, (cuuint64_t)T * H * kD * 2};
  const cuuint32_t box[4] = {box_d, 1, (cuuint32_t)kC, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(EVIE_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return EVIE_OK;
}

}  // namespace

unsigned int* device_timeout_counter() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  static unsigned int* ptrs[kMaxDevices] = {};
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  if (!ptrs[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_tc_timeouts) != cudaSuccess) return nullptr;
    ptrs[dev] = static_cast<unsigned int*>(p);
  }
  return ptrs[dev];
}

evie_status launch_gdn_chunk_prefill_bf16(const void* q, const void* k, const void* v, const float* g,
                                          const float* beta, float* state, void* o, int B, int T, int H,
                                          cudaStream_t st) {
  if ((long)B * H == 0 || T == 0) return EVIE_OK;
  CUtensorMap mq, mk, mv;
  evie_status s;
  if ((s = token_major_map(&mq, q, B, T, H, 64, CU_TENSOR_MAP_SWIZZLE_128B)) != EVIE_OK) return s;
  if ((s = token_major_map(&mk, k, B, T, H, 64, CU_TENSOR_MAP_SWIZZLE_128B)) != EVIE_OK) return s;
  if ((s = token_major_map(&mv, v, B, T, H, 128, CU_TENSOR_MAP_SWIZZLE_NONE)) != EVIE_OK) return s;
  unsigned int* counter = device_timeout_counter();
  if (!counter) return fail(EVIE_ERR_CUDA, "device timeout counter unavailable");
  constexpr uint32_t smem = Map<false>::kSmemBytes;
  EVIE_TRY(max_dynamic_smem((const void*)gdn_chunk_prefill_kernel<false>, (int)smem));
  ChunkArgs a{};
  a.g = g;
  a.beta = beta;
  a.state = state;
  a.o = static_cast<__nv_bfloat16*>(o);
  a.T = T;
  a.H = H;
  a.timeouts = counter;
  gdn_chunk_prefill_kernel<false><<<B * H, kThreads, smem, st>>>(mq, mk, mv, a);
  EVIE_CHECK_LAUNCH("gdn_chunk_prefill_kernel");
  return EVIE_OK;
}

evie_status launch_gdn_chunk_model(float* act, YView y, int ldy, int R, const SegInfo* segs, int nseg,
                                   float* rec_state, size_t rs_slot, const float* neg_a, const float* dt_bias,
                                   int conv_dim, int key_dim, int vd, int hv, int hk, cudaStream_t st) {
  if (nseg == 0 || R == 0) return EVIE_OK;
  if (hk <= 0 || hv % hk != 0 || key_dim != hk * kD || vd != hv * kD || conv_dim != 2 * key_dim + vd)
    return fail(EVIE_ERR_ARG, "chunked DeltaNet prefill: head dims must be 128 with value heads a multiple of key heads");
  if (((uintptr_t)act & 15u) != 0)
    return fail(EVIE_ERR_ARG, "chunked DeltaNet prefill: activation rows must be 16-byte aligned");
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return fail(EVIE_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  // The q/k columns of the activation rows as bf16 [R][2 planes][2 key_dim]; box = 64 elements x 1 plane x 64 rows.
  CUtensorMap m;
  const cuuint64_t dims[3] = {(cuuint64_t)2 * key_dim, 2, (cuuint64_t)R};
  const cuuint64_t strides[2] = {(cuuint64_t)2 * key_dim * 2, (cuuint64_t)conv_dim * 4};
  const cuuint32_t box[3] = {64, 1, (cuuint32_t)kC};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = enc(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, act, dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(EVIE_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  unsigned int* counter = device_timeout_counter();
  if (!counter) return fail(EVIE_ERR_CUDA, "device timeout counter unavailable");
  constexpr uint32_t smem = Map<true>::kSmemBytes;
  EVIE_TRY(max_dynamic_smem((const void*)gdn_chunk_prefill_kernel<true>, (int)smem));
  ChunkArgs a{};
  a.segs = segs;
  a.y = y;
  a.ldy = ldy;
  a.neg_a = neg_a;
  a.dt_bias = dt_bias;
  a.act = act;
  a.rec_state = rec_state;
  a.rs_slot = rs_slot;
  a.conv_dim = conv_dim;
  a.key_dim = key_dim;
  a.vd = vd;
  a.hv = hv;
  a.ratio = hv / hk;
  a.timeouts = counter;
  EVIE_CUDA_TRY(launch_k(gdn_chunk_prefill_kernel<true>, dim3(nseg * hv), dim3(kThreads), smem, st, m, m, m, a));
  EVIE_CHECK_LAUNCH("gdn_chunk_prefill_kernel<model>");
  return EVIE_OK;
}

namespace {

// One thread waits, bounded by `limit_ns`, on an mbarrier that nothing arrives at. That is the path every bounded
// wait of these kernels takes when a copy or an MMA never completes: the wait gives up and the thread counts it
// in the device counter that evie_poll_device_errors reads.
__global__ void bounded_wait_probe_kernel(uint64_t limit_ns, unsigned int* timeouts, int* gave_up) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x != 0) return;
  tc::mbar_init(&bar, 1);
  tc::fence_barrier_init();
  const bool done = tc::mbar_wait_for(&bar, 0, limit_ns);
  *gave_up = done ? 0 : 1;
  if (!done) atomicAdd(timeouts, 1u);
}

}  // namespace

}  // namespace evie

extern "C" evie_status evie_bounded_wait_probe(uint64_t limit_ns, int* gave_up) {
  if (!gave_up) return evie::fail(EVIE_ERR_ARG, "evie_bounded_wait_probe: null output");
  if (limit_ns > evie::tc::kWaitNs)
    return evie::fail(EVIE_ERR_ARG, "evie_bounded_wait_probe: limit above %llu ns",
                      (unsigned long long)evie::tc::kWaitNs);
  unsigned int* counter = evie::device_timeout_counter();
  if (!counter) return evie::fail(EVIE_ERR_CUDA, "device timeout counter unavailable");
  int* d = nullptr;
  EVIE_CUDA_TRY(cudaMalloc(&d, sizeof(int)));
  evie::bounded_wait_probe_kernel<<<1, 32>>>(limit_ns, counter, d);
  cudaError_t rc = cudaGetLastError();
  int h = -1;
  if (rc == cudaSuccess) rc = cudaMemcpy(&h, d, sizeof h, cudaMemcpyDeviceToHost);
  cudaFree(d);
  if (rc != cudaSuccess) return evie::fail(EVIE_ERR_CUDA, "evie_bounded_wait_probe: %s", cudaGetErrorString(rc));
  *gave_up = h;
  return EVIE_OK;
}

extern "C" evie_status evie_poll_device_errors(void) {
  unsigned int* p = evie::device_timeout_counter();
  if (!p) return evie::fail(EVIE_ERR_CUDA, "device timeout counter unavailable");
  unsigned int n = 0;
  EVIE_CUDA_TRY(cudaDeviceSynchronize());
  EVIE_CUDA_TRY(cudaMemcpy(&n, p, sizeof n, cudaMemcpyDeviceToHost));
  if (n) {
    const unsigned int zero = 0;
    EVIE_CUDA_TRY(cudaMemcpy(p, &zero, sizeof zero, cudaMemcpyHostToDevice));
    return evie::fail(EVIE_ERR_TIMEOUT, "%u thread(s) gave up a bounded device-side wait since the last poll", n);
  }
  return EVIE_OK;
}
