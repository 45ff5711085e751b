// Chunked Gated DeltaNet prefill on sm_100a tensor cores (tcgen05 MMA with TMEM accumulators, TMA tile loads).
//
// The recurrence is evie-core's token-sequential DeltaNet loop (crates/evie-core/src/model.rs:362-387, recur_body
// model.rs:501-541): per token, S <- exp(g) S + k (beta (v - exp(g) S^T k))^T and o = S^T q with the updated S.
// Grouped into chunks of C = 64 tokens it reads, for one head with S the [dk][dv] state entering the chunk,
// G_t = g_0 + ... + g_t (in-chunk cumulative log decay) and Gam_t = exp(G_t):
//   N[t][s] = beta_t (k_t . k_s) exp(G_t - G_s)          for s < t (strictly lower triangular)
//   T       = (I + N)^-1 diag(beta)                       (forward substitution)
//   U       = T (V - diag(Gam) K S)                       (the chunk's delta rows, [C][dv])
//   O       = diag(Gam) Q S + P U,   P[t][s] = (q_t . k_s) exp(G_t - G_s) for s <= t, else 0
//   S'      = Gam_C S + K^T diag(exp(G_C - G_t)) U
// Only exponentials of differences G_t - G_s with s <= t appear (never exp(-G)), so nothing overflows for any
// chunk length or decay.
//
// Precision. q, k, v are bf16 and enter the tensor core exactly (kind::f16, f32 accumulation). Every f32-valued
// operand (S, V - Gam K S, U, exp-weighted U, T, P) is split into bf16 planes hi + lo (x - hi - lo ~ 2^-17 |x|);
// a product with an exact bf16 partner takes two MMAs (hi, lo), a product of two split operands three
// (hi.hi + hi.lo + lo.hi). The result follows the f32 recurrence to ~1e-5 relative.
//
// Work layout. One CTA per (sequence, head), 128 threads, one CTA per SM (it takes 226 KB of shared memory and all
// 512 TMEM columns). Every S-dependent product is computed transposed, so that M = 128 runs along dv and thread j
// (TMEM lane j) owns row dv = j of each accumulator:
//   TMEM [0,128)   S^T           [dv][dk]   persistent across chunks, rescaled by Gam_C in place
//        [128,192) [K;Q] K^T     lanes 0-63 / 64-127 = the two stacked 64-row operands, columns = s
//        [192,256) (K S)^T       [dv][t]
//        [256,320) (Q S)^T       [dv][t]
//        [320,384) U^T           [dv][t]
//        [384,448) (P U)^T       [dv][t]
// Shared memory (1024-aligned offsets):
//   [0, 48K)        q/k tiles, two dk halves of 24 KB: [K slot 0 | Q | K slot 1], 8 KB each, 128-byte swizzled
//                   K-major (TMA SW128). K is double-buffered so the next chunk's K loads during this one; the
//                   stacked [K;Q] (even chunks) or [Q;K] (odd chunks) is one 128-row MMA operand.
//   [48K, 64K)      v tile [64 t][128 dv] bf16, unswizzled (read by the epilogue threads only)
//   [64K, 128K)     S^T hi / lo planes (MMA A operand, [dv][dk] K-major, two 64-wide dk atoms)
//   [128K, 160K)    R^T = (V - Gam K S)^T hi/lo, then U^T hi/lo ([dv][t] K-major)
//   [160K, 192K)    (exp(G_C - G_t) U)^T hi/lo; earlier in the chunk the f32 N^T for the forward substitution
//   [192K, 208K)    T hi/lo ([t][s] K-major, the B operand of U^T = R^T T^T)
//   [208K, 224K)    P hi/lo ([t][s] K-major, the B operand of (P U)^T = U^T P^T)
//   [224K, +1152)   G, Gam, exp(G_C - G), beta (64 f32 each), mbarriers, TMEM base
//
// Every mbarrier wait is bounded (2 s of %globaltimer). A wait that gives up bumps a device counter (read by
// evie_poll_device_errors), makes the CTA drain its outstanding copies and MMAs (bounded again), free its TMEM and
// return.
#include <cudaTypedefs.h>

#include <mutex>

#include "common.h"
#include "gdn_chunk.h"
#include "tc.h"

namespace evie {

__device__ unsigned int g_tc_timeouts;

namespace {

constexpr int kC = 64;
constexpr int kD = 128;
constexpr int kThreads = 128;

constexpr uint32_t kKQHalf = 24576;  // one dk half of the q/k area
constexpr uint32_t kSlotQ = 8192;
__device__ __forceinline__ constexpr uint32_t kslot(int parity) { return parity ? 16384u : 0u; }  // K slots
constexpr uint32_t kOffV = 49152;
constexpr uint32_t kOffST = 65536;   // planes 32 KB apart, dk halves 16 KB apart
constexpr uint32_t kOffRU = 131072;  // planes 16 KB apart
constexpr uint32_t kOffEU = 163840;  // planes 16 KB apart
constexpr uint32_t kOffTM = 196608;  // planes 8 KB apart
constexpr uint32_t kOffPM = 212992;  // planes 8 KB apart
constexpr uint32_t kOffSmall = 229376;
constexpr uint32_t kSmallBytes = 1152;
constexpr uint32_t kSmemBytes = kOffSmall + kSmallBytes + 1024;  // + slack to align the base to 1024
static_assert(kSmemBytes <= 232448, "shared memory map exceeds 227 KB");

constexpr uint32_t kColS = 0, kColA = 128, kColKS = 192, kColQS = 256, kColU = 320, kColO = 384;

// Byte offset of 16-byte chunk `c` of row `r` in a K-major tile with 128-byte rows and the 128-byte swizzle.
__device__ __forceinline__ uint32_t swz(int r, int c) {
  return (uint32_t)r * 128u + ((uint32_t)(c ^ (r & 7)) << 4);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo_addr, float hi_addr) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo_addr, hi_addr);
  return *reinterpret_cast<uint32_t*>(&v);
}

// 8 floats -> bf16 hi = round(x) and lo = round(x - hi), 8 each packed in a uint4.
__device__ __forceinline__ void split8(const float* x, uint4& hi, uint4& lo) {
  float h[8], l[8];
#pragma unroll
  for (int i = 0; i < 8; i++) {
    h[i] = __bfloat162float(__float2bfloat16_rn(x[i]));
    l[i] = x[i] - h[i];
  }
  hi = make_uint4(pack_bf16x2(h[0], h[1]), pack_bf16x2(h[2], h[3]), pack_bf16x2(h[4], h[5]), pack_bf16x2(h[6], h[7]));
  lo = make_uint4(pack_bf16x2(l[0], l[1]), pack_bf16x2(l[2], l[3]), pack_bf16x2(l[4], l[5]), pack_bf16x2(l[6], l[7]));
}

// Row r (64 f32) of a split K-major SW128 tile: hi plane at `tile`, lo plane `plane` bytes further.
__device__ __forceinline__ void store_row64(uint8_t* tile, uint32_t plane, int r, const float* x) {
#pragma unroll
  for (int c = 0; c < 8; c++) {
    uint4 hi, lo;
    split8(x + 8 * c, hi, lo);
    *reinterpret_cast<uint4*>(tile + swz(r, c)) = hi;
    *reinterpret_cast<uint4*>(tile + plane + swz(r, c)) = lo;
  }
}

// 16 consecutive dk (dk0 a multiple of 16) of row dv of the split S^T operand.
__device__ __forceinline__ void store_st16(uint8_t* sm, int dv, int dk0, const float* x) {
  uint8_t* base = sm + kOffST + (dk0 >> 6) * 16384;
#pragma unroll
  for (int cc = 0; cc < 2; cc++) {
    uint4 hi, lo;
    split8(x + 8 * cc, hi, lo);
    const uint32_t off = swz(dv, ((dk0 & 63) >> 3) + cc);
    *reinterpret_cast<uint4*>(base + off) = hi;
    *reinterpret_cast<uint4*>(base + 32768 + off) = lo;
  }
}

__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float* v) {
#pragma unroll
  for (int i = 0; i < 4; i++) tc::tmem_ld16(taddr + 16 * i, v + 16 * i);
}

// T = (I + N)^-1 diag(beta), column j, by forward substitution (right-looking: once T[s][j] is known it is pushed
// into the partial sums of every later row). N^T[s][t] = N[t][s] is read as broadcast float4s.
__device__ __forceinline__ void solve_T_column(uint8_t* sm, const float* Bs, int j) {
  const float* NT = reinterpret_cast<const float*>(sm + kOffEU);
  float x[kC];
#pragma unroll
  for (int t = 0; t < kC; t++) x[t] = 0.f;
#pragma unroll
  for (int s = 0; s < kC; s++) {
    x[s] = (s == j ? Bs[s] : 0.f) - x[s];
#pragma unroll
    for (int t4 = ((s + 1) >> 2) << 2; t4 < kC; t4 += 4) {
      const float4 n = *reinterpret_cast<const float4*>(NT + s * kC + t4);
      if (t4 + 0 > s) x[t4 + 0] = fmaf(n.x, x[s], x[t4 + 0]);
      if (t4 + 1 > s) x[t4 + 1] = fmaf(n.y, x[s], x[t4 + 1]);
      if (t4 + 2 > s) x[t4 + 2] = fmaf(n.z, x[s], x[t4 + 2]);
      if (t4 + 3 > s) x[t4 + 3] = fmaf(n.w, x[s], x[t4 + 3]);
    }
  }
  uint8_t* tm = sm + kOffTM;
#pragma unroll
  for (int s = 0; s < kC; s++) {
    const __nv_bfloat16 hi = __float2bfloat16_rn(x[s]);
    const __nv_bfloat16 lo = __float2bfloat16_rn(x[s] - __bfloat162float(hi));
    const uint32_t off = (uint32_t)s * 128u + ((uint32_t)((j >> 3) ^ (s & 7)) << 4) + (uint32_t)(j & 7) * 2u;
    *reinterpret_cast<__nv_bfloat16*>(tm + off) = hi;
    *reinterpret_cast<__nv_bfloat16*>(tm + 8192 + off) = lo;
  }
}

// R^T row dv = V[:, dv] - Gam (K S)^T[dv, :], split into the R^T operand.
__device__ __forceinline__ void compute_R_row(uint8_t* sm, uint32_t tl, const float* Gam, int dv) {
  float r[kC];
  tmem_ld64(tl + kColKS, r);
  const __nv_bfloat16* V = reinterpret_cast<const __nv_bfloat16*>(sm + kOffV);
#pragma unroll
  for (int t = 0; t < kC; t++) r[t] = fmaf(-Gam[t], r[t], __bfloat162float(V[t * kD + dv]));
  store_row64(sm + kOffRU, 16384, dv, r);
}

struct ChunkArgs {
  const float* g;
  const float* beta;
  float* state;
  __nv_bfloat16* o;
  int T;
  int H;
  unsigned int* timeouts;
};

__global__ void __launch_bounds__(kThreads, 1)
    gdn_chunk_prefill_kernel(const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mk,
                             const __grid_constant__ CUtensorMap mv, const ChunkArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = smem_raw + ((1024u - (tc::smem_u32(smem_raw) & 1023u)) & 1023u);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bh = blockIdx.x, b = bh / a.H, h = bh % a.H;
  const int T = a.T, H = a.H;
  const int nch = (T + kC - 1) / kC;

  float* Gs = reinterpret_cast<float*>(sm + kOffSmall);  // cumulative log decay within the chunk
  float* Gam = Gs + 64;                                  // exp(G_t)
  float* Ec = Gs + 128;                                  // exp(G_63 - G_t)
  float* Bs = Gs + 192;                                  // beta_t (0 past the end of the sequence)
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + kOffSmall + 1024);  // K slot 0, K slot 1, Q, V, MMA
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + kOffSmall + 1024 + 64);

  if (warp == 0) tc::tmem_alloc(tmem_slot, 512);
  if (tid == 0) {
    for (int i = 0; i < 5; i++) tc::mbar_init(&bar[i], 1);
    tc::fence_barrier_init();
    tc::prefetch_tmap(&mq);
    tc::prefetch_tmap(&mk);
    tc::prefetch_tmap(&mv);
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tl = tmem + ((uint32_t)(warp * 32) << 16);  // this warp's quarter of the TMEM lanes

  // Completion counts per barrier: issued (thread 0) and observed (every thread); parity = observed & 1.
  uint32_t issued[5] = {0, 0, 0, 0, 0}, seen[5] = {0, 0, 0, 0, 0};
  bool ok = true;
  auto wait = [&](int i) {  // after a failure nothing more is waited for; `seen` counts completions observed
    if (ok && !tc::mbar_wait(&bar[i], seen[i] & 1)) ok = false;
    if (ok) seen[i]++;
  };
  auto issue_k = [&](int c) {
    uint64_t* bb = &bar[c & 1];
    tc::mbar_arrive_expect_tx(bb, 16384);
    for (int hf = 0; hf < 2; hf++) tc::tma_load_4d(sm + hf * kKQHalf + kslot(c & 1), &mk, bb, hf * 64, h, c * kC, b);
    issued[c & 1]++;
  };
  auto issue_q = [&](int c) {
    tc::mbar_arrive_expect_tx(&bar[2], 16384);
    for (int hf = 0; hf < 2; hf++) tc::tma_load_4d(sm + hf * kKQHalf + kSlotQ, &mq, &bar[2], hf * 64, h, c * kC, b);
    issued[2]++;
  };
  auto issue_v = [&](int c) {
    tc::mbar_arrive_expect_tx(&bar[3], 16384);
    tc::tma_load_4d(sm + kOffV, &mv, &bar[3], 0, h, c * kC, b);
    issued[3]++;
  };

  if (tid == 0 && nch > 0) {
    issue_k(0);
    issue_q(0);
    issue_v(0);
  }

  // Entering state: thread j takes column j of S ([dk][dv]) = row j of S^T, into TMEM and the split operand.
  float* Sg = a.state + (size_t)bh * kD * kD;
#pragma unroll 1
  for (int c16 = 0; c16 < 8; c16++) {
    float col[16];
#pragma unroll
    for (int i = 0; i < 16; i++) col[i] = Sg[(size_t)(c16 * 16 + i) * kD + tid];
    tc::tmem_st16(tl + kColS + c16 * 16, col);
    store_st16(sm, tid, c16 * 16, col);
  }
  tc::tmem_st_wait();
  tc::fence_proxy_async();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();

  constexpr uint32_t id64 = tc::idesc(1, 1, 128, 64);
  constexpr uint32_t idS = tc::idesc(1, 1, 128, 128, false, true);
  bool aborted = false;

#pragma unroll 1
  for (int c = 0; c < nch; c++) {
    const int p = c & 1, t0 = c * kC;

    // ---- decay and beta of this chunk; cumulative sums over the 64 tokens
    if (tid < 64) {
      const int t = t0 + tid;
      float gv = 0.f, bv = 0.f;
      if (t < T) {
        const size_t r = ((size_t)b * T + t) * H + h;
        gv = __ldg(a.g + r);
        bv = __ldg(a.beta + r);
      }
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, gv, off);
        if (lane >= off) gv += y;
      }
      Gs[tid] = gv;
      Bs[tid] = bv;
    }
    __syncthreads();
    if (tid >= 32 && tid < 64) Gs[tid] += Gs[31];
    __syncthreads();
    if (tid < 64) {
      Gam[tid] = expf(Gs[tid]);
      Ec[tid] = expf(Gs[63] - Gs[tid]);
    }

    // ---- this chunk's q, k, v tiles
    wait(p);
    wait(2);
    wait(3);
    if (__syncthreads_or(!ok)) { aborted = true; break; }

    // ---- MMA: [K;Q] K^T, (K S)^T, (Q S)^T
    if (tid == 0) {
      tc::fence_after_sync();
      const uint32_t stack = p == 0 ? kslot(0) : kSlotQ;  // [K;Q] on even chunks, [Q;K] on odd ones
#pragma unroll
      for (int s = 0; s < 8; s++) {
        const uint32_t kb = (s >> 2) * kKQHalf + (s & 3) * 32;
        tc::mma_f16(tmem + kColA, tc::sdesc_k_sw128(sm + kb + stack), tc::sdesc_k_sw128(sm + kb + kslot(p)), id64,
                    s > 0);
      }
#pragma unroll
      for (int pl = 0; pl < 2; pl++)
#pragma unroll
        for (int s = 0; s < 8; s++) {
          const uint64_t ad = tc::sdesc_k_sw128(sm + kOffST + pl * 32768 + (s >> 2) * 16384 + (s & 3) * 32);
          const uint32_t kb = (s >> 2) * kKQHalf + (s & 3) * 32;
          tc::mma_f16(tmem + kColKS, ad, tc::sdesc_k_sw128(sm + kb + kslot(p)), id64, (pl | s) > 0);
          tc::mma_f16(tmem + kColQS, ad, tc::sdesc_k_sw128(sm + kb + kSlotQ), id64, (pl | s) > 0);
        }
      tc::mma_commit(&bar[4]);
      issued[4]++;
      if (c + 1 < nch) issue_k(c + 1);  // the other K slot was last read by the previous chunk's S update
    }
    wait(4);
    if (__syncthreads_or(!ok)) { aborted = true; break; }
    tc::fence_after_sync();
    if (tid == 0 && c + 1 < nch) issue_q(c + 1);  // Q has been consumed

    // ---- N (forward-substitution matrix, transposed, f32) and P (split), one row per thread
    {
      const bool k_rows = (p == 0) == (warp < 2);  // which lane half holds K K^T this chunk
      const int r = tid & 63;
      float row[kC];
      tmem_ld64(tl + kColA, row);
      const float Gr = Gs[r];
      if (k_rows) {
        float* NT = reinterpret_cast<float*>(sm + kOffEU);
        const float br = Bs[r];
#pragma unroll
        for (int s = 0; s < kC; s++) NT[s * kC + r] = s < r ? br * row[s] * expf(Gr - Gs[s]) : 0.f;
      } else {
#pragma unroll
        for (int s = 0; s < kC; s++) row[s] = s <= r ? row[s] * expf(Gr - Gs[s]) : 0.f;
        store_row64(sm + kOffPM, 8192, r, row);
      }
    }
    tc::fence_proxy_async();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();

    // ---- T (warps 0-1, one column each) while warps 2-3 form R^T for dv 64..127; then R^T for dv 0..63
    if (warp < 2) solve_T_column(sm, Bs, tid);
    compute_R_row(sm, tl, Gam, tid);
    tc::fence_proxy_async();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();

    // ---- MMA: U^T = R^T T^T (three passes)
    if (tid == 0) {
      if (c + 1 < nch) issue_v(c + 1);  // V has been consumed
      int n = 0;
#pragma unroll
      for (int pa = 0; pa < 2; pa++)
#pragma unroll
        for (int pb = 0; pb < 2; pb++) {
          if (pa & pb) continue;
#pragma unroll
          for (int s = 0; s < 4; s++, n++)
            tc::mma_f16(tmem + kColU, tc::sdesc_k_sw128(sm + kOffRU + pa * 16384 + s * 32),
                        tc::sdesc_k_sw128(sm + kOffTM + pb * 8192 + s * 32), id64, n > 0);
        }
      tc::mma_commit(&bar[4]);
      issued[4]++;
    }
    wait(4);
    if (__syncthreads_or(!ok)) { aborted = true; break; }
    tc::fence_after_sync();

    // ---- U^T and the exp-weighted U^T as split operands; S^T <- Gam_C S^T in TMEM
    {
      float u[kC];
      tmem_ld64(tl + kColU, u);
      store_row64(sm + kOffRU, 16384, tid, u);
#pragma unroll
      for (int t = 0; t < kC; t++) u[t] *= Ec[t];
      store_row64(sm + kOffEU, 16384, tid, u);
      const float gc = Gam[63];
#pragma unroll 1
      for (int c16 = 0; c16 < 8; c16++) {
        float sv[16];
        tc::tmem_ld16(tl + kColS + c16 * 16, sv);
#pragma unroll
        for (int i = 0; i < 16; i++) sv[i] *= gc;
        tc::tmem_st16(tl + kColS + c16 * 16, sv);
      }
      tc::tmem_st_wait();
    }
    tc::fence_proxy_async();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();

    // ---- MMA: (P U)^T = U^T P^T (three passes); S^T += (E U)^T K (two passes, K as an MN-major operand)
    if (tid == 0) {
      int n = 0;
#pragma unroll
      for (int pa = 0; pa < 2; pa++)
#pragma unroll
        for (int pb = 0; pb < 2; pb++) {
          if (pa & pb) continue;
#pragma unroll
          for (int s = 0; s < 4; s++, n++)
            tc::mma_f16(tmem + kColO, tc::sdesc_k_sw128(sm + kOffRU + pa * 16384 + s * 32),
                        tc::sdesc_k_sw128(sm + kOffPM + pb * 8192 + s * 32), id64, n > 0);
        }
#pragma unroll
      for (int pa = 0; pa < 2; pa++)
#pragma unroll
        for (int s = 0; s < 4; s++)
          tc::mma_f16(tmem + kColS, tc::sdesc_k_sw128(sm + kOffEU + pa * 16384 + s * 32),
                      tc::sdesc_mn_sw128(sm + kslot(p) + s * 2048, kKQHalf, 1024), idS, 1);
      tc::mma_commit(&bar[4]);
      issued[4]++;
    }
    wait(4);
    if (__syncthreads_or(!ok)) { aborted = true; break; }
    tc::fence_after_sync();

    // ---- outputs o_t = Gam_t (Q S)^T + (P U)^T; the new S^T into the split operand (or out, after the last chunk)
    {
      __nv_bfloat16* og = a.o + (((size_t)b * T + t0) * H + h) * kD + tid;
      const int nt = min(kC, T - t0);
#pragma unroll 1
      for (int c16 = 0; c16 < 4; c16++) {
        float ov[16], qs[16];
        tc::tmem_ld16(tl + kColO + c16 * 16, ov);
        tc::tmem_ld16(tl + kColQS + c16 * 16, qs);
#pragma unroll
        for (int i = 0; i < 16; i++) {
          const int t = c16 * 16 + i;
          if (t < nt) og[(size_t)t * H * kD] = __float2bfloat16_rn(fmaf(Gam[t], qs[i], ov[i]));
        }
      }
      const bool last = c + 1 == nch;
#pragma unroll 1
      for (int c16 = 0; c16 < 8; c16++) {
        float sv[16];
        tc::tmem_ld16(tl + kColS + c16 * 16, sv);
        if (last) {
#pragma unroll
          for (int i = 0; i < 16; i++) Sg[(size_t)(c16 * 16 + i) * kD + tid] = sv[i];
        } else {
          store_st16(sm, tid, c16 * 16, sv);
        }
      }
    }
    tc::fence_proxy_async();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
  }

  if (aborted && tid == 0) {
    atomicAdd(a.timeouts, 1u);
    // Drain what this CTA still has in flight before its shared memory and TMEM are released.
    for (int i = 0; i < 5; i++) {
      uint32_t done = seen[i];
      while (done < issued[i] && tc::mbar_wait(&bar[i], done & 1)) done++;
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (warp == 0) tc::tmem_dealloc(tmem, 512);
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
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
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  static unsigned int* ptrs[64] = {};
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
  int dev = 0;
  EVIE_CUDA_TRY(cudaGetDevice(&dev));
  static bool attr_set[64] = {};
  if (dev < 64 && !attr_set[dev]) {
    EVIE_CUDA_TRY(
        cudaFuncSetAttribute(gdn_chunk_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes));
    attr_set[dev] = true;
  }
  ChunkArgs a{g, beta, state, static_cast<__nv_bfloat16*>(o), T, H, counter};
  gdn_chunk_prefill_kernel<<<B * H, kThreads, kSmemBytes, st>>>(mq, mk, mv, a);
  EVIE_CHECK_LAUNCH("gdn_chunk_prefill_kernel");
  return EVIE_OK;
}

}  // namespace evie

extern "C" evie_status evie_poll_device_errors(void) {
  unsigned int* p = evie::device_timeout_counter();
  if (!p) return evie::fail(EVIE_ERR_CUDA, "device timeout counter unavailable");
  unsigned int n = 0;
  EVIE_CUDA_TRY(cudaDeviceSynchronize());
  EVIE_CUDA_TRY(cudaMemcpy(&n, p, sizeof n, cudaMemcpyDeviceToHost));
  if (n) {
    const unsigned int zero = 0;
    EVIE_CUDA_TRY(cudaMemcpy(p, &zero, sizeof zero, cudaMemcpyHostToDevice));
    return evie::fail(EVIE_ERR_TIMEOUT, "%u CTA(s) gave up a bounded device-side wait since the last poll", n);
  }
  return EVIE_OK;
}
