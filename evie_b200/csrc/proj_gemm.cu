// Projection GEMM on sm_100a tensor cores: Y = X W^T for bf16 weights W [M][K] and f32 activations X [R][K] given as
// two bf16 planes (hi = bf16(X), lo = bf16(X - hi)). This is evie-core's `matmul` (crates/evie-core/src/kernels.rs
// :138-268: bf16 weights widened to f32, f32 activations, f32 sums) for every projection of the forward pass
// (model.rs:240-264, 305-312, 395, 402-404) and the LM head (model.rs:287-294).
//
// Tiles. The weight rows are the MMA's M side (two M = 128 halves per 256-row tile, each its own accumulator) and
// the activation rows its N side (BR = 16, 64 or 128 rows). One K step of 64 elements is a 128-byte row, so every
// operand tile is a TMA box in the 128-byte swizzle and a K-major UMMA descriptor. The hi and lo operand tiles sit
// next to each other in shared memory; for decode-shaped tiles one MMA per K = 16 step and half covers both
// (N = 2 BR, hi and lo products in separate accumulator columns, added by the epilogue), so the weight sub-tile is
// read from shared memory once. Shared-memory bandwidth is what limits these MMAs: with separate hi and lo MMAs the
// tensor core re-reads every weight sub-tile. Prefill tiles (128 weight rows x 256 activation rows, N = 256) issue
// D += W . lo^T and then D += W . hi^T into the same columns; against 256 x 128 tiles they move ~8% fewer
// shared-memory bytes per FLOP (TMA stores of the tiles plus the MMAs' reads: ~172 against ~187 bytes per
// tensor-core cycle, of ~128 available), and a prefill call's projections take 8% less time. Either way the result
// leaves as one plane.
//
// Accumulation groups. The tensor core rounds each MMA's addition into the f32 accumulator toward zero, so an
// accumulator carried over all of K drifts by about (MMA steps) x half an ulp of its own magnitude: -1.8e-5
// relative at K = 9216 (measured against float64). The accumulator is therefore restarted every `gchunks` K steps
// of 64 (4 for decode tiles, 8 for prefill tiles), in a ring of tensor-memory buffers (2 or 4), and the epilogue
// warps add each group's partial sums into f32 registers with round-to-nearest. The drift measured -2e-7 relative
// on decode shapes and -9e-7 on the prefill tiles (cuBLAS on the two planes: -2e-6 to -9e-6).
//
// Roles (320 threads, one CTA per SM): warp 0 lane 0 issues the TMA loads into a ring of stages (full / empty
// mbarriers); warp 1 owns tensor memory and lane 0 issues the MMAs; warps 2-9 drain the accumulator groups with
// tcgen05.ld into register sums and, once a tile's K range is done, store f32 rows of Y: warp w covers the 32 TMEM
// lanes (weight rows) of lane quarter w % 4 and one half of the tile's activation columns, 128 contiguous bytes
// per activation row.
//
// Work units are (K slice, M tile, R tile), K slice fastest. Decode-shaped calls (R <= 128, one R tile) cut K into
// slices until the units fill the SMs: each slice writes its own plane and the consumer adds the planes in slice
// order. Larger R runs one slice over a persistent grid of 128 x 256 tiles, in bands of ~40 MB of weight tiles (M
// fastest, then R), so that a band's weights stay in L2 while every operand tile passes through it.
//
// Programmatic dependent launch: the weights do not depend on the previous kernel, so the producer issues the weight
// half of its first ring fill, then waits (griddepcontrol.wait) for the previous grid, then loads the activations.
// With the previous kernel triggering its dependents early, the first weight tiles stream while it finishes.
//
// Every mbarrier wait is bounded (2 s); a thread that gives up stops its loop, bumps the device timeout counter,
// and the CTA drains its copies and MMAs (bounded again) before it frees tensor memory and exits.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <map>
#include <mutex>
#include <tuple>

#include "gdn_chunk.h"
#include "proj_gemm.h"
#include "tc.h"
#include "tmap.h"

namespace evie {

namespace {

constexpr int kKC = 64;        // K elements per stage: one 128-byte swizzled row per operand row
constexpr int kThreads = 320;  // warp 0 producer, warp 1 MMA + TMEM owner, warps 2-9 epilogue
constexpr int kEpiThreads = 256;
constexpr uint32_t kRingBudget = 196608;

struct GemmArgs {
  float* y;      // [planes][R][M]
  size_t plane;  // R * M
  int M, R, K, kc, ksplit, n_mt, n_rt, band, units;
  int gchunks;  // K steps of 64 per accumulation group
  unsigned int* timeouts;
  int evict_first;  // weights read once per call (decode): L2 evict-first; otherwise evict-last
};

template <int BM, int BR>
struct Cfg {
  static constexpr uint32_t kWBytes = BM * 128;
  static constexpr uint32_t kXBytes = BR * 128;  // one operand plane
  static constexpr uint32_t kStage = kWBytes + 2 * kXBytes;
  static constexpr int kStagesRaw = (int)(kRingBudget / kStage);
  static constexpr int kStages = kStagesRaw > 8 ? 8 : kStagesRaw;
  static constexpr int kHalves = BM / 128;
  // Stacked: one MMA per K step and half with N = 2 BR over the adjacent hi and lo tiles (hi products in accumulator
  // columns [0, BR), lo products in [BR, 2 BR)), so the weight sub-tile is read from shared memory once for both
  // planes. Otherwise (prefill tiles, whose stacked accumulator would not leave room for two buffers) two MMAs
  // per K step accumulate lo and then hi into the same columns.
  static constexpr bool kStack = 2 * kHalves * 2 * BR <= 512;
  static constexpr int kPlaneCols = kStack ? BR : 0;      // column offset of the lo products
  static constexpr uint32_t kAccCols = kHalves * (kStack ? 2 * BR : BR);  // one accumulator buffer
  static constexpr int kBufs = kAccCols <= 128 ? 4 : 2;  // accumulator buffers in flight between MMA and epilogue
  static constexpr int kCT = BR / 2;                     // activation columns per epilogue thread and half
  static constexpr int kPiece = kCT < 32 ? kCT : 32;     // columns per tcgen05.ld
  static constexpr uint32_t kTmemRaw = kBufs * kAccCols;
  static constexpr uint32_t kTmemCols = kTmemRaw < 32 ? 32 : kTmemRaw;
  static constexpr uint32_t kBarOff = kStages * kStage;
  static constexpr uint32_t kSmem = kBarOff + 256 + 1024;  // + barriers, + slack to align the base to 1024
  static_assert(kStage % 1024 == 0, "stage tiles must keep 1024-byte alignment");
  static_assert(kTmemCols >= 32 && kTmemCols <= 512 && (kTmemCols & (kTmemCols - 1)) == 0, "TMEM allocation");
  static_assert(kSmem <= 232448, "shared memory");
  static_assert(2 * kStages + 2 * kBufs + 1 <= 30, "barrier area");
};

struct Unit {
  int ks, mt, rt, c0, c1;
};
// Unit u -> (K slice, M tile, R tile). Tiles go in bands of `band` M tiles: within a band the M tile is fastest and
// the R tile next, so the CTAs working at the same time share a band's weights (sized to stay in L2) and a few
// operand tiles, and the weights are read from DRAM once per call, the operand once per band.
__device__ __forceinline__ Unit unit_of(const GemmArgs& a, int u) {
  Unit x;
  x.ks = u % a.ksplit;
  const int t = u / a.ksplit;
  const int per_band = a.band * a.n_rt;
  const int b = t / per_band, v = t - b * per_band;
  const int cnt = min(a.band, a.n_mt - b * a.band);
  x.rt = v / cnt;
  x.mt = b * a.band + v % cnt;
  x.c0 = (int)((long)x.ks * a.kc / a.ksplit);
  x.c1 = (int)((long)(x.ks + 1) * a.kc / a.ksplit);
  return x;
}

template <int BM, int BR>
__global__ void __launch_bounds__(kThreads, 1)
    proj_gemm_kernel(const __grid_constant__ CUtensorMap mw, const __grid_constant__ CUtensorMap mx,
                     const GemmArgs a) {
  using C = Cfg<BM, BR>;
  constexpr int S = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;
  uint64_t* tempty = tfull + C::kBufs;
  uint64_t* drain = tempty + C::kBufs;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  __shared__ int s_fail;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // The next kernel may launch now; it waits for this grid's completion before it reads what this grid writes.
  tc::griddep_launch_dependents();
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; s++) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < C::kBufs; b++) {
      tc::mbar_init(&tfull[b], 1);
      tc::mbar_init(&tempty[b], kEpiThreads);
    }
    tc::mbar_init(drain, 1);
    s_fail = 0;
    tc::fence_barrier_init();
    tc::prefetch_tmap(&mw);
    tc::prefetch_tmap(&mx);
  }
  if (warp == 1) tc::tmem_alloc(tmem_slot, C::kTmemCols);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;
  int fills[8] = {0, 0, 0, 0, 0, 0, 0, 0};  // producer: times each stage was armed

  if (warp == 0) {
    if (lane == 0) {
      // ---- TMA producer
      const uint64_t pol = a.evict_first ? tc::l2_evict_first() : tc::l2_evict_last();
      int it = 0, npend = 0;
      int pend_k[8], pend_r[8];
      bool waited = false;
      auto flush = [&]() {  // the previous grid is complete: load the activation halves of the first ring fill
        tc::griddep_wait();
        waited = true;
        for (int i = 0; i < npend; i++) {
          uint8_t* st = smem + (uint32_t)i * C::kStage;
          tc::tma_load_3d(st + C::kWBytes, &mx, &full[i], pend_k[i], pend_r[i], 0);
          tc::tma_load_3d(st + C::kWBytes + C::kXBytes, &mx, &full[i], pend_k[i], pend_r[i], 1);
        }
        npend = 0;
      };
      for (int u = blockIdx.x; u < a.units && ok; u += gridDim.x) {
        const Unit x = unit_of(a, u);
        for (int c = x.c0; c < x.c1; c++, it++) {
          const int s = it % S, j = it / S;
          if (j >= 1) {
            if (!waited) flush();
            if (!tc::mbar_wait(&empty[s], (j - 1) & 1)) {
              ok = false;
              break;
            }
          }
          uint8_t* st = smem + (uint32_t)s * C::kStage;
          tc::mbar_arrive_expect_tx(&full[s], C::kStage);
          fills[s]++;
          tc::tma_load_2d_hint(st, &mw, &full[s], c * kKC, x.mt * BM, pol);
          if (waited) {
            tc::tma_load_3d(st + C::kWBytes, &mx, &full[s], c * kKC, x.rt * BR, 0);
            tc::tma_load_3d(st + C::kWBytes + C::kXBytes, &mx, &full[s], c * kKC, x.rt * BR, 1);
          } else {
            pend_k[npend] = c * kKC;
            pend_r[npend] = x.rt * BR;
            npend++;
          }
        }
      }
      if (!waited) flush();
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA issuer
      constexpr uint32_t idesc = tc::idesc(1, 1, 128, C::kStack ? 2 * BR : BR);
      int it = 0, grp = 0;
      for (int u = blockIdx.x; u < a.units && ok; u += gridDim.x) {
        const Unit x = unit_of(a, u);
        int b = 0;
        for (int c = x.c0; c < x.c1; c++, it++) {
          const bool first = (c - x.c0) % a.gchunks == 0;
          if (first) {  // a new accumulation group in the next buffer, once the epilogue has drained it
            b = grp % C::kBufs;
            const int ub = grp / C::kBufs;
            if (ub >= 1 && !tc::mbar_wait(&tempty[b], (ub - 1) & 1)) {
              ok = false;
              break;
            }
            tc::fence_after_sync();
          }
          const int s = it % S, j = it / S;
          if (!tc::mbar_wait(&full[s], j & 1)) {
            ok = false;
            break;
          }
          tc::fence_after_sync();
          const uint8_t* st = smem + (uint32_t)s * C::kStage;
          const uint64_t dh = tc::sdesc_k_sw128(st + C::kWBytes);
          const uint64_t dl = tc::sdesc_k_sw128(st + C::kWBytes + C::kXBytes);
#pragma unroll
          for (int h = 0; h < C::kHalves; h++) {
            const uint64_t da = tc::sdesc_k_sw128(st + h * 128 * 128);
            const uint32_t d = tmem + (uint32_t)(b * C::kAccCols + h * (C::kAccCols / C::kHalves));
            if constexpr (C::kStack) {
#pragma unroll
              for (int kk = 0; kk < kKC / 16; kk++)
                tc::mma_f16(d, da + 2 * kk, dh + 2 * kk, idesc, (!first || kk > 0) ? 1u : 0u);
            } else {
#pragma unroll
              for (int kk = 0; kk < kKC / 16; kk++)
                tc::mma_f16(d, da + 2 * kk, dl + 2 * kk, idesc, (!first || kk > 0) ? 1u : 0u);
#pragma unroll
              for (int kk = 0; kk < kKC / 16; kk++) tc::mma_f16(d, da + 2 * kk, dh + 2 * kk, idesc, 1u);
            }
          }
          tc::mma_commit(&empty[s]);  // the stage is free once these MMAs have read it
          if (c + 1 == x.c1 || (c + 1 - x.c0) % a.gchunks == 0) {
            tc::mma_commit(&tfull[b]);  // the group's partial sums are final
            grp++;
          }
        }
      }
      // Every MMA this thread issued is complete before tensor memory is freed.
      tc::mma_commit(drain);
      if (!tc::mbar_wait(drain, 0)) ok = false;
    }
  } else {
    // ---- epilogue: warp w sums TMEM lanes 32 (w % 4) .. + 31 (weight rows) of each half, columns ch * kCT ..
    tc::griddep_wait();
    const int q = warp & 3, ch = (warp - 2) >> 2;
    int grp = 0;
    for (int u = blockIdx.x; u < a.units && ok; u += gridDim.x) {
      const Unit x = unit_of(a, u);
      float acc[C::kHalves][C::kCT];
#pragma unroll
      for (int h = 0; h < C::kHalves; h++)
#pragma unroll
        for (int j = 0; j < C::kCT; j++) acc[h][j] = 0.f;
      const int ngroups = (x.c1 - x.c0 + a.gchunks - 1) / a.gchunks;
      for (int gi = 0; gi < ngroups; gi++, grp++) {
        const int b = grp % C::kBufs, ub = grp / C::kBufs;
        if (!tc::mbar_wait(&tfull[b], ub & 1)) {
          ok = false;
          break;
        }
        tc::fence_after_sync();
#pragma unroll
        for (int h = 0; h < C::kHalves; h++) {
#pragma unroll
          for (int p = 0; p < C::kCT; p += C::kPiece) {
            float v[C::kPiece];
            const uint32_t ta = tmem + ((uint32_t)(q * 32) << 16) +
                                (uint32_t)(b * C::kAccCols + h * (C::kAccCols / C::kHalves) + ch * C::kCT + p);
            if constexpr (C::kPiece == 32) tc::tmem_ld32(ta, v);
            else if constexpr (C::kPiece == 16) tc::tmem_ld16(ta, v);
            else tc::tmem_ld8(ta, v);
            if constexpr (C::kStack) {  // + the lo products of the same columns
              float w[C::kPiece];
              if constexpr (C::kPiece == 32) tc::tmem_ld32(ta + C::kPlaneCols, w);
              else if constexpr (C::kPiece == 16) tc::tmem_ld16(ta + C::kPlaneCols, w);
              else tc::tmem_ld8(ta + C::kPlaneCols, w);
#pragma unroll
              for (int j = 0; j < C::kPiece; j++) v[j] += w[j];
            }
#pragma unroll
            for (int j = 0; j < C::kPiece; j++) acc[h][p + j] += v[j];
          }
        }
        tc::fence_before_sync();
        tc::mbar_arrive(&tempty[b]);
      }
      if (!ok) break;
      float* yb = a.y + (size_t)x.ks * a.plane;
      const int r0 = x.rt * BR + ch * C::kCT;
#pragma unroll
      for (int h = 0; h < C::kHalves; h++) {
        const int m = x.mt * BM + h * 128 + q * 32 + lane;
        if (m < a.M) {
#pragma unroll
          for (int j = 0; j < C::kCT; j++)
            if (r0 + j < a.R) yb[(size_t)(r0 + j) * a.M + m] = acc[h][j];
        }
      }
    }
  }

  if (!ok) atomicExch(&s_fail, 1);
  __syncthreads();
  if (s_fail) {
    if (!ok) atomicAdd(a.timeouts, 1u);
    if (threadIdx.x == 0) {  // copies still in flight land before the CTA exits (bounded)
      for (int s = 0; s < S; s++)
        if (fills[s] > 0) tc::mbar_wait(&full[s], (fills[s] - 1) & 1);
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (warp == 1) tc::tmem_dealloc(tmem, C::kTmemCols);
}


// W [M][K] bf16 as a 2-D tensor (k, m); box (64, bm), 128-byte swizzle, zero fill past M and K.
evie_status weight_map(CUtensorMap* m, const void* W, int M, int K, int bm) {
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return fail(EVIE_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
  const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kKC, (cuuint32_t)bm};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(W), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(EVIE_ERR_CUDA, "cuTensorMapEncodeTiled (weights %d x %d) failed (%d)", M, K, (int)r);
  return EVIE_OK;
}

// X2 [2][R][K] bf16 as a 3-D tensor (k, r, plane); box (64, br, 1), 128-byte swizzle, zero fill past R and K.
evie_status operand_map(CUtensorMap* m, const void* X2, int R, int K, int br) {
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return fail(EVIE_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  const cuuint64_t dims[3] = {(cuuint64_t)K, (cuuint64_t)R, 2};
  const cuuint64_t strides[2] = {(cuuint64_t)K * 2, (cuuint64_t)R * K * 2};
  const cuuint32_t box[3] = {(cuuint32_t)kKC, (cuuint32_t)br, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(X2), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(EVIE_ERR_CUDA, "cuTensorMapEncodeTiled (operand %d x %d) failed (%d)", R, K, (int)r);
  return EVIE_OK;
}

template <int BM, int BR>
evie_status launch_tiles(const __nv_bfloat16* W, const __nv_bfloat16* X2, float* y, const ProjGemmPlan& p, int M,
                         int K, int R, bool pdl, cudaStream_t st) {
  using C = Cfg<BM, BR>;
  CUtensorMap mw, mx;
  EVIE_TRY(weight_map(&mw, W, M, K, BM));
  EVIE_TRY(operand_map(&mx, X2, R, K, BR));
  unsigned int* counter = device_timeout_counter();
  if (!counter) return fail(EVIE_ERR_CUDA, "device timeout counter unavailable");
  auto* kern = proj_gemm_kernel<BM, BR>;
  EVIE_TRY(max_dynamic_smem((const void*)kern, (int)C::kSmem));
  static const int group_env = [] {
    const char* e = getenv("EVIE_GEMM_GROUP");
    return e ? std::max(1, atoi(e)) : 0;
  }();
  // Accumulation group: 4 K steps of 64 for decode tiles (drift -2e-7 relative, within 2% of the fastest setting),
  // 8 for the prefill tiles (-9e-7). EVIE_GEMM_GROUP overrides both.
  const int gchunks = group_env ? group_env : (R > 128 ? 8 : 4);
  const int n_mt = (M + BM - 1) / BM, n_rt = (R + BR - 1) / BR;
  const int band = std::max(1, std::min(n_mt, (int)((40u << 20) / ((size_t)BM * K * 2))));  // ~40 MB of weights
  GemmArgs a{y, (size_t)R * M, M, R, K, (K + kKC - 1) / kKC, p.ksplit, n_mt, n_rt, band, p.units,
             gchunks, counter, R <= 128 ? 1 : 0};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = C::kSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, mw, mx, a);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(EVIE_ERR_CUDA, "launch of proj_gemm_kernel<%d,%d> (%d x %d x %d): %s", BM, BR, M, R, K,
                cudaGetErrorString(e));
  }
  return EVIE_OK;
}

}  // namespace

ProjGemmPlan plan_proj_gemm(int M, int K, int R, int max_planes, size_t y_cap, int num_sms) {
  ProjGemmPlan best;
  const int kc = (K + kKC - 1) / kKC;
  // EVIE_GEMM_PREFILL_NARROW=1 keeps the earlier 256 x 128 prefill tiles, for comparison
  static const bool narrow = [] {
    const char* e = getenv("EVIE_GEMM_PREFILL_NARROW");
    return e && e[0] == '1';
  }();
  if (R > 128) {  // prefill-shaped: persistent 128 x 256 tiles, one K slice
    best.bm = narrow ? 256 : 128;
    best.br = narrow ? 128 : 256;
    best.ksplit = 1;
    best.units = ((M + best.bm - 1) / best.bm) * ((R + best.br - 1) / best.br);
    best.grid = std::min(best.units, num_sms);
    return best;
  }
  const int br = R <= 16 ? 16 : R <= 64 ? 64 : 128;
  double best_util = -1.0;
  for (int bm : {256, 128}) {  // on equal fill the 256-row tiles win: each activation tile is read from L2 once
    if (br == 128 && bm == 128) continue;
    const int tiles = (M + bm - 1) / bm;
    int ks = std::max(1, num_sms / tiles);
    ks = std::min({ks, max_planes, std::max(1, kc / 4)});
    while (ks > 1 && (size_t)ks * R * M > y_cap) ks--;
    const int units = tiles * ks;
    const int waves = (units + num_sms - 1) / num_sms;
    const double util = (double)units / ((double)waves * num_sms);
    if (util > best_util + 0.02) {
      best_util = util;
      best.bm = bm;
      best.br = br;
      best.ksplit = ks;
      best.units = units;
      best.grid = std::min(units, num_sms);
    }
  }
  return best;
}

evie_status launch_proj_gemm(const __nv_bfloat16* W, int M, int K, const __nv_bfloat16* X2, int R, float* y,
                             size_t y_cap, int max_planes, bool pdl, cudaStream_t st, int* planes) {
  // EVIE_GEMM_TILE=<bm>x<slices> (decode-shaped calls, e.g. 128x1) pins the tile plan, for measurements
  static const std::pair<int, int> force = [] {
    const char* e = getenv("EVIE_GEMM_TILE");
    int bm = 0, ks = 0;
    if (e && sscanf(e, "%dx%d", &bm, &ks) == 2 && (bm == 128 || bm == 256) && ks >= 1) return std::make_pair(bm, ks);
    return std::make_pair(0, 0);
  }();
  if (M <= 0 || K <= 0 || R <= 0) return fail(EVIE_ERR_ARG, "proj_gemm: empty shape %d x %d x %d", M, R, K);
  if (K % 8 != 0) return fail(EVIE_ERR_ARG, "proj_gemm: K = %d must be a multiple of 8 (16-byte rows)", K);
  if (((uintptr_t)W | (uintptr_t)X2) & 15) return fail(EVIE_ERR_ARG, "proj_gemm: W and X2 must be 16-byte aligned");
  if (max_planes < 1) return fail(EVIE_ERR_ARG, "proj_gemm: max_planes must be >= 1");
  if ((size_t)R * M > y_cap) return fail(EVIE_ERR_ARG, "proj_gemm: output of %d x %d floats exceeds its buffer", R, M);
  ProjGemmPlan p = plan_proj_gemm(M, K, R, max_planes, y_cap, sm_count());
  if (force.first && R <= 128 && p.br != 128 && (size_t)force.second * R * M <= y_cap) {
    p.bm = force.first;
    p.ksplit = std::min(force.second, std::max(1, (K + kKC - 1) / kKC));
    p.units = ((M + p.bm - 1) / p.bm) * p.ksplit;
    p.grid = std::min(p.units, sm_count());
  }
  evie_status s;
  if (p.bm == 256 && p.br == 128) s = launch_tiles<256, 128>(W, X2, y, p, M, K, R, pdl, st);
  else if (p.bm == 128 && p.br == 256) s = launch_tiles<128, 256>(W, X2, y, p, M, K, R, pdl, st);
  else if (p.bm == 256 && p.br == 64) s = launch_tiles<256, 64>(W, X2, y, p, M, K, R, pdl, st);
  else if (p.bm == 256 && p.br == 16) s = launch_tiles<256, 16>(W, X2, y, p, M, K, R, pdl, st);
  else if (p.bm == 128 && p.br == 64) s = launch_tiles<128, 64>(W, X2, y, p, M, K, R, pdl, st);
  else if (p.bm == 128 && p.br == 16) s = launch_tiles<128, 16>(W, X2, y, p, M, K, R, pdl, st);
  else return fail(EVIE_ERR_ARG, "proj_gemm: no tile configuration for %d x %d x %d", M, R, K);
  if (s != EVIE_OK) return s;
  if (planes) *planes = p.ksplit;
  return EVIE_OK;
}

}  // namespace evie

// Isolated form of the projection GEMM, for tests and callers that hold the split operand themselves.
extern "C" evie_status evie_proj_gemm(const void* w, const void* x2, float* y, size_t y_cap, int M, int K, int R,
                                      int max_planes, int* planes, void* stream) {
  if (!w || !x2 || !y || !planes) return evie::fail(EVIE_ERR_ARG, "evie_proj_gemm: null pointer");
  return evie::launch_proj_gemm(static_cast<const __nv_bfloat16*>(w), M, K, static_cast<const __nv_bfloat16*>(x2), R,
                                y, y_cap, max_planes, false, static_cast<cudaStream_t>(stream), planes);
}
