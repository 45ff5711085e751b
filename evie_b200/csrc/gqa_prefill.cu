// Gated GQA softmax attention for prefill (many query rows of one sequence in a call), flash style, for sm_100a.
//
// Semantics are those of the decode kernel (the attention core of Model::attention, crates/evie-core/src/model.rs:
// 445-464): for query row r at position pos_r and head h (KV head h / 4),
//   o = softmax(scale * q . k_j, j <= pos_r) V * sigmoid(gate),
// over the paged bf16 KV cache that this call's rows were just appended to.
//
// Design: one CTA per (block of 16 consecutive rows of one segment, KV head), 8 warps; warp w serves rows 2w, 2w+1
// of the block for the 4 query heads of the KV head: the 8 columns of every mma.sync m16n8k16 are (row, head) pairs.
// K and V are streamed through shared memory in 32-token tiles (cp.async, double-buffered), so every K/V byte
// is read once per block of 16 rows instead of once per row. q and p are split into bf16 hi + lo (two MMAs into one
// accumulator), which keeps the scores and outputs at f32 accuracy on the bf16 K/V, as in the decode kernel. The
// softmax is online across tiles (running max and sum per column, in the log2 domain); causal masking per column.
// Shared-memory rows are 512 bytes, so tiles are XOR-swizzled in 16-byte chunks to keep the fragment loads free of
// bank conflicts: K (read as rows g, g+8 at chunk 4p + c) flips chunk bit 2 by row bit 0; V (read at rows
// 2c + {0,1} (+8), chunks 16h + 2g + {0,1}) flips chunk bits 0 and 2 by row bits 1 and 2.
#include "common.h"
#include "gqa_decode.h"
#include "model_kernels.h"
#include "mma_sync.h"

namespace evie {

namespace {

constexpr int kHD = 256;
constexpr int kGroup = 4;
constexpr int kRowsPerCta = 16;
constexpr int kThreads = 256;
constexpr int kTile = 32;                            // tokens per shared-memory tile
constexpr uint32_t kTileBytes = kTile * kHD * 2;     // 16 KB of K (or V)
constexpr uint32_t kPBytes = 8 * 2 * 8 * 16 * 2;     // per warp: [hi/lo][8 columns][16 tokens] bf16
constexpr uint32_t kSmem = 2 * 2 * kTileBytes + kPBytes;
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ uint32_t k_off(int row, int chunk) {
  return (uint32_t)row * 512u + ((uint32_t)(chunk ^ ((row & 1) << 2)) << 4);
}
__device__ __forceinline__ uint32_t v_off(int row, int chunk) {
  return (uint32_t)row * 512u + ((uint32_t)(chunk ^ (((row >> 1) & 1) | (((row >> 2) & 1) << 2))) << 4);
}
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem)),
               "l"(gmem)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
__device__ __forceinline__ uint4 lds128(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }

__global__ void __launch_bounds__(kThreads, 1)
    gqa_prefill_kernel(const float* __restrict__ q_rot, YView y, int ldy, __nv_bfloat16* __restrict__ X2,
                       size_t xplane, const RowInfo* __restrict__ rows, const SegInfo* __restrict__ segs,
                       const int* __restrict__ page_table, int pages_per_slot, const __nv_bfloat16* __restrict__ kc,
                       const __nv_bfloat16* __restrict__ vc, int Hq, int Hkv, int page_size, float scale) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ __align__(128) uint8_t sm[];
  const int kvh = blockIdx.z;
  const SegInfo sg = segs[blockIdx.y];
  const int r_first = blockIdx.x * kRowsPerCta;
  if (r_first >= sg.count) return;
  const int n_rows = min(kRowsPerCta, sg.count - r_first);
  const int row0 = sg.start + r_first;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, c = lane & 3;
  const int wrow = 2 * warp;  // block-relative first row of this warp
  const int pos_last = rows[row0 + n_rows - 1].pos;
  const int n_tiles = pos_last / kTile + 1;
  const int32_t* pt = page_table + (size_t)sg.slot * pages_per_slot;

  // Q^T fragments for column g = (row g / 4, head g % 4), hi and lo, k-step 2p + e <-> dims 32p + 8c + 4e + {0..3}
  uint32_t qh[16][2], ql[16][2];
  {
    const bool valid = wrow + (g >> 2) < n_rows;
    const float* qp = q_rot + ((size_t)(row0 + wrow + (g >> 2)) * Hq + kvh * kGroup + (g & 3)) * kHD + 8 * c;
    const float f = scale * kLog2e;
#pragma unroll
    for (int p = 0; p < 8; p++) {
      float x[8];
      if (valid) {
        const float4 a = *reinterpret_cast<const float4*>(qp + 32 * p);
        const float4 b = *reinterpret_cast<const float4*>(qp + 32 * p + 4);
        x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
      } else {
#pragma unroll
        for (int j = 0; j < 8; j++) x[j] = 0.f;
      }
      float hi[8], lo[8];
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const float v = x[j] * f;
        hi[j] = bf16_round(v);
        lo[j] = v - hi[j];
      }
#pragma unroll
      for (int e = 0; e < 2; e++) {
        qh[2 * p + e][0] = pack_bf16x2(hi[4 * e], hi[4 * e + 1]);
        qh[2 * p + e][1] = pack_bf16x2(hi[4 * e + 2], hi[4 * e + 3]);
        ql[2 * p + e][0] = pack_bf16x2(lo[4 * e], lo[4 * e + 1]);
        ql[2 * p + e][1] = pack_bf16x2(lo[4 * e + 2], lo[4 * e + 3]);
      }
    }
  }
  // This lane's accumulator columns 2c, 2c+1 belong to row c / 2 of the warp (heads 2 (c % 2) + {0, 1}).
  const bool valid_c = wrow + (c >> 1) < n_rows;
  const int pos_c = valid_c ? rows[row0 + wrow + (c >> 1)].pos : -1;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  float o[16][4];  // O^T: m-tile 8 h + i <-> dims {128 h + 16 g + i | 128 h + 16 g + 8 + i}, columns 2c, 2c+1
#pragma unroll
  for (int i = 0; i < 16; i++) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  uint16_t* sP = reinterpret_cast<uint16_t*>(sm + 4 * kTileBytes) + warp * (kPBytes / 8 / 2);  // [2][8][16]

  auto load_tile = [&](int t, int stage) {
    const int tok0 = t * kTile;
    const int page = pt[tok0 / page_size];
    const size_t base = (((size_t)page * Hkv + kvh) * page_size + tok0 % page_size) * kHD;
    uint8_t* ks = sm + stage * 2 * kTileBytes;
    uint8_t* vs = ks + kTileBytes;
#pragma unroll
    for (int it = 0; it < kTile * 32 / kThreads; it++) {
      const int i = tid + it * kThreads, row = i >> 5, ch = i & 31;
      if (tok0 + row <= pos_last) {
        cp_async16(ks + k_off(row, ch), kc + base + (size_t)row * kHD + ch * 8);
        cp_async16(vs + v_off(row, ch), vc + base + (size_t)row * kHD + ch * 8);
      } else {  // past the block's context: zeros (the cache there may hold anything)
        *reinterpret_cast<uint4*>(ks + k_off(row, ch)) = make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(vs + v_off(row, ch)) = make_uint4(0, 0, 0, 0);
      }
    }
  };

  load_tile(0, 0);
  cp_async_commit();
#pragma unroll 1
  for (int t = 0; t < n_tiles; t++) {
    const int stage = t & 1;
    if (t + 1 < n_tiles) load_tile(t + 1, stage ^ 1);
    cp_async_commit();
    cp_async_wait1();  // this thread's copies of tile t have landed
    __syncthreads();   // and everyone's
    const uint8_t* ks = sm + stage * 2 * kTileBytes;
    const uint8_t* vs = ks + kTileBytes;
    const int tok0 = t * kTile;

    // ---- scores of the two 16-token halves, S^T[token][column]
    float sc[2][4];
#pragma unroll
    for (int st = 0; st < 2; st++) {
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int p = 0; p < 8; p++) {
        const uint4 ka = lds128(ks + k_off(16 * st + g, 4 * p + c));
        const uint4 kb = lds128(ks + k_off(16 * st + g + 8, 4 * p + c));
#pragma unroll
        for (int e = 0; e < 2; e++) {
          const uint32_t a0 = word_of(ka, 2 * e), a1 = word_of(kb, 2 * e);
          const uint32_t a2 = word_of(ka, 2 * e + 1), a3 = word_of(kb, 2 * e + 1);
          mma_bf16_16816(acc, a0, a1, a2, a3, qh[2 * p + e][0], qh[2 * p + e][1]);
          mma_bf16_16816(acc, a0, a1, a2, a3, ql[2 * p + e][0], ql[2 * p + e][1]);
        }
      }
      const int ta = tok0 + 16 * st + g, tb = ta + 8;
      sc[st][0] = ta <= pos_c ? acc[0] : -INFINITY;
      sc[st][1] = ta <= pos_c ? acc[1] : -INFINITY;
      sc[st][2] = tb <= pos_c ? acc[2] : -INFINITY;
      sc[st][3] = tb <= pos_c ? acc[3] : -INFINITY;
    }
    // ---- online softmax: lanes with equal c hold the same two columns
    float tm0 = fmaxf(fmaxf(sc[0][0], sc[0][2]), fmaxf(sc[1][0], sc[1][2]));
    float tm1 = fmaxf(fmaxf(sc[0][1], sc[0][3]), fmaxf(sc[1][1], sc[1][3]));
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      tm0 = fmaxf(tm0, __shfl_xor_sync(0xffffffffu, tm0, off));
      tm1 = fmaxf(tm1, __shfl_xor_sync(0xffffffffu, tm1, off));
    }
    const float mn0 = fmaxf(m0, tm0), mn1 = fmaxf(m1, tm1);
    const float b0 = mn0 == -INFINITY ? 0.f : mn0, b1 = mn1 == -INFINITY ? 0.f : mn1;
    const float a0 = exp2f(m0 - b0), a1 = exp2f(m1 - b1);  // 0 while nothing was accumulated
    m0 = mn0;
    m1 = mn1;
#pragma unroll
    for (int st = 0; st < 2; st++) {
      sc[st][0] = exp2f(sc[st][0] - b0);
      sc[st][1] = exp2f(sc[st][1] - b1);
      sc[st][2] = exp2f(sc[st][2] - b0);
      sc[st][3] = exp2f(sc[st][3] - b1);
    }
    l0 = l0 * a0 + sc[0][0] + sc[0][2] + sc[1][0] + sc[1][2];
    l1 = l1 * a1 + sc[0][1] + sc[0][3] + sc[1][1] + sc[1][3];
#pragma unroll
    for (int i = 0; i < 16; i++) {
      o[i][0] *= a0;
      o[i][1] *= a1;
      o[i][2] *= a0;
      o[i][3] *= a1;
    }

    // ---- O^T += V^T P^T per 16-token half; P^T goes through shared memory as [hi/lo][column][token]
#pragma unroll
    for (int st = 0; st < 2; st++) {
      __syncwarp();
      {
        const float pv[4] = {sc[st][0], sc[st][1], sc[st][2], sc[st][3]};
        const int cols[4] = {2 * c, 2 * c + 1, 2 * c, 2 * c + 1};
        const int toks[4] = {g, g, g + 8, g + 8};
#pragma unroll
        for (int k = 0; k < 4; k++) {
          const __nv_bfloat16 hi = __float2bfloat16_rn(pv[k]);
          const __nv_bfloat16 lo = __float2bfloat16_rn(pv[k] - __bfloat162float(hi));
          sP[cols[k] * 16 + toks[k]] = *reinterpret_cast<const uint16_t*>(&hi);
          sP[128 + cols[k] * 16 + toks[k]] = *reinterpret_cast<const uint16_t*>(&lo);
        }
      }
      __syncwarp();
      const uint32_t bh0 = *reinterpret_cast<const uint32_t*>(&sP[g * 16 + 2 * c]);
      const uint32_t bh1 = *reinterpret_cast<const uint32_t*>(&sP[g * 16 + 2 * c + 8]);
      const uint32_t bl0 = *reinterpret_cast<const uint32_t*>(&sP[128 + g * 16 + 2 * c]);
      const uint32_t bl1 = *reinterpret_cast<const uint32_t*>(&sP[128 + g * 16 + 2 * c + 8]);
#pragma unroll
      for (int h = 0; h < 2; h++) {
        uint4 v[4][2];
#pragma unroll
        for (int tk = 0; tk < 4; tk++) {
          const int row = 16 * st + 2 * c + (tk & 1) + 8 * (tk >> 1);
#pragma unroll
          for (int r = 0; r < 2; r++) v[tk][r] = lds128(vs + v_off(row, 16 * h + 2 * g + r));
        }
#pragma unroll
        for (int i = 0; i < 8; i++) {
          const int wi = i >> 1;
          const uint32_t sel = (i & 1) ? 0x7632u : 0x5410u;
          const uint32_t x0 = __byte_perm(word_of(v[0][0], wi), word_of(v[1][0], wi), sel);
          const uint32_t x1 = __byte_perm(word_of(v[0][1], wi), word_of(v[1][1], wi), sel);
          const uint32_t x2 = __byte_perm(word_of(v[2][0], wi), word_of(v[3][0], wi), sel);
          const uint32_t x3 = __byte_perm(word_of(v[2][1], wi), word_of(v[3][1], wi), sel);
          mma_bf16_16816(o[8 * h + i], x0, x1, x2, x3, bh0, bh1);
          mma_bf16_16816(o[8 * h + i], x0, x1, x2, x3, bl0, bl1);
        }
      }
    }
    __syncthreads();  // the stage is refilled by the next iteration's load
  }

  // ---- normalise, gate, and write the o_proj operand planes
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, off);
    l1 += __shfl_xor_sync(0xffffffffu, l1, off);
  }
  if (!valid_c) return;
  const int row = row0 + wrow + (c >> 1);
  const float inv[2] = {1.0f / l0, 1.0f / l1};
#pragma unroll
  for (int k = 0; k < 2; k++) {
    const int head = kvh * kGroup + 2 * (c & 1) + k;
    const size_t gy = (size_t)row * ldy + (size_t)head * 2 * kHD + kHD;
    const size_t ox = ((size_t)row * Hq + head) * kHD;
#pragma unroll
    for (int h = 0; h < 2; h++)
#pragma unroll
      for (int i = 0; i < 8; i++) {
        const int d0 = 128 * h + 16 * g + i, d1 = d0 + 8;
        store_split(X2, xplane, ox + d0, o[8 * h + i][k] * inv[k] * sigmoidf_(y.at(gy + d0)));
        store_split(X2, xplane, ox + d1, o[8 * h + i][2 + k] * inv[k] * sigmoidf_(y.at(gy + d1)));
      }
  }
}

}  // namespace

evie_status launch_gqa_prefill_model(const float* q_rot, YView y, int ldy, __nv_bfloat16* X2, size_t xplane,
                                     const RowInfo* rows, const SegInfo* segs, int nseg, int max_seg_rows,
                                     const int* page_table, int pages_per_slot, const __nv_bfloat16* kc,
                                     const __nv_bfloat16* vc, int Hq, int Hkv, int page_size, float scale,
                                     cudaStream_t st) {
  if (nseg == 0 || max_seg_rows == 0) return EVIE_OK;
  if (Hq != kGroup * Hkv) return fail(EVIE_ERR_ARG, "prefill attention: GQA group %d not supported (4)", Hq / Hkv);
  if (page_size % kTile != 0) return fail(EVIE_ERR_ARG, "prefill attention: page size must be a multiple of %d", kTile);
  EVIE_TRY(max_dynamic_smem((const void*)gqa_prefill_kernel, (int)kSmem));
  dim3 grid((max_seg_rows + kRowsPerCta - 1) / kRowsPerCta, nseg, Hkv);
  EVIE_CUDA_TRY(launch_k(gqa_prefill_kernel, dim3(grid), dim3(kThreads), kSmem, st, q_rot, y, ldy, X2, xplane, rows, segs, page_table, pages_per_slot,
                                                    kc, vc, Hq, Hkv, page_size, scale));
  EVIE_CHECK_LAUNCH("gqa_prefill_kernel");
  return EVIE_OK;
}

}  // namespace evie
