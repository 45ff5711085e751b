// Kernels of the full-model forward pass (model_kernels.cu) and the shapes they share with the host runtime.
//
// Projection operands: the reference multiplies bf16 weights by f32 activations (crates/evie-core/src/kernels.rs
// :1-4). On tensor cores both operands must be bf16, so every activation matrix X that feeds a projection is
// written as two stacked bf16 planes, X = hi + lo with hi = bf16(X) and lo = bf16(X - hi) (16 significant bits).
// The projection GEMM (proj_gemm.h) multiplies both planes by the weights it reads once and adds the products in f32;
// its output is one plane per K slice, which consumers add when they read it (YView). The result matches the f32
// product to ~2^-16 relative.
#pragma once
#include <vector>

#include "common.h"

namespace evie {

struct RowInfo {
  int slot, pos, token, seg;
};
struct SegInfo {
  int slot, start, count, pos0;
};

// Split-plane helpers: plane 0 = hi, plane 1 = lo, plane stride R*ld elements.
__device__ __forceinline__ void store_split(__nv_bfloat16* X2, size_t plane, size_t idx, float v) {
  const __nv_bfloat16 hi = __float2bfloat16_rn(v);
  X2[idx] = hi;
  X2[plane + idx] = __float2bfloat16_rn(v - __bfloat162float(hi));
}
__device__ __forceinline__ float load_y(const float* Y2, size_t plane, size_t idx) { return Y2[idx] + Y2[plane + idx]; }

// A projection output as `n` partial planes of `plane` floats each, added in a fixed order when read: the K-slice
// partials of the projection GEMM (one plane when K is not sliced).
struct YView {
  static constexpr int kMaxPlanes = 16;
  const float* p;
  size_t plane;
  int n;
  // Planes are loaded two at a time and added in plane order: consumers near their register limit keep few values
  // live, and two planes (the common K-slice counts are 1 to 3) cost one L2 round trip.
  // A single plane (every projection of a many-row call) is one load: the plane loop, even with no plane to add,
  // cost the prefill SwiGLU half its time (39.0 against 17.8 ms per 4B call).
  __device__ __forceinline__ float at(size_t i) const {
    if (n == 1) return p[i];
    float s = p[i];
    int k = 1;
    for (; k + 1 < n; k += 2) {
      const float a = p[(size_t)k * plane + i], b = p[(size_t)(k + 1) * plane + i];
      s += a;
      s += b;
    }
    if (k < n) s += p[(size_t)k * plane + i];
    return s;
  }
  // Four consecutive elements (i a multiple of 4; rows and planes 16-byte aligned), planes added in plane order.
  // Each plane is added as it arrives: the loads are independent, so the compiler still issues them ahead, without
  // holding every plane in registers at once.
  __device__ __forceinline__ float4 at4(size_t i) const {
    float4 s = *reinterpret_cast<const float4*>(p + i);
    if (n == 1) return s;
#pragma unroll
    for (int k = 1; k < kMaxPlanes; k++)
      if (k < n) {
        const float4 v = *reinterpret_cast<const float4*>(p + (size_t)k * plane + i);
        s.x += v.x, s.y += v.y, s.z += v.z, s.w += v.w;
      }
    return s;
  }
  // at4 for consumers of projections with few K slices (SwiGLU after gate/up's 2, attention prep after the
  // attention input's 3): 2 or 3 planes are loaded before the first add, same sum. Measured per 4B decode step: SwiGLU
  // 0.28 against 0.34 ms; in the add+norm (14 planes, which this form would only pass through) the extra branch cost
  // 0.70 against 0.56 ms, so that kernel keeps at4.
  __device__ __forceinline__ float4 at4_few(size_t i) const {
    if (n == 2 || n == 3) {
      float4 s = *reinterpret_cast<const float4*>(p + i);
      const float4 a = *reinterpret_cast<const float4*>(p + plane + i);
      const float4 b = n == 3 ? *reinterpret_cast<const float4*>(p + 2 * plane + i) : make_float4(0.f, 0.f, 0.f, 0.f);
      s.x += a.x, s.y += a.y, s.z += a.z, s.w += a.w;
      if (n == 3) s.x += b.x, s.y += b.y, s.z += b.z, s.w += b.w;
      return s;
    }
    return at4(i);
  }
};

struct ModelShape {
  int d, n, L, V;
  float eps;
  int nh, nkv, hd, rot;
  int K, hk, hv, dk, dv, conv_dim, vd, key_dim;
  int in_dn;   // rows of the fused DeltaNet input projection: conv_dim + vd + 2 hv
  int in_at;   // rows of the fused attention input projection: (2 nh + 2 nkv) hd
};

// seen: per-slot bitmap (seen_words words per slot) of every token fed since the slot's reset, the sampler's
// repetition history; the kernel sets each row's token bit.
evie_status k_embed_norm(const RowInfo* rows, int R, const __nv_bfloat16* embed, float* x, const float* gain,
                         float eps, int d, __nv_bfloat16* X2, uint32_t* seen, int seen_words, cudaStream_t st);
// x += Y (its K-slice planes); optional f16 capture of x as the residual leaving `cap_layer`; then X2 = split(rmsnorm(x)).
evie_status k_add_norm(float* x, YView y, int ldy, int R, const float* gain, float eps, int d,
                       __nv_bfloat16* X2, uint16_t* resid, int cap_layer, int L, cudaStream_t st);
// Final residual add (+ capture of the last layer) and final norm of each segment's last row into X2 [2][nseg][d].
evie_status k_add_final(float* x, YView y, int ldy, int R, const RowInfo* rows, const SegInfo* segs,
                        int nseg, const float* gain, float eps, int d, __nv_bfloat16* X2, uint16_t* resid,
                        int cap_layer, int L, cudaStream_t st);
// Causal depthwise conv over [conv state ; new rows] + SiLU, then L2 norm of the q and k heads (q also 1/sqrt(dk)).
// conv_state points at this layer's window of slot 0; cs_slot is the element stride between slots.
// update_window: every segment has exactly one row (decode); the kernel then also shifts the conv windows in place
// (replacing k_conv_state_update). For a 4-tap conv with 16-byte aligned operands that is a warp per 128-channel
// head block with four channels per lane; otherwise one thread per channel. With max_seg_rows > 1 (and a 4-tap
// conv) a sliding-window kernel walks each segment's rows in blocks of 64 (a warp per head block with four channels
// per lane when the operands are 16-byte aligned, else a thread per channel); split_qk (that form only) writes the q
// and k channels as split bf16 planes in place of their f32 values, the chunked prefill's operand format.
evie_status k_conv_silu_norm(YView y, int ldy, int R, const RowInfo* rows, const SegInfo* segs,
                             float* conv_state, size_t cs_slot, const float* conv_w, const ModelShape& s,
                             float* act, cudaStream_t st, bool update_window, int nseg = 0, int max_seg_rows = 0,
                             bool split_qk = false);
evie_status k_conv_state_update(YView y, int ldy, int R, const SegInfo* segs, int nseg, float* conv_state,
                                size_t cs_slot, const ModelShape& s, cudaStream_t st);
// Gated delta rule over each segment's rows (state resident in registers) + gated RMSNorm -> X2 [R][vd].
// rec_state points at this layer's [hv][dk][dv] state of slot 0; rs_slot is the element stride between slots.
evie_status k_gdn_mixer(const float* act, YView y, int ldy, int R, const SegInfo* segs, int nseg,
                        float* rec_state, size_t rs_slot, const float* neg_a, const float* dt_bias,
                        const float* norm_w, const ModelShape& s, __nv_bfloat16* X2, cudaStream_t st);
// Gated RMSNorm of the chunked prefill's outputs (f32 over the v columns of act) -> X2 [R][vd].
evie_status k_gdn_gated_norm(const float* act, YView y, int ldy, int R, const float* norm_w, const ModelShape& s,
                             __nv_bfloat16* X2, cudaStream_t st);
// q/k RMSNorm (1+w gains) + partial RoPE; q -> q_rot f32 [R][nh][hd]; k, v -> paged cache (bf16 or f32).
template <typename KV>
evie_status k_attn_prep(YView y, int ldy, int R, const RowInfo* rows, const float* q_norm,
                        const float* k_norm, const float* inv_freq, const ModelShape& s, float* q_rot, KV* kc,
                        KV* vc, const int* page_table, int pages_per_slot, int page_size, cudaStream_t st);
// A latching detector gate of a slot's plan (GateSpec, steering.rs:91-95): its detectors sit in layers
// first_layer..last_layer, it decides at last_layer (both 0 when it has no detector in range).
struct GateSpec {
  float threshold;
  int first_layer, last_layer, pad;
};
struct DetSpec {
  int gate, neuron;
  float weight;
  int pad;
};
// Per-slot gate state: open latches across calls; from is the first position a gate covers at or after its
// deciding layer in the current call (INT_MIN when it was open before the call).
struct GateTables {
  const GateSpec* gates;   // [slots][max_gates]
  const int* n_gates;      // [slots]
  const DetSpec* dets;     // [slots][max_dets], each slot's detectors sorted by layer (stable)
  const int* det_range;    // [slots][L][2] (first, count) into the slot's detectors
  int max_gates, max_dets;
  int* open;               // [slots][max_gates]
  float* score;            // [slots][max_gates] detector sum on the last row of the latest call
  int* from;               // [slots][max_gates]
  float* partial;          // [max_rows][max_gates] running detector sums of the call's rows
};
// silu(gate) * up, per-slot steering ops, capture, max tracking -> X2 [R][n].
struct SteerTables {
  const evie_op* ops;      // [slots][max_ops], each slot's ops sorted by layer (stable)
  const int* range;        // [slots][L][2] (first, count) into the slot's ops
  int max_ops;
  const int* op_gate;      // [slots][max_ops] gate of each op, -1 = ungated
  const GateSpec* gates;   // [slots][max_gates]
  const int* open;         // [slots][max_gates]
  const int* from;         // [slots][max_gates]
  int max_gates;
};
// Plan::apply's detector half (steering.rs:164-187) for `layer`, before the layer's SwiGLU kernel applies the ops:
// adds every detector term of this layer to each row's running sums, then lets the gates that decide here take
// their score and latch open at the first row over the threshold. One CTA per segment.
evie_status k_gate_detect(YView y, int ldy, const SegInfo* segs, int nseg, int layer, const ModelShape& s,
                          GateTables t, cudaStream_t st);
evie_status k_swiglu(YView y, int ldy, int R, const RowInfo* rows, int layer, const ModelShape& s,
                     SteerTables steer, const float* scale, int8_t* frames, uint32_t* maxbuf, __nv_bfloat16* X2,
                     cudaStream_t st);
// top_active (mcp.rs:242-256) per frame row: the k largest |q|, equal |q| by increasing index -> out [rows][k].
evie_status k_top_active(const int8_t* frames, int rows, long long width, int k, int32_t* out, cudaStream_t st);
// logits = two planes summed (optional copy out), greedy argmax (first index of the maximum).
evie_status k_logits_argmax(YView L2, int nseg, int V, float* logits, unsigned long long* best,
                            uint32_t* next_tokens, cudaStream_t st);

// Decode loop step: row s (one per sequence) moves to the next position and takes the greedy token next[s].
evie_status k_advance_rows(RowInfo* rows, int nseq, const uint32_t* next, cudaStream_t st);

}  // namespace evie
