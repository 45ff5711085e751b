// Offline analysis on the device (analysis.cu): evie-core's lens readouts, unembedding statistics, per-neuron logit
// spread and neuron search (crates/evie-core/src/analysis.rs, lens.rs), every product on the projection GEMM.
#pragma once
#include <vector>

#include "common.h"

namespace evie {

// A 16-bit [rows][cols] matrix on the device as exact bf16 planes: one plane holds a bf16 matrix, two (hi + lo) an
// f16 one (f16 has 11 significant bits, so hi = bf16(x) and lo = x - hi are both exact in bf16).
struct Planes16 {
  const __nv_bfloat16* p = nullptr;
  int planes = 0, rows = 0, cols = 0;
};

// A lens (lens.rs:10-16) on the device: per layer the map J_l and its transpose as exact planes (planes == 0: the
// file has no map for the layer); layers past `target` read out with the identity (lens.rs:57-62).
struct LensDev {
  std::vector<Planes16> J, JT;
  long target = -1;
  void* mem = nullptr;
  const Planes16* map(int layer) const;
  const Planes16* map_t(int layer) const;
};

// What the analysis jobs read of a loaded model.
struct AnalysisModel {
  const __nv_bfloat16* lm_head = nullptr;  // [V][d] (tied embedding)
  int V = 0, d = 0, n = 0;                  // vocabulary, hidden, intermediate
  const float* final_norm = nullptr;        // [d] gains (1 + w)
  float eps = 0.f;
  std::vector<const __nv_bfloat16*> w_down;  // per layer [d][n]
  const LensDev* lens = nullptr;             // nullptr or a lens without maps: no lens
  cudaStream_t st = nullptr;
};

// maps[l]: host [d][d] 16-bit values (kind 0 = f16, 1 = bf16) or nullptr. Replaces any lens held in `lens`.
evie_status lens_upload(LensDev& lens, const uint16_t* const* maps, int n_layers, int d, int kind, long target,
                        cudaStream_t st);
void lens_free(LensDev& lens);

// analysis.rs:129-201: sigma [L][n] (host), the unembedding mean [d] (host, optional) and m_scale (optional).
evie_status neuron_sigma_run(const AnalysisModel& am, float* sigma, float* mean_out, float* m_scale_out);
// analysis.rs:28-34: [n][V] logits (host) of residual-basis vectors vecs [n][d] (host) at `layer`.
evie_status lens_logits_run(const AnalysisModel& am, int layer, const float* vecs, int n, float* logits);
// analysis.rs:37-67: [n][V] logits (host) of the write directions W_down[:, neurons[i]] of layers[i].
evie_status neuron_logits_run(const AnalysisModel& am, const int32_t* layers, const int32_t* neurons, int n,
                              float* logits);
// analysis.rs:213-240 up to the per-neuron best z: z_up / z_dn [L][n] (host) = max over the tokens of z and -z,
// z = (W_down^T J_l^T a_t)_i / sigma_i with a_t = (W_U[t] - mean) * g (analysis.rs:173-179).
evie_status search_scores_run(const AnalysisModel& am, const uint32_t* tokens, int nt, const float* mean,
                              const float* sigma, float* z_up, float* z_dn);

}  // namespace evie
