// Next-token sampling on the device: evie-core's Sampler (crates/evie-core/src/sampling.rs:21-93) — repetition
// penalty over the sequence's history, greedy (topk(logits, 1)) at temperature 0, otherwise the top 512 logits,
// softmax at the temperature, min-p and top-p cuts and one splitmix64 uniform per draw.
#pragma once
#include "model_kernels.h"

namespace evie {

// The f32 half of SampleParams (sampling.rs:5-13); the seed lives on as the per-slot generator state.
struct SamplerParams {
  float temperature, top_p, min_p, repetition_penalty;
};

// Sampler::new (sampling.rs:27-29): the generator state a seed starts from.
inline uint64_t sampler_seed_state(uint64_t seed) { return (seed * 0x9E3779B97F4A7C15ull) ^ 0xD1B54A32D192ED03ull; }

// What one launch samples from. Sequence s reads logits row s (s * V) and its sampler: the slot's entry when segs
// is given (the model's per-slot tables), else entry s. The history is either a per-slot bitmap of every token
// fed since the slot's reset (seen, seen_words per slot) or, without segs, a list per sequence
// (hist[hist_off[s] .. hist_off[s+1])).
struct SampleArgs {
  YView logits;
  int V;
  const SegInfo* segs;
  const SamplerParams* params;
  uint64_t* rng;
  const uint32_t* seen;
  int seen_words;
  const uint32_t* hist;
  const long long* hist_off;
  uint32_t* next;
};

evie_status k_sample(const SampleArgs& a, int nseq, cudaStream_t st);

}  // namespace evie
