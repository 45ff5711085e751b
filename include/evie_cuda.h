/* evie_cuda.h — C ABI of libevie_cuda.so, a B200 (sm_100a) implementation of the Qwen3.5 token-mixing hot path
 * of the evie neuron-steering engine.
 *
 * The ABI mirrors evie-core's GPU backend (`GpuModel`, crates/evie-core/src/gpu/mod.rs) so that evie-core's
 * forward loop, caches and per-neuron hooks can call it through a Rust `extern "C"` block: plain pointers,
 * sizes and status codes; no C++ or CUDA types cross the boundary. Every function returns a status and never
 * aborts the process; the message for the last failure is available from `evie_last_error` (per context) or
 * `evie_last_global_error` (calls without a context, and context creation).
 *
 * Threading: one context per GPU; a context is not re-entrant (drive it from one host thread, as evie's
 * inference thread drives `GpuModel`, crates/evie/src/worker.rs:209-237). Isolated-op entry points may be
 * called from any thread; they enqueue work on the stream they are given.
 */
#ifndef EVIE_CUDA_H
#define EVIE_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define EVIE_API __attribute__((visibility("default")))
#else
#define EVIE_API
#endif

typedef int evie_status;
#define EVIE_OK 0
#define EVIE_ERR_ARG 1     /* invalid argument or size limit (the reference's `ensure!` limits) */
#define EVIE_ERR_CUDA 2    /* CUDA / cuBLAS runtime error */
#define EVIE_ERR_IO 3      /* checkpoint could not be read or parsed */
#define EVIE_ERR_OOM 4     /* device allocation failed */
#define EVIE_ERR_TIMEOUT 5 /* a bounded device-side wait gave up */

typedef struct evie_ctx evie_ctx;

/* One sequence in a forward call (GpuSeq, gpu/mod.rs:147-154). `tokens` is a host pointer. */
typedef struct {
  int32_t slot;            /* cache slot, 0..slots-1 */
  int32_t pos0;            /* absolute position of the first new token */
  const uint32_t* tokens;  /* n_tokens token ids */
  int32_t n_tokens;
} evie_seq;

/* One steering op for a slot (the tuple of GpuModel::set_ops, gpu/mod.rs:555-565).
 * mode 1 = add `value` (already dose x unit, engine.rs:102-108), 2 = multiply by `value`, 3 = set to `value`. */
typedef struct {
  int32_t layer;
  int32_t neuron;
  int32_t mode;
  float value;
} evie_op;

/* One op of a compiled steering plan with its gate (the Op of Plan, crates/evie-core/src/steering.rs:85-89).
 * gate = -1 for an ungated op, else the index of the gate (0..n_gates-1) in the same evie_set_plan call. */
typedef struct {
  int32_t layer;
  int32_t neuron;
  int32_t mode;  /* 1 add, 2 mul, 3 set, as evie_op */
  float value;
  int32_t gate;
} evie_plan_op;

/* One detector term of a gate (Detector, steering.rs:21-27; Plan::detectors entries, steering.rs:102-103). */
typedef struct {
  int32_t gate;
  int32_t layer;
  int32_t neuron;
  float weight;
} evie_detector;

/* Sampling parameters of one sequence (SampleParams, crates/evie-core/src/sampling.rs:5-13). temperature <= 0 is
 * greedy; top_p 1, min_p 0 and repetition_penalty 1 switch those steps off. */
typedef struct {
  float temperature;
  float top_p;
  float min_p;
  float repetition_penalty;
  uint64_t seed;
} evie_sample_params;

/* Model dimensions, for sizing host buffers. */
typedef struct {
  int32_t hidden, intermediate, n_layers, vocab;
  int32_t n_linear_layers, n_full_layers;
  int32_t slots, max_ctx, max_rows, max_ops;
  int64_t weight_bytes, cache_bytes;
} evie_model_info;

/* Creates a context on `device` and uploads the checkpoint in `ckpt_dir` (config.json + *.safetensors, bf16).
 * Replaces GpuModel::new(model, max_ctx) (gpu/mod.rs:226). `slots` sequences can be cached at once, each up
 * to `max_ctx` positions; one forward call carries at most `max_rows` new tokens in total. */
EVIE_API evie_status evie_create(const char* ckpt_dir, int device, int slots, int max_ctx, int max_rows, evie_ctx** out);
EVIE_API void evie_destroy(evie_ctx* ctx);
EVIE_API const char* evie_last_error(const evie_ctx* ctx);
EVIE_API const char* evie_last_global_error(void);
EVIE_API evie_status evie_info(const evie_ctx* ctx, evie_model_info* out);

/* Runs the new tokens of `n_seqs` sequences (GpuModel::forward, gpu/mod.rs:615). All output pointers are host
 * buffers and may be NULL when not wanted:
 *   logits       [n_seqs][vocab] f32, next-token logits of each sequence's last new token (if want_logits);
 *   frames       [rows][layers*intermediate] i8 sqrt-companded activations after steering (if capture);
 *   resid        [rows][layers*hidden] f16 bits, residual stream leaving each layer (if capture);
 *   next_tokens  [n_seqs] the token each sequence's slot sampler picks from its last row's logits: greedy = the
 *                first index of the maximum logit (topk(logits, 1), sampling.rs:60) unless evie_set_sampler
 *                gave the slot other parameters (Sampler::sample, sampling.rs:41-93).
 * rows are the concatenation of every sequence's new tokens, in call order.
 * Returns EVIE_ERR_TIMEOUT when a kernel on this device gave up a bounded device-side wait since the last check
 * (this call's, or one enqueued earlier on the device): the outputs are then incomplete. The count restarts. */
EVIE_API evie_status evie_forward(evie_ctx* ctx, const evie_seq* seqs, int n_seqs, int want_logits, int capture, float* logits,
                         int8_t* frames, uint16_t* resid, uint32_t* next_tokens);

/* The decode loop of evie's worker (crates/evie/src/worker.rs:442-526) kept on the device: every sequence carries
 * its first token (n_tokens = 1) at pos0; step i runs the model on each sequence's token of step i-1 at position
 * pos0 + i, with no host round trip between steps. Tokens come from each slot's sampler as in evie_forward: greedy
 * unless evie_set_sampler says otherwise (the name keeps the greedy default).
 *   out_tokens  [steps][n_seqs] host, the token produced by each step (may be NULL);
 *   frames      [steps][n_seqs][layers*intermediate] i8 host, captured activations per step (if capture);
 *   resid       [steps][n_seqs][layers*hidden] f16 bits host (if capture).
 * Returns EVIE_ERR_TIMEOUT as evie_forward does. */
EVIE_API evie_status evie_decode_greedy(evie_ctx* ctx, const evie_seq* seqs, int n_seqs, int steps,
                                        uint32_t* out_tokens, int capture, int8_t* frames, uint16_t* resid);
/* The CUDA stream (cudaStream_t) all of the context's work is enqueued on, for timing with CUDA events. */
EVIE_API void* evie_stream(const evie_ctx* ctx);

/* Profiling mode: when on, every kernel group of later calls is bracketed by CUDA events on the context's stream,
 * and its device time is accumulated per group. The groups are: one per projection weight (DeltaNet input and
 * output, attention input and output, MLP gate/up and down), LM head, conv, DeltaNet mixer, attention prep,
 * attention, add+norm, SwiGLU, other. In evie_decode_greedy (without EVIE_NO_GRAPH) each step is captured as a
 * graph of its own, with the events as event-record nodes, so a group is timed as a replayed step runs it. Each
 * node adds a few microseconds. Other calls run eagerly. A call whose events cannot be recorded or timed returns
 * EVIE_ERR_CUDA. Turning the mode on or off clears the totals. */
EVIE_API evie_status evie_profile(evie_ctx* ctx, int on);
/* Group i's name, accumulated milliseconds and number of bracketed launches; returns the number of groups
 * (0 when i is out of range). */
EVIE_API int evie_profile_read(const evie_ctx* ctx, int i, const char** name, double* ms, int64_t* launches);

/* Replaces a slot's steering ops (GpuModel::set_ops, gpu/mod.rs:556). Ops apply in the given order. Clears the
 * slot's gates (as evie_set_plan with no gates). */
EVIE_API evie_status evie_set_ops(evie_ctx* ctx, int slot, const evie_op* ops, int n_ops);

/* Replaces a slot's steering plan with one that may hold latching detector gates (Plan, steering.rs:97-104,
 * compiled by Plan::compile, steering.rs:118-139; evie-core's wgpu backend has no gates). gate g opens, and stays
 * open across calls, once on some new row the weighted sum of its detectors' activations exceeds thresholds[g]:
 *   - detectors read the activations of their layer before that layer's ops (Plan::apply, steering.rs:163-172);
 *     their terms are summed in f32 layer by layer, within a layer in the given order (a detector's position in
 *     `dets` among those of its layer is its position in Plan::detectors);
 *   - a gate decides at its last detector layer (0 when none of its detectors is in range): its score becomes the
 *     sum on the call's last row of that sequence, and a closed gate opens at the first row over the threshold;
 *   - a gated op applies to every row while its gate was open before the call; a gate that opened during the call
 *     applies from the trigger row on at layers at or after its deciding layer, and from the next call on before
 *     it (steering.rs:189-199).
 * Ops and detectors whose layer or neuron is out of range are dropped (steering.rs:121, 128). Setting a plan
 * closes the slot's gates and zeroes their scores (Plan::new_state, steering.rs:145-148). Limits: evie_info's
 * max_ops ops, 32 gates and 128 detectors per slot. */
EVIE_API evie_status evie_set_plan(evie_ctx* ctx, int slot, const evie_plan_op* ops, int n_ops, const float* thresholds,
                                   int n_gates, const evie_detector* dets, int n_dets);
/* Reads a slot's gate state after the calls so far (GateState::open and ::score, steering.rs:106-114): n_gates
 * entries each (the slot's plan count; fewer is an error). Either pointer may be NULL. */
EVIE_API evie_status evie_gate_state(evie_ctx* ctx, int slot, int32_t* open, float* score, int n_gates);
/* Closes a slot's gates and zeroes their scores, keeping its plan (a fresh GateState for a new conversation). */
EVIE_API evie_status evie_reset_gates(evie_ctx* ctx, int slot);
/* Sets a slot's sampler (Sampler::new, sampling.rs:27-29): the parameters and a generator state started from
 * params->seed; NULL restores the greedy default. The repetition penalty's history is every token fed to the slot
 * since its last evie_reset_slot (the worker's prompt ids + generated tokens, worker.rs:241, 320). One uniform is
 * drawn per sampled token at temperature > 0. */
EVIE_API evie_status evie_set_sampler(evie_ctx* ctx, int slot, const evie_sample_params* params);
/* Zeroes a slot's recurrent and conv state (GpuModel::reset_slot, gpu/mod.rs:568) and its sampler history. */
EVIE_API evie_status evie_reset_slot(evie_ctx* ctx, int slot);
/* Per-neuron activation scales used to normalise captured frames, layer-major (gpu/mod.rs:549). */
EVIE_API evie_status evie_set_scale(evie_ctx* ctx, const float* scale, size_t n);
/* Offline analysis (crates/evie-core/src/analysis.rs, lens.rs). Every call below is synchronous, allocates its
 * device scratch and frees it before it returns, and runs its products on the library's tensor-core projection
 * GEMM. A bounded wait that gives up inside one of them makes the call return EVIE_ERR_TIMEOUT.
 *
 * A lens (lens.rs:10-83, Lens::load once the torch file is read): per-layer [hidden][hidden] maps J_l, row-major
 * 16-bit values (kind 0 = f16, 1 = bf16), maps[l] = NULL where the file has no map for layer l; layers past
 * target_layer, and layers without a map, read out with the identity (Lens::map). The maps are copied to the device
 * (as J_l and J_l^T); the host arrays may be freed after the call. Replaces the context's previous lens. */
EVIE_API evie_status evie_set_lens(evie_ctx* ctx, const uint16_t* const* maps, int n_layers, int kind,
                                   int target_layer);
/* Drops the lens: the analysis calls read out through the identity (the logit lens). */
EVIE_API evie_status evie_clear_lens(evie_ctx* ctx);
/* The unembedding statistics (analysis.rs:129-171, UnembedStats::compute: mean of the LM-head rows, gain-weighted
 * covariance of a strided subsample stored as f16 with its scale) and every neuron's logit spread sqrt(u^T M u)
 * over its down_proj column u carried through the lens (analysis.rs:183-201, neuron_sigma).
 *   sigma    [layers * intermediate] host, layer-major (n must equal that count);
 *   mean     [hidden] host or NULL;  m_scale  host or NULL. */
EVIE_API evie_status evie_neuron_sigma(evie_ctx* ctx, float* sigma, size_t n, float* mean, float* m_scale);
/* lens_logits (analysis.rs:28-34): logits [n][vocab] (host) of n residual-basis vectors vecs [n][hidden] (host)
 * living at `layer`: the lens map of the layer, then the final RMSNorm and the LM head (model.rs:287-294). */
EVIE_API evie_status evie_lens_logits(evie_ctx* ctx, int layer, const float* vecs, int n, float* logits);
/* neuron_logits (analysis.rs:37-67): logits [n][vocab] (host) of the write directions W_down[:, neurons[i]] of
 * layers[i] through the lens and the unembedding. neuron_readouts / token_ranks (analysis.rs:70-105) rank these rows. */
EVIE_API evie_status evie_neuron_logits(evie_ctx* ctx, const int32_t* layers, const int32_t* neurons, int n,
                                        float* logits);
/* search (analysis.rs:213-240) up to the ranking: for every neuron the best standardized score over the tokens of
 * each pole, z = (W_down^T J_l^T a_t)_n / sigma_n with a_t = (W_U[t] - mean) * g (analysis.rs:173-179):
 *   z_up[l][n] = max_t z, z_dn[l][n] = max_t -z  (host, [layers * intermediate] each);
 *   mean, sigma: evie_neuron_sigma's outputs under the same lens. The caller sorts (stable, z descending; per
 *   layer, then merged) and keeps the top `limit` (analysis.rs:241-250). */
EVIE_API evie_status evie_search_scores(evie_ctx* ctx, const uint32_t* tokens, int n_tokens, const float* mean,
                                        const float* sigma, float* z_up, float* z_dn);
/* Track the max |activation| of every neuron over positions > 0 across later calls (gpu/mod.rs:578). */
EVIE_API evie_status evie_track_max(evie_ctx* ctx, int on);
/* Reads the tracked maxima, layer-major (gpu/mod.rs:590). */
EVIE_API evie_status evie_read_max(evie_ctx* ctx, float* out, size_t n);
/* The k (1..100) most active neurons of every row the last capturing call left on the device (the rows of the last
 * evie_forward with capture, or of the last step of evie_decode_greedy with capture), as evie's top_active tool
 * ranks one token's frame (crates/evie/src/mcp.rs:242-256): by |q| of the i8 frame, largest first, equal |q| in
 * increasing flat index (layer * intermediate + neuron). out: [rows][k] host; *rows receives the row count. */
EVIE_API evie_status evie_read_top_active(evie_ctx* ctx, int k, int32_t* out, int* rows);

/* ---- isolated ops: device pointers, enqueued on `stream` (a cudaStream_t, NULL = legacy default) ---- */

/* top_active (mcp.rs:242-256) over `rows` device frames of `width` i8 entries: out [rows][k] device int32 flat
 * indices, by |q| descending, equal |q| in increasing index. 1 <= k <= 100 (k > width leaves the tail unwritten). */
EVIE_API evie_status evie_top_active(const int8_t* frames, int rows, long long width, int k, int32_t* out,
                                     void* stream);

/* Sampler::new's generator state for a seed (sampling.rs:27-29), for evie_sample's rng array. */
EVIE_API uint64_t evie_sampler_seed_state(uint64_t seed);
/* Sampler::sample (sampling.rs:41-93) for B sequences; synchronous (returns after the stream has run it).
 *   logits    [B][V] f32 device;
 *   params    [B] host; rng [B] host generator states (evie_sampler_seed_state), advanced in place;
 *   history   device token ids, sequence b's at history[hist_off[b] .. hist_off[b+1]) (hist_off [B+1] host);
 *   out       [B] host tokens.
 * V <= 1048576. */
EVIE_API evie_status evie_sample(const float* logits, int B, int V, const evie_sample_params* params, uint64_t* rng,
                                 const uint32_t* history, const int64_t* hist_off, uint32_t* out, void* stream);

/* One Gated DeltaNet recurrent decode step over B*H heads (recur_step, crates/evie-core/src/model.rs:501-541;
 * the `deltanet` WGSL kernel, gpu/kernels.wgsl:379-442):
 *   kv = S^T k; delta = (v - exp(g) kv) beta; S <- exp(g) S + k delta^T; o = S^T q (updated S).
 * q,k: [B][H][dk] bf16; v: [B][H][dv] bf16; g (log decay), beta: [B][H] f32; state: [B][H][dk][dv] f32 updated
 * in place; o: [B][H][dv] f32. dk = dv = 128. */
EVIE_API evie_status evie_gdn_decode_step(const void* q, const void* k, const void* v, const float* g, const float* beta,
                                 float* state, float* o, int B, int H, int dk, int dv, void* stream);

/* Gated DeltaNet prefill over T tokens, chunked (chunk = 64) on tcgen05 tensor cores: the recurrence of evie-core's
 * token-sequential loop (model.rs:362-387, recur_body model.rs:501-541) regrouped per chunk with a triangular solve,
 * every f32 operand split into bf16 hi + lo planes so that the result follows the f32 recurrence (~1e-5 relative).
 * q,k: [B][T][H][dk] bf16; v: [B][T][H][dv] bf16 (all three 16-byte aligned); g (log decay, <= 0), beta: [B][T][H]
 * f32; state: [B][H][dk][dv] f32 (16-byte aligned), initial state in, final state out; o: [B][T][H][dv] bf16.
 * dk = dv = 128, chunk = 64. One CTA per (sequence, head). */
EVIE_API evie_status evie_gdn_chunk_prefill(const void* q, const void* k, const void* v, const float* g, const float* beta,
                                   float* state, void* o, int B, int T, int H, int dk, int dv, int chunk,
                                   void* stream);

/* The same prefill, token by token (the order of evie-core's loop, model.rs:362-387) with the state slice held in
 * registers: for short prompts, where chunking has nothing to amortise. Same layouts as evie_gdn_chunk_prefill
 * (o 8-byte aligned). */
EVIE_API evie_status evie_gdn_prefill_tokenwise(const void* q, const void* k, const void* v, const float* g,
                                                const float* beta, float* state, void* o, int B, int T, int H, int dk,
                                                int dv, void* stream);

/* Projection GEMM on tcgen05 tensor cores (evie-core's `matmul` with bf16 weights and f32 activations,
 * crates/evie-core/src/kernels.rs:138-268; the WGSL `matmul_small` / `matmul_tiled`, gpu/kernels.wgsl:112-235), the
 * kernel behind every projection and the LM head of evie_forward:
 *   y[s][r][m] = sum over k in K slice s of w[m][k] (hi[r][k] + lo[r][k]),   s = 0 .. *planes - 1,
 * where x2 = [hi; lo] ([2][R][K] bf16) is an f32 activation matrix split into bf16 planes (hi = bf16(x),
 * lo = bf16(x - hi)) and w is [M][K] bf16 (both 16-byte aligned, K % 8 == 0). The full product is the sum of the
 * *planes planes in slice order; R <= 128 cuts K into up to max_planes slices so that the weight stream fills every
 * SM. y holds y_cap floats (at least R x M; *planes x R x M are written). */
EVIE_API evie_status evie_proj_gemm(const void* w, const void* x2, float* y, size_t y_cap, int M, int K, int R,
                                    int max_planes, int* planes, void* stream);

/* Synchronises the current device and reports whether any kernel gave up a bounded device-side wait (an mbarrier
 * that did not complete within 2 s) since the last poll: EVIE_ERR_TIMEOUT with the count in the message, then the
 * count restarts at zero. Such a kernel drained its copies, freed its tensor memory and left its outputs
 * incomplete. */
EVIE_API evie_status evie_poll_device_errors(void);
/* Diagnostic for the failure path above (no reference counterpart; evie-core's backends have no device-side waits):
 * one thread on the current device waits at most limit_ns (<= 2 s) on an mbarrier that nothing completes, gives
 * up, counts the give-up for evie_poll_device_errors as the kernels do, and returns. *gave_up is 1 when it gave up.
 * The device stays usable. */
EVIE_API evie_status evie_bounded_wait_probe(uint64_t limit_ns, int* gave_up);

/* Gated GQA softmax attention decode over a paged bf16 KV cache (the attention core of Model::attention,
 * model.rs:445-464; WGSL attn_scores/attn_out, gpu/kernels.wgsl:508-589), split-KV with an in-kernel combine:
 *   out[b,h] = softmax(scale * q[b,h] . K[b, 0..ctx_b)) V[b, 0..ctx_b) * sigmoid(gate[b,h]).
 * q, gate (logits): [B][Hq][hd] bf16; k_pages, v_pages: [num_pages][Hkv][page_size][hd] bf16;
 * page_table: [B][max_pages] int32; ctx_lens: [B] int32 (0 <= ctx_b <= max_pages*page_size);
 * out: [B][Hq][hd] f32. hd = 256, Hq/Hkv in {2,4}, page_size a multiple of 64, max_pages*page_size <= 262144.
 * Scratch for the split partials is allocated by the library on first use, per (device, stream), and kept. */
EVIE_API evie_status evie_gqa_decode_paged(const void* q, const void* gate, const void* k_pages, const void* v_pages,
                                  const int32_t* page_table, const int32_t* ctx_lens, float* out, int B, int Hq,
                                  int Hkv, int hd, int page_size, int max_pages, float scale, void* stream);

/* Gated GQA softmax attention for prefill rows (the attention core of Model::attention, model.rs:445-464, for every
 * new row of a prompt; WGSL attn_scores/attn_out, gpu/kernels.wgsl:508-589) on tcgen05 tensor cores:
 *   out[r,h] = softmax(scale * q[r,h] . K[s, 0..pos_r]) V[s, 0..pos_r] * sigmoid(gate[r,h]),
 * where sequence s owns rows [start_s, start_s + seq_rows[s]) (sequences in order), row i of it at position
 * pos_r = seq_pos0[s] + i, whose keys and values (those of the row itself included) are already in its pages.
 *   q, gate (logits), out: [rows][Hq][hd] f32 device (q, gate 16-byte aligned);
 *   k_pages, v_pages: [num_pages][Hkv][page_size][hd] bf16 device (16-byte aligned);
 *   page_table: [n_seqs][max_pages] int32 device; seq_rows, seq_pos0: [n_seqs] int32 host.
 * hd = 256, Hq = 4 Hkv, page_size a multiple of 64. The segment table is copied to a device buffer the library keeps
 * per (device, stream); the call waits for that copy. */
EVIE_API evie_status evie_gqa_prefill_paged(const float* q, const float* gate, const void* k_pages, const void* v_pages,
                                            int num_pages, const int32_t* page_table, int max_pages,
                                            const int32_t* seq_rows, const int32_t* seq_pos0, int n_seqs, float* out,
                                            int Hq, int Hkv, int hd, int page_size, float scale, void* stream);

/* The same attention as evie_gqa_decode_paged, for callers that cannot let the library allocate device memory:
 * serving engines that reserve nearly all GPU memory for their own allocator at start-up, and latency-critical
 * callers that cannot afford cudaMalloc's device synchronisation. It calls no cudaMalloc, cudaFree or allocating
 * library routine; its split scratch is a fixed 32 MiB array compiled into the library, held on every GPU that
 * loads the library until the process exits. No counterpart in the reference (evie allocates its buffers itself).
 *   - Sizes whose scratch exceeds 32 MiB are rejected with EVIE_ERR_ARG (about B x Hkv x ceil(max_pages x
 *     page_size / 512) <= 8100 for GQA group 4); the allocating entry point has no such limit.
 *   - The first call on a device looks up the array's device address (cudaGetSymbolAddress) with that device
 *     current; make that first call before any stream capture.
 *   - Every call on a device shares the one array and it keeps the last call's contents (each call clears the part
 *     that must start at zero); calls that may overlap on the GPU (other streams, other host threads) race on it,
 *     so serialise them. */
EVIE_API evie_status evie_gqa_decode_paged_noalloc(const void* q, const void* gate, const void* k_pages,
                                                   const void* v_pages, const int32_t* page_table,
                                                   const int32_t* ctx_lens, float* out, int B, int Hq, int Hkv, int hd,
                                                   int page_size, int max_pages, float scale, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* EVIE_CUDA_H */
