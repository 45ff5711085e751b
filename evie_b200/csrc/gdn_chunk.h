// Launcher of the chunked Gated DeltaNet prefill (gdn_chunk.cu).
#pragma once
#include "common.h"

namespace evie {
// Chunked (C = 64) prefill of T tokens for B*H heads on tcgen05 tensor cores. q,k,v: [B][T][H][128] bf16, 16-byte
// aligned; g, beta: [B][T][H] f32; state: [B][H][128][128] f32 in/out; o: [B][T][H][128] bf16.
evie_status launch_gdn_chunk_prefill_bf16(const void* q, const void* k, const void* v, const float* g,
                                          const float* beta, float* state, void* o, int B, int T, int H,
                                          cudaStream_t st);
struct SegInfo;
struct YView;
// The same chunked recurrence inside the forward pass: one CTA per (segment, value head) over the call's R rows.
// act [R][conv_dim]: the q/k columns hold split bf16 planes ([2][2 key_dim] bf16 per row, written by the conv
// kernel), v in f32; o (before the gated norm) is written in f32 over v. y: the DeltaNet input projection (b, a
// logits); rec_state: the layer's [hv][128][128] state of slot 0, rs_slot elements between slots; head dims 128.
evie_status launch_gdn_chunk_model(float* act, YView y, int ldy, int R, const SegInfo* segs, int nseg,
                                   float* rec_state, size_t rs_slot, const float* neg_a, const float* dt_bias,
                                   int conv_dim, int key_dim, int vd, int hv, int hk, cudaStream_t st);
// Device address of this device's counter of bounded waits that gave up (kernels bump it; the host polls it).
unsigned int* device_timeout_counter();
}  // namespace evie
