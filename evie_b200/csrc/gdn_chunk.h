// Launcher of the chunked Gated DeltaNet prefill (gdn_chunk.cu).
#pragma once
#include "common.h"

namespace evie {
// Chunked (C = 64) prefill of T tokens for B*H heads on tcgen05 tensor cores. q,k,v: [B][T][H][128] bf16, 16-byte
// aligned; g, beta: [B][T][H] f32; state: [B][H][128][128] f32 in/out; o: [B][T][H][128] bf16.
evie_status launch_gdn_chunk_prefill_bf16(const void* q, const void* k, const void* v, const float* g,
                                          const float* beta, float* state, void* o, int B, int T, int H,
                                          cudaStream_t st);
// Device address of this device's counter of bounded waits that gave up (kernels bump it; the host polls it).
unsigned int* device_timeout_counter();
}  // namespace evie
