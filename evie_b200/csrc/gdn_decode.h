// Launchers of the Gated DeltaNet decode kernels (gdn_decode.cu).
#pragma once
#include "common.h"

namespace evie {
// One recurrent step for `heads` independent [128][128] states; q,k,v bf16.
evie_status launch_gdn_decode_step_bf16(const void* q, const void* k, const void* v, const float* g,
                                        const float* beta, float* state, float* o, int heads, cudaStream_t st);
// Token-sequential prefill of T tokens for B*H heads; o is bf16 [B][T][H][dv].
evie_status launch_gdn_prefill_seq_bf16(const void* q, const void* k, const void* v, const float* g,
                                        const float* beta, float* state, void* o, int B, int T, int H,
                                        cudaStream_t st);
}  // namespace evie
