// Launchers of the gated GQA decode-attention kernels (gqa_decode.cu).
#pragma once
#include "common.h"

namespace evie {
// Longest context one call can cover: the split merge stages GROUP x splits weights in shared memory.
constexpr long kGqaMaxContext = 512L * 512L;

evie_status launch_gqa_decode_bf16(const void* q, const void* gate, const void* kp, const void* vp,
                                   const int32_t* page_table, const int32_t* ctx_lens, float* out, int B, int Hq,
                                   int Hkv, int page_size, int max_pages, float scale, cudaStream_t st);
}  // namespace evie
