// Launchers of the gated GQA decode-attention kernels (gqa_decode.cu).
#pragma once
#include "common.h"

namespace evie {
// Longest context one call can cover: the split merge stages GROUP x splits weights in shared memory.
constexpr long kGqaMaxContext = 512L * 512L;

evie_status launch_gqa_decode_bf16(const void* q, const void* gate, const void* kp, const void* vp,
                                   const int32_t* page_table, const int32_t* ctx_lens, float* out, int B, int Hq,
                                   int Hkv, int page_size, int max_pages, float scale, cudaStream_t st);
struct RowInfo;
struct YView;
// Scratch bytes the model's attention needs for `rows` query rows (tickets must start zeroed).
size_t gqa_scratch_bytes(int rows, int Hkv, int group, int max_ctx);
// Model variant: one query per row (ctx = pos + 1), KV in bf16 or f32 pages, output into the o_proj planes.
template <typename KV>
evie_status launch_gqa_model(const float* q_rot, YView y, int ldy, __nv_bfloat16* X2,
                             size_t xplane, const RowInfo* rows, int R, const int* page_table, int pages_per_slot,
                             const KV* kc, const KV* vc, int Hq, int Hkv, int page_size, int max_ctx, float scale,
                             void* scratch, int ticket_rows, cudaStream_t st);
struct SegInfo;
// Prefill rows (several rows per segment): flash-style blocks of 16 rows per KV head over bf16 pages, GQA group 4,
// page size a multiple of 32 (gqa_prefill.cu). max_seg_rows = the largest segment's row count.
evie_status launch_gqa_prefill_model(const float* q_rot, YView y, int ldy, __nv_bfloat16* X2, size_t xplane,
                                     const RowInfo* rows, const SegInfo* segs, int nseg, int max_seg_rows,
                                     const int* page_table, int pages_per_slot, const __nv_bfloat16* kc,
                                     const __nv_bfloat16* vc, int Hq, int Hkv, int page_size, float scale,
                                     cudaStream_t st);
// The same rows on tcgen05 tensor cores (gqa_prefill_tc.cu): blocks of 32 rows x the 4 query heads of a KV head,
// 64-token K/V tiles by TMA, S and O accumulated in tensor memory. cache_rows = pages x Hkv x page_size (the rows of
// the cache viewed as [rows][256]); page size a multiple of 64.
evie_status launch_gqa_prefill_tc_model(const float* q_rot, YView y, int ldy, __nv_bfloat16* X2, size_t xplane,
                                        const SegInfo* segs, int nseg, int max_seg_rows, const int* page_table,
                                        int pages_per_slot, const __nv_bfloat16* kc, const __nv_bfloat16* vc,
                                        long cache_rows, int Hq, int Hkv, int page_size, float scale,
                                        cudaStream_t st);
}  // namespace evie
