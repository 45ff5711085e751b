// Projection GEMM on sm_100a tensor cores (proj_gemm.cu): every weight projection of the forward pass and the LM
// head. The reference multiplies bf16 weights by f32 activations (crates/evie-core/src/kernels.rs:138-268, `matmul`
// / `matvec`; the wgpu twins `matmul_small` / `matmul_tiled`, gpu/kernels.wgsl:112-235).
#pragma once
#include "common.h"

namespace evie {

// Y = X W^T for W [M][K] bf16 (row-major, 16-byte aligned rows: K % 8 == 0) and X [R][K] f32 given as the two
// bf16 planes X2 = [hi; lo] ([2][R][K], hi = bf16(X), lo = bf16(X - hi)). The hi and lo products accumulate in the
// same f32 tensor-memory accumulator, so the result is one plane per K slice:
//   y[s][r][m] = sum over k in slice s of W[m][k] (hi[r][k] + lo[r][k]),   s = 0 .. *planes - 1,
// and the consumer adds the planes in slice order (YView). Decode-shaped calls (R <= 128) cut K into slices so
// that the weight stream fills every SM; larger R runs one slice over persistent 128 x 256 tiles.
//   y_cap      floats available at y (the planes must fit: planes * R * M <= y_cap)
//   max_planes upper bound on the K slices (>= 1)
//   pdl        launch with programmatic stream serialisation: the kernel streams its first weight tiles before it
//              waits for the previous kernel in the stream (weights do not depend on it), then loads X2.
//   timeouts   device counter bumped when a bounded wait gives up
struct ProjGemmPlan {
  int bm = 0, br = 0, ksplit = 0, grid = 0, units = 0;
};
ProjGemmPlan plan_proj_gemm(int M, int K, int R, int max_planes, size_t y_cap, int num_sms);
evie_status launch_proj_gemm(const __nv_bfloat16* W, int M, int K, const __nv_bfloat16* X2, int R, float* y,
                             size_t y_cap, int max_planes, bool pdl, cudaStream_t st, int* planes);

}  // namespace evie
