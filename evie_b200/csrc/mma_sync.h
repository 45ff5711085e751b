// Warp-level bf16 tensor-core helpers (mma.sync m16n8k16) shared by the attention kernels.
#pragma once
#include <cuda_bf16.h>
#include <stdint.h>

namespace evie {

// D[16x8] += A[16x16] . B[16x8], bf16 inputs, f32 accumulation. Fragments per lane (g = lane / 4, c = lane % 4):
// a0 = A[g][2c..2c+1], a1 = A[g+8][2c..2c+1], a2 = A[g][2c+8..2c+9], a3 = A[g+8][2c+8..2c+9];
// b0 = B[2c..2c+1][g], b1 = B[2c+8..2c+9][g]; d = {D[g][2c], D[g][2c+1], D[g+8][2c], D[g+8][2c+1]}.
__device__ __forceinline__ void mma_bf16_16816(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
__device__ __forceinline__ uint4 ldg_stream128(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
__device__ __forceinline__ uint32_t word_of(const uint4& u, int i) {
  return i == 0 ? u.x : i == 1 ? u.y : i == 2 ? u.z : u.w;
}

}  // namespace evie
