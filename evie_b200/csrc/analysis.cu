// Offline analysis on the device: evie-core's unembedding statistics and per-neuron logit spread
// (crates/evie-core/src/analysis.rs:129-175 UnembedStats::compute, 183-201 neuron_sigma, without a lens).
//
//   mean_i   = (sum over the V unembedding rows of W_U[r][i], in f64) / V
//   x[j][i]  = (W_U[j * stride][i] - mean_i) * g_i   for a strided subsample of s = min(16384, V) rows
//   C        = x^T . f16(64 x) / (64 s)              (the reference multiplies by the f16-rounded copy)
//   m_scale  = max |C|,  M = f16(C / m_scale)
//   sigma_n  = sqrt(max(u_n . (M u_n) * m_scale, 1e-30)) for every down_proj column u_n of every layer
//
// Dense and tensor-bound (~4 TFLOP at 4B shapes): the two products run as f32 cuBLAS GEMMs on exactly the operands
// the reference forms (f16 roundings included), the rest as small kernels. Only the summation orders differ from
// the CPU engine, so the results agree to f32 rounding of the sums.
#include <cublas_v2.h>

#include <vector>

#include "model_kernels.h"

namespace evie {

namespace {

constexpr int kSumChunks = 64;

// partial[c][i] = sum over rows r of chunk c of W[r][i] (f64)
__global__ void col_partial_sums_kernel(const __nv_bfloat16* __restrict__ W, int V, int d, double* __restrict__ part) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= d) return;
  const int c = blockIdx.y;
  const int r0 = (int)((long)V * c / kSumChunks), r1 = (int)((long)V * (c + 1) / kSumChunks);
  double s = 0.0;
  for (int r = r0; r < r1; r++) s += (double)__bfloat162float(W[(size_t)r * d + i]);
  part[(size_t)c * d + i] = s;
}

__global__ void mean_kernel(const double* __restrict__ part, int V, int d, float* __restrict__ mean) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= d) return;
  double s = 0.0;
  for (int c = 0; c < kSumChunks; c++) s += part[(size_t)c * d + i];
  mean[i] = (float)(s / (double)V);
}

// xt[i][j] = (W[j * stride][i] - mean_i) * g_i and xw = f16(64 xt) widened, both [d][s]
__global__ void centred_kernel(const __nv_bfloat16* __restrict__ W, const float* __restrict__ mean,
                               const float* __restrict__ g, int d, int s, int stride, float* __restrict__ xt,
                               float* __restrict__ xw) {
  const size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= (size_t)d * s) return;
  const int i = (int)(e % d), j = (int)(e / d);  // consecutive threads: consecutive i of one sampled row
  const float x = __fmul_rn(__fsub_rn(__bfloat162float(W[(size_t)j * stride * d + i]), mean[i]), g[i]);
  xt[(size_t)i * s + j] = x;
  xw[(size_t)i * s + j] = __half2float(__float2half_rn(__fmul_rn(x, 64.0f)));
}

// C *= norm, then max |C| into *mx (non-negative floats order as their bit patterns)
__global__ void scale_max_kernel(float* __restrict__ C, size_t n, float norm, unsigned int* __restrict__ mx) {
  unsigned int m = 0;
  for (size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (size_t)gridDim.x * blockDim.x) {
    const float v = __fmul_rn(C[e], norm);
    C[e] = v;
    m = max(m, __float_as_uint(fabsf(v)));
  }
  for (int off = 16; off >= 1; off >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, off));
  if ((threadIdx.x & 31) == 0) atomicMax(mx, m);
}

// M = f16(C / m_scale) widened, m_scale = max(max |C|, 1e-30)
__global__ void quantise_kernel(const float* __restrict__ C, size_t n, const unsigned int* __restrict__ mx,
                                float* __restrict__ M, float* __restrict__ m_scale) {
  const float ms = fmaxf(__uint_as_float(*mx), 1e-30f);
  const size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e == 0) *m_scale = ms;
  if (e < n) M[e] = __half2float(__float2half_rn(__fdiv_rn(C[e], ms)));
}

__global__ void widen_kernel(const __nv_bfloat16* __restrict__ w, size_t n, float* __restrict__ f) {
  const size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e < n) f[e] = __bfloat162float(w[e]);
}

// sigma[i] = sqrt(max(sum_j U[j][i] * MU[j][i] * m_scale, 1e-30)), U and MU [d][n]
__global__ void sigma_kernel(const float* __restrict__ U, const float* __restrict__ MU, int d, int n,
                             const float* __restrict__ m_scale, float* __restrict__ sigma) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float acc = 0.f;
  for (int j = 0; j < d; j++) acc = fmaf(U[(size_t)j * n + i], MU[(size_t)j * n + i], acc);
  sigma[i] = sqrtf(fmaxf(__fmul_rn(acc, *m_scale), 1e-30f));
}

struct DevBufs {
  std::vector<void*> p;
  ~DevBufs() {
    for (void* q : p) cudaFree(q);
  }
  template <typename T>
  evie_status get(T** out, size_t count) {
    void* q = nullptr;
    if (cudaMalloc(&q, count * sizeof(T) + 16) != cudaSuccess) {
      cudaGetLastError();
      return fail(EVIE_ERR_OOM, "neuron_sigma: cannot allocate %zu bytes", count * sizeof(T));
    }
    p.push_back(q);
    *out = static_cast<T*>(q);
    return EVIE_OK;
  }
};

#define AN_TRY(x)                        \
  do {                                   \
    evie_status rc_ = (x);               \
    if (rc_ != EVIE_OK) return rc_;      \
  } while (0)

}  // namespace

evie_status neuron_sigma_run(cublasHandle_t blas, cudaStream_t st, const __nv_bfloat16* lm_head, int V, int d,
                             const float* gain, const std::vector<const __nv_bfloat16*>& w_down, int n, float* sigma,
                             float* mean_out, float* m_scale_out) {
  if (V < 1 || d < 1 || n < 1) return fail(EVIE_ERR_ARG, "neuron_sigma: empty model");
  const int s = V < 16384 ? V : 16384, stride = V / s;
  const int L = (int)w_down.size();
  DevBufs b;
  double* part;
  float *mean, *xt, *xw, *C, *M, *Wf, *MU, *sig, *ms;
  unsigned int* mx;
  AN_TRY(b.get(&part, (size_t)kSumChunks * d));
  AN_TRY(b.get(&mean, d));
  AN_TRY(b.get(&xt, (size_t)d * s));
  AN_TRY(b.get(&xw, (size_t)d * s));
  AN_TRY(b.get(&C, (size_t)d * d));
  AN_TRY(b.get(&M, (size_t)d * d));
  AN_TRY(b.get(&Wf, (size_t)d * n));
  AN_TRY(b.get(&MU, (size_t)d * n));
  AN_TRY(b.get(&sig, (size_t)L * n));
  AN_TRY(b.get(&ms, 1));
  AN_TRY(b.get(&mx, 1));
  EVIE_CUDA_TRY(cudaMemsetAsync(mx, 0, sizeof(unsigned int), st));
  col_partial_sums_kernel<<<dim3((d + 127) / 128, kSumChunks), 128, 0, st>>>(lm_head, V, d, part);
  EVIE_CHECK_LAUNCH("col_partial_sums_kernel");
  mean_kernel<<<(d + 127) / 128, 128, 0, st>>>(part, V, d, mean);
  EVIE_CHECK_LAUNCH("mean_kernel");
  const size_t nx = (size_t)d * s;
  centred_kernel<<<(unsigned)((nx + 255) / 256), 256, 0, st>>>(lm_head, mean, gain, d, s, stride, xt, xw);
  EVIE_CHECK_LAUNCH("centred_kernel");
  cublasSetStream(blas, st);
  const float one = 1.0f, zero = 0.0f;
  // C[t][r] = sum_k xt[t][k] xw[r][k]  (row-major d x d)
  if (cublasSgemm(blas, CUBLAS_OP_T, CUBLAS_OP_N, d, d, s, &one, xw, s, xt, s, &zero, C, d) != CUBLAS_STATUS_SUCCESS)
    return fail(EVIE_ERR_CUDA, "neuron_sigma: covariance GEMM failed");
  scale_max_kernel<<<1184, 256, 0, st>>>(C, (size_t)d * d, 1.0f / ((float)s * 64.0f), mx);
  EVIE_CHECK_LAUNCH("scale_max_kernel");
  quantise_kernel<<<(unsigned)(((size_t)d * d + 255) / 256), 256, 0, st>>>(C, (size_t)d * d, mx, M, ms);
  EVIE_CHECK_LAUNCH("quantise_kernel");
  for (int l = 0; l < L; l++) {
    const size_t nw = (size_t)d * n;
    widen_kernel<<<(unsigned)((nw + 255) / 256), 256, 0, st>>>(w_down[l], nw, Wf);
    EVIE_CHECK_LAUNCH("widen_kernel");
    // MU[j][i] = sum_k M[j][k] Wf[k][i]  (row-major d x n)
    if (cublasSgemm(blas, CUBLAS_OP_N, CUBLAS_OP_N, n, d, d, &one, Wf, n, M, d, &zero, MU, n) !=
        CUBLAS_STATUS_SUCCESS)
      return fail(EVIE_ERR_CUDA, "neuron_sigma: projection GEMM failed");
    sigma_kernel<<<(n + 255) / 256, 256, 0, st>>>(Wf, MU, d, n, ms, sig + (size_t)l * n);
    EVIE_CHECK_LAUNCH("sigma_kernel");
  }
  EVIE_CUDA_TRY(cudaMemcpyAsync(sigma, sig, (size_t)L * n * sizeof(float), cudaMemcpyDeviceToHost, st));
  if (mean_out) EVIE_CUDA_TRY(cudaMemcpyAsync(mean_out, mean, (size_t)d * sizeof(float), cudaMemcpyDeviceToHost, st));
  float msh = 0.f;
  EVIE_CUDA_TRY(cudaMemcpyAsync(&msh, ms, sizeof(float), cudaMemcpyDeviceToHost, st));
  EVIE_CUDA_TRY(cudaStreamSynchronize(st));
  if (m_scale_out) *m_scale_out = msh;
  return EVIE_OK;
}

}  // namespace evie
