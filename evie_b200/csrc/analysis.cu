// Offline analysis on the device: evie-core's lenses and readouts (crates/evie-core/src/lens.rs:10-83,
// analysis.rs:28-67 lens_logits / write_dirs / neuron_logits), unembedding statistics and per-neuron logit spread
// (analysis.rs:129-179 UnembedStats, 183-201 neuron_sigma) and neuron search (analysis.rs:213-251).
//
//   mean_i   = (sum over the V unembedding rows of W_U[r][i], in f64) / V
//   x[j][i]  = (W_U[j * stride][i] - mean_i) * g_i   for a strided subsample of s = min(16384, V) rows
//   C        = x^T . f16(64 x) / (64 s)              (the reference multiplies by the f16-rounded copy)
//   m_scale  = max |C|,  M = f16(C / m_scale)
//   u_n      = J_l w_n (w_n the down_proj column of neuron n; J_l the lens map of layer l, or the identity)
//   sigma_n  = sqrt(max(u_n . (M u_n) * m_scale, 1e-30))
//   lens logits of vectors h at layer l: unembed(J_l h) = W_U rmsnorm(J_l h)
//   search:  z_t(n) = (W_down^T J_l^T a_t)_n / sigma_n,  a_t = (W_U[t] - mean) * g
//
// Every product runs on the projection GEMM (proj_gemm.cu), which multiplies a bf16 weight matrix by an f32 operand
// given as two bf16 planes (hi + lo, ~16 significant bits) with f32 accumulation. The 16-bit matrices the reference
// multiplies (bf16 weights, the f16 lens maps, the f16-rounded covariance operands) enter as exact bf16 planes
// (Planes16), so only the f32 operands are rounded, to 2^-17 relative; the rest are small kernels. Summation orders
// differ from the CPU engine, so results agree to f32 rounding of the sums.
#include <algorithm>
#include <cstring>
#include <numeric>

#include "analysis.h"
#include "gdn_chunk.h"
#include "model_kernels.h"
#include "proj_gemm.h"

namespace evie {

const Planes16* LensDev::map(int layer) const {
  if (layer < 0 || (long)layer > target || layer >= (int)J.size() || J[layer].planes == 0) return nullptr;
  return &J[layer];
}
const Planes16* LensDev::map_t(int layer) const {
  const Planes16* m = map(layer);
  return m ? &JT[layer] : nullptr;
}

namespace {

constexpr int kSumChunks = 64;
constexpr int kRowsPerUnembed = 64;  // readout rows per LM-head product

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

// xt[i][j] = (W[j * stride][i] - mean_i) * g_i ([d][ld] f32, j < s) and the exact bf16 planes of f16(64 xt)
// ([2][d][ld]); columns s .. ld - 1 are left as they are (zero)
__global__ void centred_kernel(const __nv_bfloat16* __restrict__ W, const float* __restrict__ mean,
                               const float* __restrict__ g, int d, int s, int ld, int stride, float* __restrict__ xt,
                               __nv_bfloat16* __restrict__ xw2) {
  const size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= (size_t)d * s) return;
  const int i = (int)(e % d), j = (int)(e / d);  // consecutive threads: consecutive i of one sampled row
  const float x = __fmul_rn(__fsub_rn(__bfloat162float(W[(size_t)j * stride * d + i]), mean[i]), g[i]);
  xt[(size_t)i * ld + j] = x;
  store_split(xw2, (size_t)d * ld, (size_t)i * ld + j, __half2float(__float2half_rn(__fmul_rn(x, 64.0f))));
}

// X2 = [hi; lo] planes of the n values of x: hi = bf16(x), lo = bf16(x - hi)
__global__ void split_kernel(YView x, size_t n, __nv_bfloat16* __restrict__ X2) {
  for (size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (size_t)gridDim.x * blockDim.x)
    store_split(X2, n, e, x.at(e));
}

// out = x (its planes added)
__global__ void sum_planes_kernel(YView x, size_t n, float* __restrict__ out) {
  for (size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (size_t)gridDim.x * blockDim.x)
    out[e] = x.at(e);
}

// C = x * norm (planes added), then max |C| into *mx (non-negative floats order as their bit patterns)
__global__ void scale_max_kernel(YView x, size_t n, float norm, float* __restrict__ C, unsigned int* __restrict__ mx) {
  unsigned int m = 0;
  for (size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (size_t)gridDim.x * blockDim.x) {
    const float v = __fmul_rn(x.at(e), norm);
    C[e] = v;
    m = max(m, __float_as_uint(fabsf(v)));
  }
  for (int off = 16; off >= 1; off >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, off));
  if ((threadIdx.x & 31) == 0) atomicMax(mx, m);
}

// M = f16(C / m_scale) as exact bf16 planes [2][n], m_scale = max(max |C|, 1e-30)
__global__ void quantise_kernel(const float* __restrict__ C, size_t n, const unsigned int* __restrict__ mx,
                                __nv_bfloat16* __restrict__ M2, float* __restrict__ m_scale) {
  const float ms = fmaxf(__uint_as_float(*mx), 1e-30f);
  const size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e == 0) *m_scale = ms;
  if (e < n) store_split(M2, n, e, __half2float(__float2half_rn(__fdiv_rn(C[e], ms))));
}

// WT[c][r] = W[r][c] for a [rows][cols] bf16 matrix, through 32 x 32 shared-memory tiles
__global__ void transpose_kernel(const __nv_bfloat16* __restrict__ W, int rows, int cols, __nv_bfloat16* __restrict__ WT) {
  __shared__ __nv_bfloat16 tile[32][33];
  const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32, tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8 threads
  for (int k = ty; k < 32; k += 8) {
    const int r = r0 + k, c = c0 + tx;
    if (r < rows && c < cols) tile[k][tx] = W[(size_t)r * cols + c];
  }
  __syncthreads();
  for (int k = ty; k < 32; k += 8) {
    const int c = c0 + k, r = r0 + tx;
    if (c < cols && r < rows) WT[(size_t)c * rows + r] = tile[tx][k];
  }
}

// A host-given 16-bit [d][d] matrix (f16 or bf16 bits), or its transpose, as exact bf16 planes [planes][d][d]
__global__ void planes16_kernel(const uint16_t* __restrict__ src, int d, int is_f16, int transpose,
                                __nv_bfloat16* __restrict__ dst) {
  const size_t n = (size_t)d * d;
  for (size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (size_t)gridDim.x * blockDim.x) {
    const size_t r = e / d, c = e % d;
    const uint16_t b = src[transpose ? c * d + r : e];
    if (is_f16) store_split(dst, n, e, __half2float(__ushort_as_half(b)));
    else dst[e] = __ushort_as_bfloat16(b);
  }
}

// sigma[i] = sqrt(max(sum_k u[i][k] mu[i][k] * m_scale, 1e-30)); u from ub (bf16 [n][d]) when given, else from u.
// One warp per neuron.
__global__ void sigma_kernel(const __nv_bfloat16* __restrict__ ub, YView u, YView mu, int n, int d,
                             const float* __restrict__ m_scale, float* __restrict__ sigma) {
  const int i = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (i >= n) return;
  float acc = 0.f;
  for (int k = lane; k < d; k += 32) {
    const size_t e = (size_t)i * d + k;
    acc = fmaf(ub ? __bfloat162float(ub[e]) : u.at(e), mu.at(e), acc);
  }
  for (int off = 16; off >= 1; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) sigma[i] = sqrtf(fmaxf(__fmul_rn(acc, *m_scale), 1e-30f));
}

// model.rs:287-294 + kernels.rs:607-613: X2 rows = split(x / rms(x) * g) for R rows of width d (one CTA per row)
__global__ void __launch_bounds__(256) norm_rows_kernel(YView x, int d, const float* __restrict__ g, float eps,
                                                        size_t plane, __nv_bfloat16* __restrict__ X2) {
  __shared__ float red[8];
  const int r = blockIdx.x;
  float ss = 0.f;
  for (int i = threadIdx.x; i < d; i += 256) {
    const float v = x.at((size_t)r * d + i);
    ss = fmaf(v, v, ss);
  }
  for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float t = 0.f;
  for (int w = 0; w < 8; w++) t += red[w];
  const float inv = 1.0f / sqrtf(t / (float)d + eps);
  for (int i = threadIdx.x; i < d; i += 256) {
    const size_t e = (size_t)r * d + i;
    store_split(X2, plane, e, x.at(e) * inv * g[i]);
  }
}

// analysis.rs:37-43 (write_dirs): dirs[r][k] = W_down[k][col[r]] of row r's layer (bases[r], [d][n])
__global__ void gather_cols_kernel(const __nv_bfloat16* const* __restrict__ bases, const int* __restrict__ cols,
                                   int d, int n, float* __restrict__ dirs) {
  const int r = blockIdx.y;
  const int k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k < d) dirs[(size_t)r * d + k] = __bfloat162float(bases[r][(size_t)k * n + cols[r]]);
}

// analysis.rs:173-179 (centered): a[t][i] = (W_U[tokens[t]][i] - mean_i) * g_i
__global__ void centered_rows_kernel(const __nv_bfloat16* __restrict__ W, const uint32_t* __restrict__ tokens, int d,
                                     const float* __restrict__ mean, const float* __restrict__ g,
                                     float* __restrict__ a) {
  const int t = blockIdx.y, i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < d)
    a[(size_t)t * d + i] = __fmul_rn(__fsub_rn(__bfloat162float(W[(size_t)tokens[t] * d + i]), mean[i]), g[i]);
}

// analysis.rs:229-240: per neuron, the best z = score / sigma over the tokens for each pole
__global__ void zscore_kernel(YView scores, int nt, int n, const float* __restrict__ sigma, float* __restrict__ z_up,
                              float* __restrict__ z_dn) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float up = -INFINITY, dn = -INFINITY;
  for (int t = 0; t < nt; t++) {
    const float z = __fdiv_rn(scores.at((size_t)t * n + i), sigma[i]);
    up = fmaxf(up, z);
    dn = fmaxf(dn, -z);
  }
  z_up[i] = up;
  z_dn[i] = dn;
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
      return fail(EVIE_ERR_OOM, "analysis: cannot allocate %zu bytes", count * sizeof(T));
    }
    p.push_back(q);
    *out = static_cast<T*>(q);
    return EVIE_OK;
  }
};

unsigned grid_for(size_t n, int threads = 256) {
  return (unsigned)std::min<size_t>((n + threads - 1) / threads, 148 * 16);
}

evie_status split(YView x, size_t n, __nv_bfloat16* X2, cudaStream_t st) {
  split_kernel<<<grid_for(n), 256, 0, st>>>(x, n, X2);
  EVIE_CHECK_LAUNCH("split_kernel");
  return EVIE_OK;
}

YView dense(const float* p, size_t n) { return YView{p, n, 1}; }

// y = X W^T summed over W's planes: each plane's product is appended to y as its own K-slice planes, so the result
// is one YView. X2 = [2][R][W.cols]; y holds at most y_cap floats.
constexpr int kSlicesPerPlane = YView::kMaxPlanes / 2;
size_t product_cap(const Planes16& W, int R) { return (size_t)W.planes * (R <= 128 ? kSlicesPerPlane : 1) * R * W.rows; }
evie_status product(const Planes16& W, const __nv_bfloat16* X2, int R, float* y, size_t y_cap, cudaStream_t st,
                    YView* out) {
  const size_t plane = (size_t)R * W.rows;
  int used = 0;
  for (int p = 0; p < W.planes; p++) {
    int planes = 0;
    if ((size_t)(used + 1) * plane > y_cap) return fail(EVIE_ERR_ARG, "analysis: product output exceeds its buffer");
    EVIE_TRY(launch_proj_gemm(W.p + (size_t)p * W.rows * W.cols, W.rows, W.cols, X2, R, y + (size_t)used * plane,
                              y_cap - (size_t)used * plane, kSlicesPerPlane, false, st, &planes));
    used += planes;
  }
  *out = YView{y, plane, used};
  return EVIE_OK;
}

evie_status transpose(const __nv_bfloat16* W, int rows, int cols, __nv_bfloat16* WT, cudaStream_t st) {
  transpose_kernel<<<dim3((cols + 31) / 32, (rows + 31) / 32), dim3(32, 8), 0, st>>>(W, rows, cols, WT);
  EVIE_CHECK_LAUNCH("transpose_kernel");
  return EVIE_OK;
}

// Reads the bounded-wait give-up counter (after the stream's work): the analysis calls report a give-up of any
// projection-GEMM wait they launched as EVIE_ERR_TIMEOUT.
evie_status read_timeouts(cudaStream_t st, unsigned int* v) {
  unsigned int* c = device_timeout_counter();
  if (!c) return fail(EVIE_ERR_CUDA, "device timeout counter unavailable");
  EVIE_CUDA_TRY(cudaMemcpyAsync(v, c, sizeof *v, cudaMemcpyDeviceToHost, st));
  EVIE_CUDA_TRY(cudaStreamSynchronize(st));
  return EVIE_OK;
}

struct TimeoutGuard {
  cudaStream_t st;
  unsigned int before = 0;
  evie_status begin() { return read_timeouts(st, &before); }
  evie_status end() {
    unsigned int after = 0;
    EVIE_TRY(read_timeouts(st, &after));
    if (after != before) return fail(EVIE_ERR_TIMEOUT, "analysis: %u bounded wait(s) gave up", after - before);
    return EVIE_OK;
  }
};

// unembed (model.rs:287-294) of the R rows of t (width d) into dense logits [R][V] on the device, in blocks of
// kRowsPerUnembed rows. X2 holds [2][kRowsPerUnembed][d], y product_cap(lm_head, kRowsPerUnembed) floats.
evie_status unembed(const AnalysisModel& am, YView t, int R, __nv_bfloat16* X2, float* y, size_t y_cap,
                    float* logits) {
  const Planes16 head{am.lm_head, 1, am.V, am.d};
  for (int r0 = 0; r0 < R; r0 += kRowsPerUnembed) {
    const int nr = std::min(kRowsPerUnembed, R - r0);
    YView tv{t.p + (size_t)r0 * am.d, t.plane, t.n};
    norm_rows_kernel<<<nr, 256, 0, am.st>>>(tv, am.d, am.final_norm, am.eps, (size_t)nr * am.d, X2);
    EVIE_CHECK_LAUNCH("norm_rows_kernel");
    YView lg;
    EVIE_TRY(product(head, X2, nr, y, y_cap, am.st, &lg));
    const size_t n = (size_t)nr * am.V;
    sum_planes_kernel<<<grid_for(n), 256, 0, am.st>>>(lg, n, logits + (size_t)r0 * am.V);
    EVIE_CHECK_LAUNCH("sum_planes_kernel");
  }
  return EVIE_OK;
}

}  // namespace

evie_status lens_upload(LensDev& lens, const uint16_t* const* maps, int n_layers, int d, int kind, long target,
                        cudaStream_t st) {
  if (kind != 0 && kind != 1) return fail(EVIE_ERR_ARG, "lens: kind must be 0 (f16) or 1 (bf16)");
  lens_free(lens);
  const int planes = kind == 0 ? 2 : 1;
  const size_t per = (size_t)planes * d * d;  // elements per map (J or JT)
  int count = 0;
  for (int l = 0; l < n_layers; l++) count += maps[l] != nullptr;
  lens.J.assign(n_layers, Planes16{});
  lens.JT.assign(n_layers, Planes16{});
  lens.target = target;
  if (count == 0) return EVIE_OK;
  if (cudaMalloc(&lens.mem, 2 * per * count * sizeof(__nv_bfloat16)) != cudaSuccess) {
    cudaGetLastError();
    lens.mem = nullptr;
    return fail(EVIE_ERR_OOM, "lens: cannot allocate %zu bytes", 2 * per * count * sizeof(__nv_bfloat16));
  }
  uint16_t* stage = nullptr;
  if (cudaMalloc(&stage, (size_t)d * d * sizeof(uint16_t)) != cudaSuccess) {
    cudaGetLastError();
    lens_free(lens);
    return fail(EVIE_ERR_OOM, "lens: cannot allocate the staging buffer");
  }
  auto* base = static_cast<__nv_bfloat16*>(lens.mem);
  evie_status rc = EVIE_OK;
  int k = 0;
  for (int l = 0; l < n_layers && rc == EVIE_OK; l++) {
    if (!maps[l]) continue;
    __nv_bfloat16* j = base + (size_t)(2 * k) * per;
    __nv_bfloat16* jt = j + per;
    k++;
    cudaError_t e = cudaMemcpyAsync(stage, maps[l], (size_t)d * d * sizeof(uint16_t), cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) {
      rc = fail(EVIE_ERR_CUDA, "lens upload: %s", cudaGetErrorString(e));
      break;
    }
    planes16_kernel<<<grid_for((size_t)d * d), 256, 0, st>>>(stage, d, kind == 0, 0, j);
    planes16_kernel<<<grid_for((size_t)d * d), 256, 0, st>>>(stage, d, kind == 0, 1, jt);
    if ((e = cudaGetLastError()) != cudaSuccess) {
      rc = fail(EVIE_ERR_CUDA, "planes16_kernel: %s", cudaGetErrorString(e));
      break;
    }
    lens.J[l] = Planes16{j, planes, d, d};
    lens.JT[l] = Planes16{jt, planes, d, d};
    // the staging buffer is reused by the next layer's copy, which the stream orders after these kernels; the
    // host array must stay valid until then: synchronise per layer
    if ((e = cudaStreamSynchronize(st)) != cudaSuccess) rc = fail(EVIE_ERR_CUDA, "lens upload: %s", cudaGetErrorString(e));
  }
  cudaFree(stage);
  if (rc != EVIE_OK) lens_free(lens);
  return rc;
}

void lens_free(LensDev& lens) {
  if (lens.mem) cudaFree(lens.mem);
  lens.mem = nullptr;
  lens.J.clear();
  lens.JT.clear();
  lens.target = -1;
}

evie_status neuron_sigma_run(const AnalysisModel& am, float* sigma, float* mean_out, float* m_scale_out) {
  const int V = am.V, d = am.d, n = am.n, L = (int)am.w_down.size();
  if (V < 1 || d < 1 || n < 1 || L < 1) return fail(EVIE_ERR_ARG, "neuron_sigma: empty model");
  if (d % 8 != 0) return fail(EVIE_ERR_ARG, "neuron_sigma: hidden size %d must be a multiple of 8", d);
  const int s = V < 16384 ? V : 16384, stride = V / s;
  const int s8 = (s + 7) / 8 * 8;  // the covariance's K, padded to whole 16-byte rows (padding is zero in both)
  cudaStream_t st = am.st;
  TimeoutGuard tg{st};
  EVIE_TRY(tg.begin());
  DevBufs b;
  double* part;
  float *mean, *xt, *yC, *Cd, *yU, *yMU, *sig, *ms;
  __nv_bfloat16 *xw2, *X2c, *M2, *X2u, *X2m;
  unsigned int* mx;
  const Planes16 Wx{nullptr, 2, d, s8};
  EVIE_TRY(b.get(&part, (size_t)kSumChunks * d));
  EVIE_TRY(b.get(&mean, d));
  EVIE_TRY(b.get(&xt, (size_t)d * s8));
  EVIE_TRY(b.get(&xw2, (size_t)2 * d * s8));
  EVIE_TRY(b.get(&X2c, (size_t)2 * d * s8));
  EVIE_TRY(b.get(&yC, product_cap(Wx, d)));
  EVIE_TRY(b.get(&Cd, (size_t)d * d));
  EVIE_TRY(b.get(&M2, (size_t)2 * d * d));
  EVIE_TRY(b.get(&X2u, (size_t)2 * n * d));
  EVIE_TRY(b.get(&X2m, (size_t)2 * n * d));
  const Planes16 Mp{M2, 2, d, d};
  EVIE_TRY(b.get(&yU, product_cap(Mp, n)));
  EVIE_TRY(b.get(&yMU, product_cap(Mp, n)));
  EVIE_TRY(b.get(&sig, (size_t)L * n));
  EVIE_TRY(b.get(&ms, 1));
  EVIE_TRY(b.get(&mx, 1));
  EVIE_CUDA_TRY(cudaMemsetAsync(mx, 0, sizeof(unsigned int), st));
  if (s8 != s) {  // the padding columns of both covariance operands stay zero
    EVIE_CUDA_TRY(cudaMemsetAsync(xt, 0, (size_t)d * s8 * sizeof(float), st));
    EVIE_CUDA_TRY(cudaMemsetAsync(xw2, 0, (size_t)2 * d * s8 * sizeof(__nv_bfloat16), st));
  }
  col_partial_sums_kernel<<<dim3((d + 127) / 128, kSumChunks), 128, 0, st>>>(am.lm_head, V, d, part);
  EVIE_CHECK_LAUNCH("col_partial_sums_kernel");
  mean_kernel<<<(d + 127) / 128, 128, 0, st>>>(part, V, d, mean);
  EVIE_CHECK_LAUNCH("mean_kernel");
  const size_t nx = (size_t)d * s;
  centred_kernel<<<(unsigned)((nx + 255) / 256), 256, 0, st>>>(am.lm_head, mean, am.final_norm, d, s, s8, stride, xt,
                                                               xw2);
  EVIE_CHECK_LAUNCH("centred_kernel");
  // C[r][o] = sum_j f16(64 x)[o][j] x[r][j]  (analysis.rs:164: matmul(xm, xt))
  YView C;
  EVIE_TRY(split(dense(xt, (size_t)d * s8), (size_t)d * s8, X2c, st));
  EVIE_TRY(product(Planes16{xw2, 2, d, s8}, X2c, d, yC, product_cap(Wx, d), st, &C));
  scale_max_kernel<<<grid_for((size_t)d * d), 256, 0, st>>>(C, (size_t)d * d, 1.0f / ((float)s * 64.0f), Cd, mx);
  EVIE_CHECK_LAUNCH("scale_max_kernel");
  quantise_kernel<<<(unsigned)(((size_t)d * d + 255) / 256), 256, 0, st>>>(Cd, (size_t)d * d, mx, M2, ms);
  EVIE_CHECK_LAUNCH("quantise_kernel");
  // X2u = [W_down^T ; 0]: the transposed bf16 columns are exact, so the lo plane is zero
  EVIE_CUDA_TRY(cudaMemsetAsync(X2u + (size_t)n * d, 0, (size_t)n * d * sizeof(__nv_bfloat16), st));
  for (int l = 0; l < L; l++) {
    EVIE_TRY(transpose(am.w_down[l], d, n, X2u, st));
    const Planes16* J = am.lens ? am.lens->map(l) : nullptr;
    YView MU;
    if (J) {  // u = J_l w (analysis.rs:188-191), then M u
      YView U;
      EVIE_TRY(product(*J, X2u, n, yU, product_cap(Mp, n), st, &U));
      EVIE_TRY(split(U, (size_t)n * d, X2m, st));
      EVIE_TRY(product(Mp, X2m, n, yMU, product_cap(Mp, n), st, &MU));
      sigma_kernel<<<(n + 7) / 8, 256, 0, st>>>(nullptr, U, MU, n, d, ms, sig + (size_t)l * n);
    } else {
      EVIE_TRY(product(Mp, X2u, n, yMU, product_cap(Mp, n), st, &MU));
      sigma_kernel<<<(n + 7) / 8, 256, 0, st>>>(X2u, YView{}, MU, n, d, ms, sig + (size_t)l * n);
    }
    EVIE_CHECK_LAUNCH("sigma_kernel");
  }
  EVIE_CUDA_TRY(cudaMemcpyAsync(sigma, sig, (size_t)L * n * sizeof(float), cudaMemcpyDeviceToHost, st));
  if (mean_out) EVIE_CUDA_TRY(cudaMemcpyAsync(mean_out, mean, (size_t)d * sizeof(float), cudaMemcpyDeviceToHost, st));
  float msh = 0.f;
  EVIE_CUDA_TRY(cudaMemcpyAsync(&msh, ms, sizeof(float), cudaMemcpyDeviceToHost, st));
  EVIE_TRY(tg.end());
  if (m_scale_out) *m_scale_out = msh;
  return EVIE_OK;
}

evie_status lens_logits_run(const AnalysisModel& am, int layer, const float* vecs, int n, float* logits) {
  const int d = am.d;
  if (n < 1) return EVIE_OK;
  if (layer < 0 || layer >= (int)am.w_down.size()) return fail(EVIE_ERR_ARG, "lens_logits: bad layer %d", layer);
  cudaStream_t st = am.st;
  TimeoutGuard tg{st};
  EVIE_TRY(tg.begin());
  DevBufs b;
  float *x, *yT, *t, *yL, *lg;
  __nv_bfloat16 *X2, *X2n;
  const Planes16 head{am.lm_head, 1, am.V, d};
  const Planes16* J = am.lens ? am.lens->map(layer) : nullptr;
  EVIE_TRY(b.get(&x, (size_t)n * d));
  EVIE_TRY(b.get(&t, (size_t)n * d));
  EVIE_TRY(b.get(&X2, (size_t)2 * n * d));
  EVIE_TRY(b.get(&yT, J ? product_cap(*J, n) : 1));
  EVIE_TRY(b.get(&X2n, (size_t)2 * kRowsPerUnembed * d));
  EVIE_TRY(b.get(&yL, product_cap(head, kRowsPerUnembed)));
  const int blk = std::min(n, 1024);  // logits rows per device block
  EVIE_TRY(b.get(&lg, (size_t)blk * am.V));
  EVIE_CUDA_TRY(cudaMemcpyAsync(x, vecs, (size_t)n * d * sizeof(float), cudaMemcpyHostToDevice, st));
  YView tv = dense(x, (size_t)n * d);
  if (J) {  // lens.rs:64-73 (transport)
    YView T;
    EVIE_TRY(split(tv, (size_t)n * d, X2, st));
    EVIE_TRY(product(*J, X2, n, yT, product_cap(*J, n), st, &T));
    sum_planes_kernel<<<grid_for((size_t)n * d), 256, 0, st>>>(T, (size_t)n * d, t);
    EVIE_CHECK_LAUNCH("sum_planes_kernel");
    tv = dense(t, (size_t)n * d);
  }
  for (int r0 = 0; r0 < n; r0 += blk) {
    const int nr = std::min(blk, n - r0);
    EVIE_TRY(unembed(am, YView{tv.p + (size_t)r0 * d, tv.plane, 1}, nr, X2n, yL, product_cap(head, kRowsPerUnembed),
                     lg));
    EVIE_CUDA_TRY(cudaMemcpyAsync(logits + (size_t)r0 * am.V, lg, (size_t)nr * am.V * sizeof(float),
                                  cudaMemcpyDeviceToHost, st));
    EVIE_CUDA_TRY(cudaStreamSynchronize(st));
  }
  return tg.end();
}

evie_status neuron_logits_run(const AnalysisModel& am, const int32_t* layers, const int32_t* neurons, int n,
                              float* logits) {
  const int d = am.d, L = (int)am.w_down.size();
  if (n < 1) return EVIE_OK;
  for (int i = 0; i < n; i++)
    if (layers[i] < 0 || layers[i] >= L || neurons[i] < 0 || neurons[i] >= am.n)
      return fail(EVIE_ERR_ARG, "neuron_logits: bad neuron (%d, %d)", layers[i], neurons[i]);
  cudaStream_t st = am.st;
  TimeoutGuard tg{st};
  EVIE_TRY(tg.begin());
  // rows grouped by layer (ascending, input order inside a layer), as analysis.rs:50-60 transports them
  std::vector<int> order(n);
  std::iota(order.begin(), order.end(), 0);
  std::stable_sort(order.begin(), order.end(), [&](int a, int c) { return layers[a] < layers[c]; });
  std::vector<const __nv_bfloat16*> bases(n);
  std::vector<int> cols(n);
  for (int j = 0; j < n; j++) {
    bases[j] = am.w_down[layers[order[j]]];
    cols[j] = neurons[order[j]];
  }
  DevBufs b;
  const __nv_bfloat16** dbases;
  int* dcols;
  float *dirs, *yT, *yL, *lg;
  __nv_bfloat16 *X2, *X2n;
  const Planes16 head{am.lm_head, 1, am.V, d};
  size_t tcap = 1;
  if (am.lens)
    for (int l = 0; l < L; l++)
      if (const Planes16* J = am.lens->map(l)) tcap = std::max(tcap, product_cap(*J, n));
  EVIE_TRY(b.get(&dbases, n));
  EVIE_TRY(b.get(&dcols, n));
  EVIE_TRY(b.get(&dirs, (size_t)n * d));
  EVIE_TRY(b.get(&X2, (size_t)2 * n * d));
  EVIE_TRY(b.get(&yT, tcap));
  EVIE_TRY(b.get(&X2n, (size_t)2 * kRowsPerUnembed * d));
  EVIE_TRY(b.get(&yL, product_cap(head, kRowsPerUnembed)));
  EVIE_TRY(b.get(&lg, (size_t)n * am.V));
  EVIE_CUDA_TRY(cudaMemcpyAsync(dbases, bases.data(), n * sizeof(void*), cudaMemcpyHostToDevice, st));
  EVIE_CUDA_TRY(cudaMemcpyAsync(dcols, cols.data(), n * sizeof(int), cudaMemcpyHostToDevice, st));
  gather_cols_kernel<<<dim3((d + 255) / 256, n), 256, 0, st>>>(dbases, dcols, d, am.n, dirs);
  EVIE_CHECK_LAUNCH("gather_cols_kernel");
  for (int g0 = 0; g0 < n;) {
    int g1 = g0;
    const int l = layers[order[g0]];
    while (g1 < n && layers[order[g1]] == l) g1++;
    if (const Planes16* J = am.lens ? am.lens->map(l) : nullptr) {  // transport this layer's rows in place
      const int nr = g1 - g0;
      YView T;
      EVIE_TRY(split(dense(dirs + (size_t)g0 * d, (size_t)nr * d), (size_t)nr * d, X2, st));
      EVIE_TRY(product(*J, X2, nr, yT, tcap, st, &T));
      sum_planes_kernel<<<grid_for((size_t)nr * d), 256, 0, st>>>(T, (size_t)nr * d, dirs + (size_t)g0 * d);
      EVIE_CHECK_LAUNCH("sum_planes_kernel");
    }
    g0 = g1;
  }
  EVIE_TRY(unembed(am, dense(dirs, (size_t)n * d), n, X2n, yL, product_cap(head, kRowsPerUnembed), lg));
  std::vector<float> host((size_t)n * am.V);
  EVIE_CUDA_TRY(cudaMemcpyAsync(host.data(), lg, host.size() * sizeof(float), cudaMemcpyDeviceToHost, st));
  EVIE_TRY(tg.end());
  for (int j = 0; j < n; j++)
    memcpy(logits + (size_t)order[j] * am.V, host.data() + (size_t)j * am.V, (size_t)am.V * sizeof(float));
  return EVIE_OK;
}

evie_status search_scores_run(const AnalysisModel& am, const uint32_t* tokens, int nt, const float* mean,
                              const float* sigma, float* z_up, float* z_dn) {
  const int d = am.d, n = am.n, L = (int)am.w_down.size();
  if (nt < 1) return fail(EVIE_ERR_ARG, "search: no tokens");
  for (int t = 0; t < nt; t++)
    if (tokens[t] >= (uint32_t)am.V) return fail(EVIE_ERR_ARG, "search: token %u out of range", tokens[t]);
  cudaStream_t st = am.st;
  TimeoutGuard tg{st};
  EVIE_TRY(tg.begin());
  DevBufs b;
  uint32_t* dt;
  float *dmean, *dsig, *a, *yP, *yS, *zu, *zd;
  __nv_bfloat16 *X2a, *X2p, *WT;
  const Planes16 Wd{nullptr, 1, n, d};
  size_t pcap = 1;
  if (am.lens)
    for (int l = 0; l < L; l++)
      if (const Planes16* J = am.lens->map_t(l)) pcap = std::max(pcap, product_cap(*J, nt));
  EVIE_TRY(b.get(&dt, nt));
  EVIE_TRY(b.get(&dmean, d));
  EVIE_TRY(b.get(&dsig, (size_t)L * n));
  EVIE_TRY(b.get(&a, (size_t)nt * d));
  EVIE_TRY(b.get(&X2a, (size_t)2 * nt * d));
  EVIE_TRY(b.get(&X2p, (size_t)2 * nt * d));
  EVIE_TRY(b.get(&yP, pcap));
  EVIE_TRY(b.get(&WT, (size_t)n * d));
  EVIE_TRY(b.get(&yS, product_cap(Wd, nt)));
  EVIE_TRY(b.get(&zu, (size_t)L * n));
  EVIE_TRY(b.get(&zd, (size_t)L * n));
  EVIE_CUDA_TRY(cudaMemcpyAsync(dt, tokens, nt * sizeof(uint32_t), cudaMemcpyHostToDevice, st));
  EVIE_CUDA_TRY(cudaMemcpyAsync(dmean, mean, d * sizeof(float), cudaMemcpyHostToDevice, st));
  EVIE_CUDA_TRY(cudaMemcpyAsync(dsig, sigma, (size_t)L * n * sizeof(float), cudaMemcpyHostToDevice, st));
  centered_rows_kernel<<<dim3((d + 255) / 256, nt), 256, 0, st>>>(am.lm_head, dt, d, dmean, am.final_norm, a);
  EVIE_CHECK_LAUNCH("centered_rows_kernel");
  EVIE_TRY(split(dense(a, (size_t)nt * d), (size_t)nt * d, X2a, st));
  for (int l = 0; l < L; l++) {
    const __nv_bfloat16* X2 = X2a;
    if (const Planes16* JT = am.lens ? am.lens->map_t(l) : nullptr) {  // lens.rs:76-82 (pullback J_l^T a)
      YView P;
      EVIE_TRY(product(*JT, X2a, nt, yP, pcap, st, &P));
      EVIE_TRY(split(P, (size_t)nt * d, X2p, st));
      X2 = X2p;
    }
    // scores[t][i] = sum_k W_down[k][i] pulled[t][k]  (analysis.rs:228: matvec_t(W_down, pulled))
    EVIE_TRY(transpose(am.w_down[l], d, n, WT, st));
    YView S;
    EVIE_TRY(product(Planes16{WT, 1, n, d}, X2, nt, yS, product_cap(Wd, nt), st, &S));
    zscore_kernel<<<(n + 255) / 256, 256, 0, st>>>(S, nt, n, dsig + (size_t)l * n, zu + (size_t)l * n,
                                                   zd + (size_t)l * n);
    EVIE_CHECK_LAUNCH("zscore_kernel");
  }
  EVIE_CUDA_TRY(cudaMemcpyAsync(z_up, zu, (size_t)L * n * sizeof(float), cudaMemcpyDeviceToHost, st));
  EVIE_CUDA_TRY(cudaMemcpyAsync(z_dn, zd, (size_t)L * n * sizeof(float), cudaMemcpyDeviceToHost, st));
  return tg.end();
}

}  // namespace evie
