// Device sampler: evie-core's Sampler::sample (crates/evie-core/src/sampling.rs:41-93), one CTA per sequence.
//
// Order of operations, as the reference:
//   1. repetition penalty on every distinct history token (sampling.rs:44-58): l / p when l > 0, else l * p;
//   2. temperature <= 0: the first index of the largest adjusted logit (topk(logits, 1), sampling.rs:60-62);
//   3. otherwise the 512 largest adjusted logits, by value and then lower index (kernels.rs:642-662), found by a
//      3-pass radix select on order-preserving keys, then sorted (bitonic) into the reference's order;
//   4. p_j = exp((l_j - l_0) / T), each divided by their sum; min-p keeps p_j >= p_0 * min_p; top-p keeps the
//      shortest prefix whose running sum reaches top_p (at least one); one splitmix64 uniform u; the first j at
//      which u * sum - p_0 - ... - p_j <= 0 is the token (sampling.rs:63-92).
// Every f32 step rounds as the reference's scalar code does (the sums are sequential, left to right). exp is
// evaluated in double and rounded once to f32, so it returns the correctly rounded f32 exponential (save for
// arguments within ~1e-9 relative of a rounding boundary), as the host libm's expf does.
#include "sampler.h"

#include <cuda_runtime.h>

#include <vector>

namespace evie {

namespace {

constexpr int kThreads = 1024;
constexpr int kCand = 512;  // sampling.rs:64
constexpr int kBins = 2048;
constexpr int kFixedSmem = kCand * 8 + kCand * 4 + kBins * 4 + 32 * 4 + 32 * 8 + 8 * 4;

// Order-preserving key of an f32: a larger value gives a larger key; -0 and +0 share one key (they compare equal
// in the reference's ordering).
__device__ __forceinline__ uint32_t ord_key(float v) {
  const uint32_t u = __float_as_uint(v == 0.0f ? 0.0f : v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_value(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}
// Candidate = key in the high word, inverted index in the low word: the larger candidate is the larger value,
// then the lower index.
__device__ __forceinline__ unsigned long long cand_of(uint32_t key, uint32_t i) {
  return ((unsigned long long)key << 32) | (0xFFFFFFFFu - i);
}
__device__ __forceinline__ uint32_t cand_index(unsigned long long c) { return 0xFFFFFFFFu - (uint32_t)c; }

// Inclusive prefix sum over the 1024 threads of the block; red holds 32 ints.
__device__ int block_scan_incl(int v, int* red) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += t;
  }
  if (lane == 31) red[w] = v;
  __syncthreads();
  if (w == 0) {
    int t = red[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, t, o);
      if (lane >= o) t += u;
    }
    red[lane] = t;
  }
  __syncthreads();
  const int r = v + (w > 0 ? red[w - 1] : 0);
  __syncthreads();
  return r;
}

__device__ unsigned long long block_max_u64(unsigned long long v, unsigned long long* red) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const unsigned long long t = __shfl_xor_sync(0xffffffffu, v, o);
    v = t > v ? t : v;
  }
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    v = red[threadIdx.x];
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
      const unsigned long long t = __shfl_xor_sync(0xffffffffu, v, o);
      v = t > v ? t : v;
    }
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  v = red[0];
  __syncthreads();
  return v;
}

// sampling.rs:31-39: splitmix64 step, top 24 bits as a uniform in [0, 1).
__device__ __forceinline__ float splitmix_uniform(uint64_t* state) {
  const uint64_t s = *state + 0x9E3779B97F4A7C15ull;
  *state = s;
  uint64_t z = s;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  z ^= z >> 31;
  return __fdiv_rn((float)(z >> 40), 16777216.0f);
}

__global__ void __launch_bounds__(kThreads, 1) sample_kernel(SampleArgs a) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ __align__(16) unsigned char smem[];
  unsigned long long* cand = reinterpret_cast<unsigned long long*>(smem);  // [kCand]
  float* prob = reinterpret_cast<float*>(cand + kCand);                   // [kCand]
  int* hist = reinterpret_cast<int*>(prob + kCand);                       // [kBins]
  int* red = hist + kBins;                                                // [32]
  unsigned long long* redl = reinterpret_cast<unsigned long long*>(red + 32);  // [32]
  int* misc = reinterpret_cast<int*>(redl + 32);                          // [8]
  uint32_t* bm = reinterpret_cast<uint32_t*>(misc + 8);                   // [ceil(V / 32)] history bitmap

  const int s = blockIdx.x;
  const int slot = a.segs ? a.segs[s].slot : s;
  const SamplerParams p = a.params[slot];
  const int V = a.V;
  const int W = (V + 31) >> 5;
  const size_t base = (size_t)s * V;
  const float rep = p.repetition_penalty;
  bool pen = rep != 1.0f;
  if (pen) {  // sampling.rs:43-58 (the model's per-slot bitmap is never empty once the slot has been fed)
    if (a.seen) {
      const uint32_t* src = a.seen + (size_t)slot * a.seen_words;
      for (int j = threadIdx.x; j < W; j += kThreads) bm[j] = src[j];
    } else {
      const long long h0 = a.hist_off[s], h1 = a.hist_off[s + 1];
      pen = h1 > h0;
      for (int j = threadIdx.x; j < W; j += kThreads) bm[j] = 0u;
      __syncthreads();
      for (long long j = h0 + threadIdx.x; j < h1; j += kThreads) {
        const uint32_t t = a.hist[j];
        if (t < (uint32_t)V) atomicOr(&bm[t >> 5], 1u << (t & 31));
      }
    }
    __syncthreads();
  }
  auto key_at = [&](int i) -> uint32_t {
    float v = a.logits.at(base + i);
    if (pen && ((bm[i >> 5] >> (i & 31)) & 1u)) v = v > 0.0f ? __fdiv_rn(v, rep) : __fmul_rn(v, rep);
    return ord_key(v);
  };

  if (p.temperature <= 0.0f) {  // sampling.rs:60-62
    unsigned long long best = 0;
    for (int i = threadIdx.x; i < V; i += kThreads) {
      const unsigned long long c = cand_of(key_at(i), (uint32_t)i);
      best = c > best ? c : best;
    }
    best = block_max_u64(best, redl);
    if (threadIdx.x == 0) a.next[s] = cand_index(best);
    return;
  }

  // sampling.rs:64 / kernels.rs:642-662: the k largest keys. Radix select: 11 + 11 + 10 bits, most significant
  // first; after the passes kstar is the k-th largest key, krem of the keys equal to it belong to the top k.
  const int k = V < kCand ? V : kCand;
  uint32_t prefix = 0, pmask = 0;
  int krem = k, tot = V, neq = 0;
  for (int pass = 0; pass < 3; pass++) {
    const int sh = pass == 0 ? 21 : (pass == 1 ? 10 : 0);
    const uint32_t dm = pass == 2 ? 0x3FFu : 0x7FFu;
    for (int b = threadIdx.x; b < kBins; b += kThreads) hist[b] = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < V; i += kThreads) {
      const uint32_t key = key_at(i);
      if ((key & pmask) == prefix) atomicAdd(&hist[(key >> sh) & dm], 1);
    }
    __syncthreads();
    // thread t owns bins 2t, 2t+1; keys above a bin = keys of this prefix with a larger digit
    const int b0 = 2 * threadIdx.x, b1 = b0 + 1;
    const int h0 = hist[b0], h1 = hist[b1];
    const int incl = block_scan_incl(h0 + h1, red);
    const int above1 = tot - incl, above0 = above1 + h1;
    if (above1 < krem && krem <= above1 + h1) misc[0] = b1, misc[1] = krem - above1, misc[2] = h1;
    if (above0 < krem && krem <= above0 + h0) misc[0] = b0, misc[1] = krem - above0, misc[2] = h0;
    __syncthreads();
    prefix |= (uint32_t)misc[0] << sh;
    pmask |= dm << sh;
    krem = misc[1];
    neq = misc[2];
    tot = neq;
    __syncthreads();
  }
  const uint32_t kstar = prefix;
  const bool all_eq = neq == krem;
  if (threadIdx.x == 0) misc[3] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < V; i += kThreads) {
    const uint32_t key = key_at(i);
    if (key > kstar || (all_eq && key == kstar)) {
      const int pos = atomicAdd(&misc[3], 1);
      if (pos < kCand) cand[pos] = cand_of(key, (uint32_t)i);
    }
  }
  __syncthreads();
  if (!all_eq) {  // ties across the cut: the lowest indices among the keys equal to kstar, in index order
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int first = k - krem;
    int taken = 0;
    for (int t0 = 0; t0 < V && taken < krem; t0 += kThreads) {
      const int i = t0 + threadIdx.x;
      const bool eq = i < V && key_at(i) == kstar;
      const unsigned bal = __ballot_sync(0xffffffffu, eq);
      if (lane == 0) red[w] = __popc(bal);
      __syncthreads();
      int before = 0, tile = 0;
      for (int q = 0; q < 32; q++) {
        const int c = red[q];
        before += q < w ? c : 0;
        tile += c;
      }
      const int rank = taken + before + __popc(bal & ((1u << lane) - 1u));
      if (eq && rank < krem) cand[first + rank] = cand_of(kstar, (uint32_t)i);
      taken += tile;
      __syncthreads();
    }
  }
  for (int j = k + threadIdx.x; j < kCand; j += kThreads) cand[j] = 0ull;
  // bitonic sort, descending
  for (int size = 2; size <= kCand; size <<= 1)
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      __syncthreads();
      const int i = threadIdx.x;
      if (i < kCand) {
        const int j = i ^ stride;
        if (j > i) {
          const bool desc = (i & size) == 0;
          const unsigned long long x = cand[i], y = cand[j];
          if ((x < y) == desc) cand[i] = y, cand[j] = x;
        }
      }
    }
  __syncthreads();

  // sampling.rs:65-68
  const float T = p.temperature;
  const float top = key_value((uint32_t)(cand[0] >> 32));
  if (threadIdx.x < k) {
    const float v = key_value((uint32_t)(cand[threadIdx.x] >> 32));
    prob[threadIdx.x] = (float)exp((double)__fdiv_rn(__fsub_rn(v, top), T));
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float total = 0.0f;
    for (int j = 0; j < k; j++) total = __fadd_rn(total, prob[j]);
    reinterpret_cast<float*>(misc)[4] = total;
  }
  __syncthreads();
  const float total = reinterpret_cast<float*>(misc)[4];
  if (threadIdx.x < k) prob[threadIdx.x] = __fdiv_rn(prob[threadIdx.x], total);
  __syncthreads();
  if (threadIdx.x == 0) {  // sampling.rs:69-92, sequential as the reference
    const uint32_t top_tok = cand_index(cand[0]);
    int m = k;
    if (p.min_p > 0.0f) {
      const float floor = __fmul_rn(prob[0], p.min_p);
      int w = 0;
      for (int j = 0; j < m; j++)
        if (prob[j] >= floor) prob[w] = prob[j], cand[w] = cand[j], w++;
      m = w;
    }
    if (p.top_p < 1.0f) {
      float acc = 0.0f;
      int keep = 0;
      for (int j = 0; j < m; j++) {
        acc = __fadd_rn(acc, prob[j]);
        keep++;
        if (acc >= p.top_p) break;
      }
      m = min(m, max(keep, 1));
    }
    float total2 = 0.0f;
    for (int j = 0; j < m; j++) total2 = __fadd_rn(total2, prob[j]);
    float r = __fmul_rn(splitmix_uniform(a.rng + slot), total2);
    uint32_t tok = m > 0 ? cand_index(cand[m - 1]) : top_tok;
    for (int j = 0; j < m; j++) {
      r = __fsub_rn(r, prob[j]);
      if (r <= 0.0f) {
        tok = cand_index(cand[j]);
        break;
      }
    }
    a.next[s] = tok;
  }
}

}  // namespace

evie_status k_sample(const SampleArgs& a, int nseq, cudaStream_t st) {
  if (nseq == 0) return EVIE_OK;
  const size_t smem = kFixedSmem + (size_t)((a.V + 31) / 32) * 4;
  if (smem > 48 * 1024) {
    const cudaError_t e =
        cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return fail(EVIE_ERR_CUDA, "sampler: %s", cudaGetErrorString(e));
  }
  EVIE_CUDA_TRY(launch_k(sample_kernel, dim3(nseq), dim3(kThreads), smem, st, a));
  EVIE_CHECK_LAUNCH("sample_kernel");
  return EVIE_OK;
}

}  // namespace evie

extern "C" {

uint64_t evie_sampler_seed_state(uint64_t seed) { return evie::sampler_seed_state(seed); }

evie_status evie_sample(const float* logits, int B, int V, const evie_sample_params* params, uint64_t* rng,
                        const uint32_t* history, const int64_t* hist_off, uint32_t* out, void* stream) {
  using evie::fail;
  if (B < 1 || V < 1 || V > (1 << 20)) return fail(EVIE_ERR_ARG, "evie_sample: B >= 1 and 1 <= V <= 1048576");
  if (!logits || !params || !rng || !hist_off || !out) return fail(EVIE_ERR_ARG, "evie_sample: null argument");
  if (hist_off[0] < 0) return fail(EVIE_ERR_ARG, "evie_sample: negative history offset");
  for (int b = 0; b < B; b++)
    if (hist_off[b + 1] < hist_off[b]) return fail(EVIE_ERR_ARG, "evie_sample: history offsets decrease at %d", b);
  if (hist_off[B] > hist_off[0] && !history) return fail(EVIE_ERR_ARG, "evie_sample: null history");
  cudaStream_t st = (cudaStream_t)stream;
  std::vector<evie::SamplerParams> sp(B);
  for (int b = 0; b < B; b++)
    sp[b] = evie::SamplerParams{params[b].temperature, params[b].top_p, params[b].min_p, params[b].repetition_penalty};
  const size_t o_rng = (size_t)B * sizeof(evie::SamplerParams), o_off = o_rng + (size_t)B * 8,
               o_next = o_off + (size_t)(B + 1) * 8, bytes = o_next + (size_t)B * 4;
  char* dev = nullptr;
  cudaError_t e = cudaMallocAsync((void**)&dev, bytes, st);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(EVIE_ERR_OOM, "evie_sample: %s", cudaGetErrorString(e));
  }
  evie_status rc = EVIE_OK;
  do {
    if ((e = cudaMemcpyAsync(dev, sp.data(), o_rng, cudaMemcpyHostToDevice, st)) != cudaSuccess) break;
    if ((e = cudaMemcpyAsync(dev + o_rng, rng, (size_t)B * 8, cudaMemcpyHostToDevice, st)) != cudaSuccess) break;
    if ((e = cudaMemcpyAsync(dev + o_off, hist_off, (size_t)(B + 1) * 8, cudaMemcpyHostToDevice, st)) != cudaSuccess)
      break;
    const evie::SampleArgs a{evie::YView{logits, 0, 1}, V, nullptr,
                             reinterpret_cast<const evie::SamplerParams*>(dev), reinterpret_cast<uint64_t*>(dev + o_rng),
                             nullptr, 0, history, reinterpret_cast<const long long*>(dev + o_off),
                             reinterpret_cast<uint32_t*>(dev + o_next)};
    if ((rc = evie::k_sample(a, B, st)) != EVIE_OK) break;
    if ((e = cudaMemcpyAsync(out, dev + o_next, (size_t)B * 4, cudaMemcpyDeviceToHost, st)) != cudaSuccess) break;
    if ((e = cudaMemcpyAsync(rng, dev + o_rng, (size_t)B * 8, cudaMemcpyDeviceToHost, st)) != cudaSuccess) break;
  } while (0);
  cudaFreeAsync(dev, st);
  const cudaError_t se = cudaStreamSynchronize(st);
  if (rc != EVIE_OK) return rc;
  if (e == cudaSuccess) e = se;
  if (e != cudaSuccess) return fail(EVIE_ERR_CUDA, "evie_sample: %s", cudaGetErrorString(e));
  return EVIE_OK;
}

}  // extern "C"
