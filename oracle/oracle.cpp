// CPU oracle for the evie-b200 test-suite and the CPU baseline leg of bench.py.
//
// TEST INFRASTRUCTURE ONLY. This is a C++ restatement of evie-core's CPU engine (Rust, which cannot be
// built in this environment: no cargo/rustc, crates not vendored). Nothing in the product library links
// or calls it; only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load it, as the checker.
//
// It follows, function by function (paths relative to the evie repository):
//   crates/evie-core/src/kernels.rs:107-117   bf16 widening
//   crates/evie-core/src/kernels.rs:138-268   matvec / matmul dispatch (n==1 dot_rows, n<8 multi_dot, else packed GEMM)
//   crates/evie-core/src/kernels.rs:270-522   AVX2/FMA micro-kernels (load8, hsum, dot_rows, multi_dot, pack_panel, micro)
//   crates/evie-core/src/kernels.rs:573-662   silu, sigmoid, softplus(thr 20), dot (8 lanes), rmsnorm, softmax, topk
//   crates/evie-core/src/model.rs:217-284     Model::forward (segments batched for projections, hooks)
//   crates/evie-core/src/model.rs:296-396     Model::deltanet (conv+SiLU, L2 norm, decay/beta, recurrence, gated norm)
//   crates/evie-core/src/model.rs:398-479     Model::attention + rope
//   crates/evie-core/src/model.rs:501-524     recur_body (loop order kept)
//   crates/evie-core/src/steering.rs:150-210  Plan::begin / Plan::apply (add / mul / set, latching gates)
//   crates/evie-core/src/sampling.rs:21-93    Sampler (splitmix64) and Sampler::sample
//   crates/evie/src/mcp.rs:242-256            top_active (ties: lower flat index first)
//   crates/evie/src/worker.rs:97-121          Capture (sqrt-companded i8 frames, f16 residual)
//   crates/evie-core/src/gpu/mod.rs:577-593   track_max semantics (max |a| over positions > 0)
//
// Floating point: build with -ffp-contract=off so that scalar `a += b * c` stays a rounded multiply followed
// by a rounded add, as Rust compiles it; the AVX2 paths use explicit _mm256_fmadd_ps exactly where the
// reference does. Transcendentals come from the same libm (expf, log1pf, sinf, cosf, powf, sqrtf).

#include <immintrin.h>
#include <stdint.h>
#include <string.h>
#include <math.h>
#include <stdlib.h>
#include <algorithm>
#include <atomic>
#include <condition_variable>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

#define EXPORT extern "C" __attribute__((visibility("default")))

// ------------------------------------------------------------------------------------------------
// thread pool (stands in for rayon's global pool; results never depend on the thread count because
// every output element is produced by exactly one task in a fixed order)

namespace {

class Pool {
 public:
  explicit Pool(int n) { resize(n); }
  ~Pool() { stop_all(); }
  int size() const { return (int)workers_.size() + 1; }
  void resize(int n) {
    stop_all();
    if (n < 1) n = 1;
    quit_ = false;
    for (int i = 0; i < n - 1; i++) workers_.emplace_back([this] { loop(); });
  }
  // Runs f(i) for i in [0, n) over all threads, dynamic chunking.
  void run(long n, const std::function<void(long)>& f) {
    if (n <= 0) return;
    if (workers_.empty() || n == 1) {
      for (long i = 0; i < n; i++) f(i);
      return;
    }
    std::unique_lock<std::mutex> lk(m_);
    job_ = &f;
    total_ = n;
    next_.store(0);
    pending_ = (int)workers_.size();
    gen_++;
    lk.unlock();
    cv_.notify_all();
    work();
    lk.lock();
    done_cv_.wait(lk, [this] { return pending_ == 0; });
    job_ = nullptr;
  }

 private:
  void work() {
    for (;;) {
      long i = next_.fetch_add(1);
      if (i >= total_) break;
      (*job_)(i);
    }
  }
  void loop() {
    long seen = 0;
    for (;;) {
      std::unique_lock<std::mutex> lk(m_);
      cv_.wait(lk, [&] { return quit_ || gen_ != seen; });
      if (quit_) return;
      seen = gen_;
      lk.unlock();
      work();
      lk.lock();
      if (--pending_ == 0) done_cv_.notify_all();
    }
  }
  void stop_all() {
    {
      std::lock_guard<std::mutex> lk(m_);
      quit_ = true;
    }
    cv_.notify_all();
    for (auto& t : workers_) t.join();
    workers_.clear();
  }
  std::vector<std::thread> workers_;
  std::mutex m_;
  std::condition_variable cv_, done_cv_;
  const std::function<void(long)>* job_ = nullptr;
  long total_ = 0;
  std::atomic<long> next_{0};
  int pending_ = 0;
  long gen_ = 0;
  bool quit_ = false;
};

Pool& pool() {
  static Pool p(1);
  return p;
}

inline void par_for(long n, const std::function<void(long)>& f) { pool().run(n, f); }

// ------------------------------------------------------------------------------------------------
// scalar helpers (kernels.rs:106-117, 572-662)

inline float bf16_to_f32(uint16_t x) {
  uint32_t u = (uint32_t)x << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}
inline float silu(float x) { return x / (1.0f + expf(-x)); }
inline float sigmoid(float x) { return 1.0f / (1.0f + expf(-x)); }
inline float softplus(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

// kernels.rs:589-603: eight lane accumulators, summed left to right, then the scalar remainder.
inline float dot(const float* a, const float* b, size_t n) {
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  size_t full = n / 8 * 8;
  for (size_t c = 0; c < full; c += 8)
    for (int i = 0; i < 8; i++) acc[i] += a[c + i] * b[c + i];
  float s = -0.0f;
  for (int i = 0; i < 8; i++) s += acc[i];
  for (size_t i = full; i < n; i++) s += a[i] * b[i];
  return s;
}

// kernels.rs:607-613
inline void rmsnorm(const float* x, const float* w, float eps, float* out, size_t n) {
  float ms = dot(x, x, n) / (float)n;
  float inv = 1.0f / sqrtf(ms + eps);
  for (size_t i = 0; i < n; i++) out[i] = x[i] * inv * w[i];
}

void rmsnorm_rows(const float* x, const float* w, float eps, float* out, size_t d, long rows) {
  par_for(rows, [&](long r) { rmsnorm(x + r * d, w, eps, out + r * d, d); });
}

void add_inplace(float* x, const float* y, size_t n) {
  long chunks = (long)((n + (1 << 14) - 1) >> 14);
  par_for(chunks, [&](long c) {
    size_t a = (size_t)c << 14, b = std::min(n, a + (1 << 14));
    for (size_t i = a; i < b; i++) x[i] += y[i];
  });
}

// kernels.rs:628-639
void softmax_inplace(float* x, size_t n) {
  float m = -INFINITY;
  for (size_t i = 0; i < n; i++) m = fmaxf(m, x[i]);
  float s = 0.0f;
  for (size_t i = 0; i < n; i++) {
    x[i] = expf(x[i] - m);
    s += x[i];
  }
  float inv = 1.0f / s;
  for (size_t i = 0; i < n; i++) x[i] *= inv;
}

// kernels.rs:642-662: strict `>` against the floor, insertion after every entry >= v, so on ties the
// lower index ranks first.
int topk(const float* v, size_t n, int k, uint32_t* idx, float* val) {
  if ((size_t)k > n) k = (int)n;
  if (k <= 0) return 0;
  std::vector<std::pair<uint32_t, float>> best;
  best.reserve(k + 1);
  float floor = -INFINITY;
  for (size_t i = 0; i < n; i++) {
    float x = v[i];
    if ((int)best.size() < k || x > floor) {
      size_t pos = 0;
      {
        size_t lo = 0, hi = best.size();
        while (lo < hi) {  // partition_point(|b| b >= x)
          size_t mid = (lo + hi) / 2;
          if (best[mid].second >= x) lo = mid + 1; else hi = mid;
        }
        pos = lo;
      }
      best.insert(best.begin() + pos, {(uint32_t)i, x});
      if ((int)best.size() > k) best.pop_back();
      if ((int)best.size() == k) floor = best[k - 1].second;
    }
  }
  for (size_t i = 0; i < best.size(); i++) {
    idx[i] = best[i].first;
    if (val) val[i] = best[i].second;
  }
  return (int)best.size();
}

// sampling.rs:21-93: Sampler (splitmix64 uniforms) and Sampler::sample.
struct Sampler {
  float temperature, top_p, min_p, repetition_penalty;
  uint64_t rng;
};

// sampling.rs:27-29
Sampler sampler_new(float t, float top_p, float min_p, float rep, uint64_t seed) {
  return Sampler{t, top_p, min_p, rep, (seed * 0x9E3779B97F4A7C15ull) ^ 0xD1B54A32D192ED03ull};
}

// sampling.rs:31-39
float sampler_uniform(Sampler& s) {
  s.rng += 0x9E3779B97F4A7C15ull;
  uint64_t z = s.rng;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  z ^= z >> 31;
  return (float)(z >> 40) / (float)(1ull << 24);
}

// sampling.rs:41-93
uint32_t sampler_sample(Sampler& s, const float* logits_in, size_t n, const uint32_t* history, size_t nh) {
  std::vector<float> adjusted;
  const float* logits = logits_in;
  if (s.repetition_penalty != 1.0f && nh > 0) {
    adjusted.assign(logits_in, logits_in + n);
    std::vector<uint32_t> seen(history, history + nh);
    std::sort(seen.begin(), seen.end());
    seen.erase(std::unique(seen.begin(), seen.end()), seen.end());
    for (uint32_t t : seen)
      if (t < n) {
        float& v = adjusted[t];
        v = v > 0.0f ? v / s.repetition_penalty : v * s.repetition_penalty;
      }
    logits = adjusted.data();
  }
  if (s.temperature <= 0.0f) {
    uint32_t i = 0;
    topk(logits, n, 1, &i, nullptr);
    return i;
  }
  std::vector<uint32_t> ci(512);
  std::vector<float> cv(512);
  const int k = topk(logits, n, 512, ci.data(), cv.data());
  const float top = cv[0];
  std::vector<std::pair<uint32_t, float>> probs(k);
  for (int j = 0; j < k; j++) probs[j] = {ci[j], expf((cv[j] - top) / s.temperature)};
  float total = 0.0f;
  for (auto& x : probs) total += x.second;
  for (auto& x : probs) x.second /= total;
  if (s.min_p > 0.0f) {
    const float floor = probs[0].second * s.min_p;
    std::vector<std::pair<uint32_t, float>> kept;
    for (auto& x : probs)
      if (x.second >= floor) kept.push_back(x);
    probs.swap(kept);
  }
  if (s.top_p < 1.0f) {
    float acc = 0.0f;
    size_t keep = 0;
    for (auto& x : probs) {
      acc += x.second;
      keep++;
      if (acc >= s.top_p) break;
    }
    if (probs.size() > std::max<size_t>(keep, 1)) probs.resize(std::max<size_t>(keep, 1));
  }
  float total2 = 0.0f;
  for (auto& x : probs) total2 += x.second;
  float r = sampler_uniform(s) * total2;
  for (auto& x : probs) {
    r -= x.second;
    if (r <= 0.0f) return x.first;
  }
  return probs.empty() ? ci[0] : probs.back().first;
}

// ------------------------------------------------------------------------------------------------
// AVX2 matmul (kernels.rs:138-268, 270-522). Weights are bf16 bits (uint16_t) or f32 widenings of 16-bit values
// (float: the f16 matrices of a lens, widened once; widening is exact, so the products and orders are the reference's).

constexpr size_t KC = 256;
constexpr size_t NR = 16;

__attribute__((target("avx2,fma,f16c"))) inline __m256 load8(const uint16_t* p) {
  __m128i v = _mm_loadu_si128((const __m128i*)p);
  return _mm256_castsi256_ps(_mm256_slli_epi32(_mm256_cvtepu16_epi32(v), 16));
}

__attribute__((target("avx2,fma"))) inline __m256 load8(const float* p) { return _mm256_loadu_ps(p); }
inline float widen(uint16_t x);
inline float widen(float x) { return x; }

__attribute__((target("avx2,fma"))) inline float hsum(__m256 v) {
  __m128 lo = _mm256_castps256_ps128(v);
  __m128 hi = _mm256_extractf128_ps(v, 1);
  __m128 s = _mm_add_ps(lo, hi);
  s = _mm_add_ps(s, _mm_movehl_ps(s, s));
  s = _mm_add_ss(s, _mm_shuffle_ps(s, s, 0x55));
  return _mm_cvtss_f32(s);
}

// kernels.rs:303-362
template <typename WT>
__attribute__((target("avx2,fma,f16c"))) void dot_rows(const WT* w, size_t cols, size_t r0,
                                                         const float* x, float* ys, size_t n) {
  size_t i = 0;
  while (i + 4 <= n) {
    const WT* p0 = w + (r0 + i) * cols;
    const WT *p1 = p0 + cols, *p2 = p0 + 2 * cols, *p3 = p0 + 3 * cols;
    __m256 z = _mm256_setzero_ps();
    __m256 a0 = z, a1 = z, a2 = z, a3 = z, b0 = z, b1 = z, b2 = z, b3 = z;
    size_t k = 0;
    while (k + 16 <= cols) {
      __m256 x0 = _mm256_loadu_ps(x + k), x1 = _mm256_loadu_ps(x + k + 8);
      a0 = _mm256_fmadd_ps(load8(p0 + k), x0, a0);
      b0 = _mm256_fmadd_ps(load8(p0 + k + 8), x1, b0);
      a1 = _mm256_fmadd_ps(load8(p1 + k), x0, a1);
      b1 = _mm256_fmadd_ps(load8(p1 + k + 8), x1, b1);
      a2 = _mm256_fmadd_ps(load8(p2 + k), x0, a2);
      b2 = _mm256_fmadd_ps(load8(p2 + k + 8), x1, b2);
      a3 = _mm256_fmadd_ps(load8(p3 + k), x0, a3);
      b3 = _mm256_fmadd_ps(load8(p3 + k + 8), x1, b3);
      k += 16;
    }
    float s[4] = {hsum(_mm256_add_ps(a0, b0)), hsum(_mm256_add_ps(a1, b1)), hsum(_mm256_add_ps(a2, b2)),
                  hsum(_mm256_add_ps(a3, b3))};
    while (k < cols) {
      float xv = x[k];
      s[0] += widen(p0[k]) * xv;
      s[1] += widen(p1[k]) * xv;
      s[2] += widen(p2[k]) * xv;
      s[3] += widen(p3[k]) * xv;
      k++;
    }
    memcpy(ys + i, s, sizeof s);
    i += 4;
  }
  while (i < n) {
    const WT* p = w + (r0 + i) * cols;
    __m256 a = _mm256_setzero_ps();
    size_t k = 0;
    while (k + 8 <= cols) {
      a = _mm256_fmadd_ps(load8(p + k), _mm256_loadu_ps(x + k), a);
      k += 8;
    }
    float s = hsum(a);
    while (k < cols) {
      s += widen(p[k]) * x[k];
      k++;
    }
    ys[i] = s;
    i++;
  }
}

// kernels.rs:365-396
template <int T, typename WT>
__attribute__((target("avx2,fma,f16c"))) void multi_dot(const WT* w, size_t cols, size_t r0, size_t nr,
                                                          const float* x, float* y, size_t ldy) {
  for (size_t r = r0; r < r0 + nr; r++) {
    const WT* p = w + r * cols;
    __m256 acc[T];
    for (int t = 0; t < T; t++) acc[t] = _mm256_setzero_ps();
    size_t k = 0;
    while (k + 8 <= cols) {
      __m256 wv = load8(p + k);
      for (int t = 0; t < T; t++) acc[t] = _mm256_fmadd_ps(wv, _mm256_loadu_ps(x + t * cols + k), acc[t]);
      k += 8;
    }
    for (int t = 0; t < T; t++) {
      float s = hsum(acc[t]);
      for (size_t kk = k; kk < cols; kk++) s += widen(p[kk]) * x[t * cols + kk];
      y[t * ldy + r] = s;
    }
  }
}

// kernels.rs:427-464 (the packed values are exact f32 widenings; the 8x8 transpose only moves them). The float
// form packs a matrix already widened from f16 (Kind16::F16), which the same micro-kernel then multiplies.
inline float widen(uint16_t x) { return bf16_to_f32(x); }
template <typename WT>
__attribute__((target("avx2,fma,f16c"))) void pack_panel(const WT* w, size_t cols, size_t rows, size_t r0,
                                                           size_t k0, size_t kc, float* pack) {
  size_t nr = std::min(NR, rows - r0);
  for (size_t k = 0; k < kc; k++)
    for (size_t i = 0; i < NR; i++) pack[k * NR + i] = i < nr ? widen(w[(r0 + i) * cols + k0 + k]) : 0.0f;
}

// kernels.rs:466-521
template <int M>
__attribute__((target("avx2,fma"))) void micro(const float* pack, size_t kc, const float* x, size_t ldx, float* y,
                                               size_t ldy, size_t nr, bool accumulate) {
  __m256 acc[M][2];
  for (int i = 0; i < M; i++) acc[i][0] = acc[i][1] = _mm256_setzero_ps();
  if (accumulate) {
    for (int i = 0; i < M; i++) {
      const float* yr = y + i * ldy;
      float tmp[NR] = {0};
      for (size_t j = 0; j < nr; j++) tmp[j] = yr[j];
      acc[i][0] = _mm256_loadu_ps(tmp);
      acc[i][1] = _mm256_loadu_ps(tmp + 8);
    }
  }
  for (size_t k = 0; k < kc; k++) {
    __m256 w0 = _mm256_loadu_ps(pack + k * NR), w1 = _mm256_loadu_ps(pack + k * NR + 8);
    for (int i = 0; i < M; i++) {
      __m256 xb = _mm256_broadcast_ss(x + i * ldx + k);
      acc[i][0] = _mm256_fmadd_ps(xb, w0, acc[i][0]);
      acc[i][1] = _mm256_fmadd_ps(xb, w1, acc[i][1]);
    }
  }
  for (int i = 0; i < M; i++) {
    float tmp[NR];
    _mm256_storeu_ps(tmp, acc[i][0]);
    _mm256_storeu_ps(tmp + 8, acc[i][1]);
    float* yr = y + i * ldy;
    for (size_t j = 0; j < nr; j++) yr[j] = tmp[j];
  }
}

int n_threads() { return pool().size(); }

// kernels.rs:138-143
template <typename WT>
void matvec(const WT* w, size_t rows, size_t cols, const float* x, float* y) {
  long chunk = (long)std::min<size_t>(512, std::max<size_t>(4, rows / (n_threads() * 6))) & ~3L;
  if (chunk < 4) chunk = 4;
  long nch = (long)((rows + chunk - 1) / chunk);
  par_for(nch, [&](long ci) {
    size_t r0 = ci * chunk, n = std::min<size_t>(chunk, rows - r0);
    dot_rows(w, cols, r0, x, y + r0, n);
  });
}

// kernels.rs:221-268: the packed GEMM for n >= 8 rows of x
template <typename WT>
void packed_gemm(const WT* w, size_t rows, size_t cols, const float* x, size_t n, float* y) {
  size_t panels = (rows + NR - 1) / NR;
  size_t tb_size = std::min<size_t>((std::max<size_t>((2u << 20) / (cols * 4), 6) / 6) * 6, 480);
  for (size_t tb0 = 0; tb0 < n; tb0 += tb_size) {
    size_t tb = std::min(tb_size, n - tb0);
    par_for((long)panels, [&](long p) {
      thread_local std::vector<float> pack;
      pack.resize(KC * NR);
      size_t r0 = p * NR, nr = std::min(NR, rows - r0);
      for (size_t k0 = 0; k0 < cols; k0 += KC) {
        size_t kc = std::min(KC, cols - k0);
        pack_panel(w, cols, rows, r0, k0, kc, pack.data());
        for (size_t t = 0; t < tb;) {
          size_t m = std::min<size_t>(6, tb - t);
          const float* xr = x + (tb0 + t) * cols + k0;
          float* yr = y + (tb0 + t) * rows + r0;
          bool acc = k0 > 0;
          switch (m) {
            case 6: micro<6>(pack.data(), kc, xr, cols, yr, rows, nr, acc); break;
            case 5: micro<5>(pack.data(), kc, xr, cols, yr, rows, nr, acc); break;
            case 4: micro<4>(pack.data(), kc, xr, cols, yr, rows, nr, acc); break;
            case 3: micro<3>(pack.data(), kc, xr, cols, yr, rows, nr, acc); break;
            case 2: micro<2>(pack.data(), kc, xr, cols, yr, rows, nr, acc); break;
            default: micro<1>(pack.data(), kc, xr, cols, yr, rows, nr, acc); break;
          }
          t += m;
        }
      }
    });
  }
}

// kernels.rs:163-268
template <typename WT>
void matmul(const WT* w, size_t rows, size_t cols, const float* x, size_t n, float* y) {
  if (n == 0) return;
  if (n == 1) return matvec(w, rows, cols, x, y);
  if (n < 8) {
    size_t chunk = std::min<size_t>(512, std::max<size_t>(4, rows / (n_threads() * 6)));
    long nch = (long)((rows + chunk - 1) / chunk);
    par_for(nch, [&](long ci) {
      size_t r0 = ci * chunk, nr = std::min(chunk, rows - r0);
      switch (n) {
        case 2: multi_dot<2>(w, cols, r0, nr, x, y, rows); break;
        case 3: multi_dot<3>(w, cols, r0, nr, x, y, rows); break;
        case 4: multi_dot<4>(w, cols, r0, nr, x, y, rows); break;
        case 5: multi_dot<5>(w, cols, r0, nr, x, y, rows); break;
        case 6: multi_dot<6>(w, cols, r0, nr, x, y, rows); break;
        default: multi_dot<7>(w, cols, r0, nr, x, y, rows); break;
      }
    });
    return;
  }
  packed_gemm(w, rows, cols, x, n, y);
}

// ------------------------------------------------------------------------------------------------
// gated delta rule step (model.rs:501-524), loop order kept

inline void recur_body(float* s, const float* q, const float* k, const float* v, float decay, float beta, float* kv,
                       float* o, int dk, int dv) {
  for (int j = 0; j < dv; j++) kv[j] = 0.0f;
  for (int i = 0; i < dk; i++) {
    const float* row = s + (size_t)i * dv;
    float ki = k[i];
    for (int j = 0; j < dv; j++) kv[j] += row[j] * ki;
  }
  for (int j = 0; j < dv; j++) kv[j] = (v[j] - decay * kv[j]) * beta;
  for (int j = 0; j < dv; j++) o[j] = 0.0f;
  for (int i = 0; i < dk; i++) {
    float* row = s + (size_t)i * dv;
    float ki = k[i], qi = q[i];
    for (int j = 0; j < dv; j++) {
      row[j] = row[j] * decay + ki * kv[j];
      o[j] += row[j] * qi;
    }
  }
}

inline uint16_t f32_to_f16(float v) { return (uint16_t)_cvtss_sh(v, _MM_FROUND_TO_NEAREST_INT); }
inline float f16_to_f32(uint16_t h) { return _cvtsh_ss(h); }

// worker.rs:97-112 companding: q = round(127 * sqrt(min(|v|, 1))), sign of v.
inline int8_t compand(float v) {
  float q = roundf(sqrtf(fminf(fabsf(v), 1.0f)) * 127.0f);
  return v < 0.0f ? (int8_t)(-(int)q) : (int8_t)(int)q;
}

// ------------------------------------------------------------------------------------------------
// model

struct Mat {
  const uint16_t* p = nullptr;
  size_t rows = 0, cols = 0;
};

struct DeltaNetW {
  Mat qkv, z, b, a, out;
  std::vector<float> conv, neg_a, dt_bias, norm;
};
struct AttnW {
  Mat q, k, v, o;
  std::vector<float> q_norm, k_norm;
};
struct LayerW {
  int kind = 0;  // 0 = linear (DeltaNet), 1 = full attention
  std::vector<float> ln1, ln2;
  DeltaNetW dn;
  AttnW at;
  Mat gate, up, down;
};

struct Cfg {
  int hidden, intermediate, n_layers, vocab;
  float eps;
  int n_heads, n_kv_heads, head_dim, rotary_dim;
  double rope_theta;
  int conv_kernel, lin_k_heads, lin_v_heads, lin_k_dim, lin_v_dim;
  int conv_dim() const { return 2 * lin_k_heads * lin_k_dim + lin_v_heads * lin_v_dim; }
};

struct Model {
  Cfg cfg;
  Mat embed, lm_head;
  std::vector<LayerW> layers;
  std::vector<float> final_norm, inv_freq;
  // The one documented deviation from model.rs, off by default: round each appended key and value to bf16
  // (round to nearest even), the storage format of the GPU's paged KV cache. model.rs:441-442 appends f32 rows.
  bool kv_bf16 = false;
  // Test aid for the bf16 cache's sensitivity: before rounding, scale each appended key and value by
  // (1 + kv_perturb * r), r uniform in [-1, 1) from a fixed generator. 0 (the default) leaves the values as they are.
  float kv_perturb = 0.0f;
  uint64_t kv_rng = 0x9E3779B97F4A7C15ull;
  // lens.rs:10-16: per-layer [d][d] maps (16-bit values widened to f32; empty = no map) and the target layer
  std::vector<std::vector<float>> lens;
  long lens_target = -1;
};

// f32 -> bf16 -> f32, round to nearest even (the rounding of the GPU cache's __float2bfloat16_rn); finite inputs.
inline float round_bf16(float x) {
  uint32_t u;
  memcpy(&u, &x, 4);
  if ((u & 0x7f800000u) != 0x7f800000u) u = (u + 0x7fffu + ((u >> 16) & 1u)) & 0xffff0000u;
  memcpy(&x, &u, 4);
  return x;
}

struct LayerCache {
  std::vector<float> conv, state;  // linear
  std::vector<float> k, v;         // full: [pos][kv][hd]
};
struct Cache {
  size_t pos = 0;
  std::vector<LayerCache> layers;
};

// steering.rs:77-104, with the ops already compiled (Add values multiplied by the dose unit).
struct Op {
  int neuron, kind;  // kind 1 add, 2 mul, 3 set
  float value;
  int gate;  // -1 none
};
struct GateSpec {
  float threshold;
  int last_layer;
};
struct Plan {
  std::vector<std::vector<Op>> ops;
  std::vector<GateSpec> gates;
  std::vector<std::vector<std::tuple<int, int, float>>> detectors;  // per layer: (gate, neuron, weight)
};
struct GateState {
  std::vector<char> open;
  std::vector<float> score;
  std::vector<std::vector<float>> partial;
  std::vector<int> opened_at;  // -1 = None
};

// steering.rs:151-160
void plan_begin(const Plan& p, GateState& st, size_t rows) {
  size_t g = p.gates.size();
  if (st.open.size() != g) {
    st.open.assign(g, 0);
    st.score.assign(g, 0.0f);
    st.partial.assign(g, {});
    st.opened_at.assign(g, -1);
  }
  for (auto& v : st.partial) {
    v.clear();
    v.resize(rows, 0.0f);
  }
  for (auto& o : st.opened_at) o = -1;
}

// steering.rs:163-210
void plan_apply(const Plan& p, int layer, float* acts, size_t n, size_t rows, GateState& st) {
  if ((size_t)layer < p.detectors.size()) {
    for (auto& [g, neuron, w] : p.detectors[layer])
      for (size_t r = 0; r < rows; r++)
        if (r < st.partial[g].size()) st.partial[g][r] += w * acts[r * n + neuron];
    for (size_t g = 0; g < p.gates.size(); g++) {
      if (p.gates[g].last_layer != layer || st.partial[g].empty()) continue;
      st.score[g] = st.partial[g].back();
      if (!st.open[g]) {
        for (size_t r = 0; r < st.partial[g].size(); r++)
          if (st.partial[g][r] > p.gates[g].threshold) {
            st.opened_at[g] = (int)r;
            st.open[g] = 1;
            break;
          }
      }
    }
  }
  if ((size_t)layer >= p.ops.size()) return;
  for (const Op& op : p.ops[layer]) {
    size_t from = 0;
    if (op.gate >= 0) {
      int g = op.gate;
      if (!st.open[g]) continue;
      if (st.opened_at[g] >= 0) {
        if (p.gates[g].last_layer <= layer) from = (size_t)st.opened_at[g];
        else continue;
      }
    }
    for (size_t r = from; r < rows; r++) {
      float& a = acts[r * n + op.neuron];
      if (op.kind == 1) a += op.value;
      else if (op.kind == 2) a *= op.value;
      else if (op.kind == 3) a = op.value;
    }
  }
}

// One sequence of a forward call.
struct SeqIO {
  Cache* cache;
  const uint32_t* tokens;
  long n;
  const Plan* plan;     // may be null
  GateState* gate;      // required when plan != null
  int8_t* frames;       // [n][layers*intermediate] or null
  uint16_t* resid;      // [n][layers*hidden] f16 or null
};

void rope(const Model& m, float* x, size_t pos) {
  int half = m.cfg.rotary_dim / 2;
  for (int i = 0; i < half; i++) {
    float ang = (float)pos * m.inv_freq[i];
    float s = sinf(ang), c = cosf(ang);
    float a = x[i], b = x[i + half];
    x[i] = a * c - b * s;
    x[i + half] = b * c + a * s;
  }
}

// model.rs:296-396
void deltanet(const Model& m, const DeltaNetW& dn, int li, const float* h, long total, SeqIO* seqs, int nseq,
              const std::vector<long>& offs, float* out) {
  const Cfg& cfg = m.cfg;
  int c = cfg.conv_dim();
  int hk = cfg.lin_k_heads, hv = cfg.lin_v_heads, dk = cfg.lin_k_dim, dv = cfg.lin_v_dim;
  int key_dim = hk * dk, vd = hv * dv, kern = cfg.conv_kernel;
  std::vector<float> qkv((size_t)total * c), z((size_t)total * vd), bb((size_t)total * hv), aa((size_t)total * hv);
  matmul(dn.qkv.p, dn.qkv.rows, dn.qkv.cols, h, total, qkv.data());
  matmul(dn.z.p, dn.z.rows, dn.z.cols, h, total, z.data());
  matmul(dn.b.p, dn.b.rows, dn.b.cols, h, total, bb.data());
  matmul(dn.a.p, dn.a.rows, dn.a.cols, h, total, aa.data());
  std::vector<float> core((size_t)total * vd, 0.0f);
  for (int s = 0; s < nseq; s++) {
    long r0 = offs[s], nrows = offs[s + 1] - offs[s];
    if (nrows == 0) continue;
    LayerCache& lc = seqs[s].cache->layers[li];
    float* rows = qkv.data() + (size_t)r0 * c;
    std::vector<float> ext((size_t)(kern - 1 + nrows) * c);
    memcpy(ext.data(), lc.conv.data(), sizeof(float) * (kern - 1) * c);
    memcpy(ext.data() + (size_t)(kern - 1) * c, rows, sizeof(float) * nrows * c);
    par_for(nrows, [&](long t) {
      float* row = rows + (size_t)t * c;
      for (int ch = 0; ch < c; ch++) {
        const float* w = dn.conv.data() + (size_t)ch * kern;
        float acc = 0.0f;
        for (int j = 0; j < kern; j++) acc += w[j] * ext[(size_t)(t + j) * c + ch];
        row[ch] = silu(acc);
      }
    });
    memcpy(lc.conv.data(), ext.data() + (size_t)nrows * c, sizeof(float) * (kern - 1) * c);
    float qscale = 1.0f / sqrtf((float)dk);
    par_for(nrows, [&](long t) {
      float* row = rows + (size_t)t * c;
      for (int head = 0; head < hk; head++) {
        int bases[2] = {head * dk, key_dim + head * dk};
        float scales[2] = {qscale, 1.0f};
        for (int u = 0; u < 2; u++) {
          float* v = row + bases[u];
          float inv = 1.0f / sqrtf(dot(v, v, dk) + 1e-6f);
          float f = inv * scales[u];
          for (int i = 0; i < dk; i++) v[i] *= f;
        }
      }
    });
    const float* bseg = bb.data() + (size_t)r0 * hv;
    const float* aseg = aa.data() + (size_t)r0 * hv;
    const float* zseg = z.data() + (size_t)r0 * vd;
    int ratio = hv / hk;
    float eps = cfg.eps;
    par_for(hv, [&](long head) {
      float* st = lc.state.data() + (size_t)head * dk * dv;
      int kh = (int)head / ratio;
      std::vector<float> kv(dv), o(dv);
      for (long t = 0; t < nrows; t++) {
        const float* row = rows + (size_t)t * c;
        const float* q = row + kh * dk;
        const float* k = row + key_dim + kh * dk;
        const float* v = row + 2 * key_dim + head * dv;
        float decay = expf(dn.neg_a[head] * softplus(aseg[t * hv + head] + dn.dt_bias[head]));
        float beta = sigmoid(bseg[t * hv + head]);
        recur_body(st, q, k, v, decay, beta, kv.data(), o.data(), dk, dv);
        const float* zt = zseg + (size_t)t * vd + head * dv;
        float inv = 1.0f / sqrtf(dot(o.data(), o.data(), dv) / (float)dv + eps);
        float* dst = core.data() + (size_t)(r0 + t) * vd + head * dv;
        for (int j = 0; j < dv; j++) dst[j] = o[j] * inv * dn.norm[j] * silu(zt[j]);
      }
    });
  }
  matmul(dn.out.p, dn.out.rows, dn.out.cols, core.data(), total, out);
}

// model.rs:398-467
void attention(const Model& m, const AttnW& at, int li, const float* h, long total, SeqIO* seqs, int nseq,
               const std::vector<long>& offs, float* out) {
  const Cfg& cfg = m.cfg;
  int nh = cfg.n_heads, nkv = cfg.n_kv_heads, hd = cfg.head_dim;
  std::vector<float> qg((size_t)total * nh * hd * 2), kk((size_t)total * nkv * hd), vv((size_t)total * nkv * hd);
  matmul(at.q.p, at.q.rows, at.q.cols, h, total, qg.data());
  matmul(at.k.p, at.k.rows, at.k.cols, h, total, kk.data());
  matmul(at.v.p, at.v.rows, at.v.cols, h, total, vv.data());
  std::vector<float> o((size_t)total * nh * hd, 0.0f);
  float scale = 1.0f / sqrtf((float)hd);
  int group = nh / nkv;
  for (int s = 0; s < nseq; s++) {
    long r0 = offs[s], nrows = offs[s + 1] - offs[s];
    if (nrows == 0) continue;
    size_t pos0 = seqs[s].cache->pos;
    par_for(nrows, [&](long t) {
      float* row = qg.data() + (size_t)(r0 + t) * nh * hd * 2;
      std::vector<float> tmp(hd);
      for (int head = 0; head < nh; head++) {
        float* q = row + (size_t)head * 2 * hd;
        memcpy(tmp.data(), q, sizeof(float) * hd);
        rmsnorm(tmp.data(), at.q_norm.data(), cfg.eps, q, hd);
        rope(m, q, pos0 + t);
      }
    });
    par_for(nrows, [&](long t) {
      float* row = kk.data() + (size_t)(r0 + t) * nkv * hd;
      std::vector<float> tmp(hd);
      for (int head = 0; head < nkv; head++) {
        float* k = row + (size_t)head * hd;
        memcpy(tmp.data(), k, sizeof(float) * hd);
        rmsnorm(tmp.data(), at.k_norm.data(), cfg.eps, k, hd);
        rope(m, k, pos0 + t);
      }
    });
    LayerCache& lc = seqs[s].cache->layers[li];
    if (m.kv_bf16) {
      Model& mm = const_cast<Model&>(m);
      auto jitter = [&](float x) {
        if (mm.kv_perturb == 0.0f) return x;
        mm.kv_rng = mm.kv_rng * 6364136223846793005ull + 1442695040888963407ull;
        const float r = (float)((mm.kv_rng >> 40) & 0xffffff) / 8388608.0f - 1.0f;
        return x * (1.0f + mm.kv_perturb * r);
      };
      for (size_t i = (size_t)r0 * nkv * hd; i < (size_t)(r0 + nrows) * nkv * hd; i++) {
        kk[i] = round_bf16(jitter(kk[i]));
        vv[i] = round_bf16(jitter(vv[i]));
      }
    }
    lc.k.insert(lc.k.end(), kk.begin() + (size_t)r0 * nkv * hd, kk.begin() + (size_t)(r0 + nrows) * nkv * hd);
    lc.v.insert(lc.v.end(), vv.begin() + (size_t)r0 * nkv * hd, vv.begin() + (size_t)(r0 + nrows) * nkv * hd);
    const float* kc = lc.k.data();
    const float* vc = lc.v.data();
    par_for(nrows * nh, [&](long i) {
      long t = i / nh;
      int head = (int)(i % nh);
      int kvh = head / group;
      const float* qrow = qg.data() + (size_t)(r0 + t) * nh * hd * 2;
      const float* q = qrow + (size_t)head * 2 * hd;
      const float* gate = q + hd;
      size_t ctx = pos0 + t + 1;
      std::vector<float> sc(ctx);
      for (size_t j = 0; j < ctx; j++) sc[j] = dot(q, kc + (j * nkv + kvh) * hd, hd) * scale;
      softmax_inplace(sc.data(), ctx);
      float* oh = o.data() + (size_t)(r0 + t) * nh * hd + (size_t)head * hd;
      for (int d = 0; d < hd; d++) oh[d] = 0.0f;
      for (size_t j = 0; j < ctx; j++) {
        const float* vr = vc + (j * nkv + kvh) * hd;
        float p = sc[j];
        for (int d = 0; d < hd; d++) oh[d] += p * vr[d];
      }
      for (int d = 0; d < hd; d++) oh[d] *= sigmoid(gate[d]);
    });
  }
  matmul(at.o.p, at.o.rows, at.o.cols, o.data(), total, out);
}

// model.rs:217-294 (+ Probe hooks, worker.rs:130-152). Returns logits for the last row of each sequence
// with rows (rows of sequences without tokens are left untouched).
void forward(Model& m, SeqIO* seqs, int nseq, const float* act_scale, float* track_max, int want_logits,
             float* logits) {
  const Cfg& cfg = m.cfg;
  size_t d = cfg.hidden, n = cfg.intermediate;
  std::vector<long> offs(nseq + 1, 0);
  for (int i = 0; i < nseq; i++) offs[i + 1] = offs[i] + seqs[i].n;
  long total = offs[nseq];
  if (total == 0) return;
  std::vector<float> x((size_t)total * d), h((size_t)total * d), mixed((size_t)total * d);
  std::vector<float> g((size_t)total * n), u((size_t)total * n);
  {
    std::vector<uint32_t> toks;
    for (int i = 0; i < nseq; i++) toks.insert(toks.end(), seqs[i].tokens, seqs[i].tokens + seqs[i].n);
    par_for(total, [&](long r) {
      const uint16_t* e = m.embed.p + (size_t)toks[r] * m.embed.cols;
      for (size_t i = 0; i < d; i++) x[r * d + i] = bf16_to_f32(e[i]);
    });
  }
  for (int i = 0; i < nseq; i++)
    if (seqs[i].plan) plan_begin(*seqs[i].plan, *seqs[i].gate, (size_t)seqs[i].n);
  for (int li = 0; li < cfg.n_layers; li++) {
    LayerW& layer = m.layers[li];
    rmsnorm_rows(x.data(), layer.ln1.data(), cfg.eps, h.data(), d, total);
    if (layer.kind == 0) deltanet(m, layer.dn, li, h.data(), total, seqs, nseq, offs, mixed.data());
    else attention(m, layer.at, li, h.data(), total, seqs, nseq, offs, mixed.data());
    add_inplace(x.data(), mixed.data(), x.size());
    rmsnorm_rows(x.data(), layer.ln2.data(), cfg.eps, h.data(), d, total);
    matmul(layer.gate.p, layer.gate.rows, layer.gate.cols, h.data(), total, g.data());
    matmul(layer.up.p, layer.up.rows, layer.up.cols, h.data(), total, u.data());
    {
      size_t nn = g.size();
      long chunks = (long)((nn + (1 << 14) - 1) >> 14);
      par_for(chunks, [&](long c) {
        size_t a = (size_t)c << 14, b = std::min(nn, a + (1 << 14));
        for (size_t i = a; i < b; i++) g[i] = silu(g[i]) * u[i];
      });
    }
    for (int s = 0; s < nseq; s++) {
      SeqIO& sq = seqs[s];
      long rows = offs[s + 1] - offs[s];
      float* acts = g.data() + (size_t)offs[s] * n;
      if (sq.plan) plan_apply(*sq.plan, li, acts, n, (size_t)rows, *sq.gate);
      if (sq.frames) {
        const float* sc = act_scale ? act_scale + (size_t)li * n : nullptr;
        par_for(rows, [&](long r) {
          int8_t* dst = sq.frames + (size_t)r * cfg.n_layers * n + (size_t)li * n;
          const float* src = acts + (size_t)r * n;
          for (size_t j = 0; j < n; j++) dst[j] = compand(sc ? src[j] / sc[j] : src[j]);
        });
      }
      if (track_max) {
        float* dst = track_max + (size_t)li * n;
        for (long r = 0; r < rows; r++) {
          if (sq.cache->pos + r == 0) continue;
          const float* src = acts + (size_t)r * n;
          for (size_t j = 0; j < n; j++) dst[j] = fmaxf(dst[j], fabsf(src[j]));
        }
      }
    }
    matmul(layer.down.p, layer.down.rows, layer.down.cols, g.data(), total, mixed.data());
    add_inplace(x.data(), mixed.data(), x.size());
    for (int s = 0; s < nseq; s++) {
      SeqIO& sq = seqs[s];
      if (!sq.resid) continue;
      long rows = offs[s + 1] - offs[s];
      for (long r = 0; r < rows; r++) {
        uint16_t* dst = sq.resid + (size_t)r * cfg.n_layers * d + (size_t)li * d;
        const float* src = x.data() + (size_t)(offs[s] + r) * d;
        for (size_t i = 0; i < d; i++) dst[i] = f32_to_f16(src[i]);
      }
    }
  }
  for (int s = 0; s < nseq; s++) seqs[s].cache->pos += seqs[s].n;
  if (!want_logits) return;
  std::vector<int> live;
  for (int s = 0; s < nseq; s++)
    if (seqs[s].n > 0) live.push_back(s);
  std::vector<float> last(live.size() * d), normed(live.size() * d);
  for (size_t i = 0; i < live.size(); i++) {
    long r = offs[live[i] + 1] - 1;
    memcpy(last.data() + i * d, x.data() + (size_t)r * d, sizeof(float) * d);
  }
  rmsnorm_rows(last.data(), m.final_norm.data(), cfg.eps, normed.data(), d, (long)live.size());
  size_t v = m.lm_head.rows;
  std::vector<float> out(live.size() * v);
  matmul(m.lm_head.p, m.lm_head.rows, m.lm_head.cols, normed.data(), live.size(), out.data());
  for (size_t i = 0; i < live.size(); i++) memcpy(logits + (size_t)live[i] * v, out.data() + i * v, sizeof(float) * v);
}

}  // namespace

// ------------------------------------------------------------------------------------------------
// C ABI for the ctypes wrapper (oracle/__init__.py)

EXPORT void oracle_set_threads(int n) { pool().resize(n); }
EXPORT int oracle_threads() { return n_threads(); }

EXPORT void oracle_matmul(const uint16_t* w, long rows, long cols, const float* x, long n, float* y) {
  matmul(w, rows, cols, x, n, y);
}
EXPORT void* oracle_sampler_new(float t, float top_p, float min_p, float rep, uint64_t seed) {
  return new Sampler(sampler_new(t, top_p, min_p, rep, seed));
}
EXPORT void oracle_sampler_free(void* s) { delete (Sampler*)s; }
EXPORT uint64_t oracle_sampler_rng(void* s) { return ((Sampler*)s)->rng; }
EXPORT uint32_t oracle_sampler_sample(void* s, const float* logits, long n, const uint32_t* history, long nh) {
  return sampler_sample(*(Sampler*)s, logits, (size_t)n, history, (size_t)nh);
}
// crates/evie/src/mcp.rs:242-256 (top_active): the k entries of one frame with the largest |q|, largest first; the
// reference leaves the order of equal |q| undefined (select_nth_unstable_by), here it is the lower flat index first.
EXPORT int oracle_top_active(const int8_t* f, long n, int k, int32_t* out) {
  if (k > n) k = (int)n;
  std::vector<int32_t> idx(n);
  for (long i = 0; i < n; i++) idx[i] = (int32_t)i;
  auto mag = [&](int32_t i) { return f[i] < 0 ? -(int)f[i] : (int)f[i]; };
  std::partial_sort(idx.begin(), idx.begin() + k, idx.end(), [&](int32_t a, int32_t b) {
    return mag(a) != mag(b) ? mag(a) > mag(b) : a < b;
  });
  for (int i = 0; i < k; i++) out[i] = idx[i];
  return k;
}
// crates/evie-core/src/analysis.rs:129-175 (UnembedStats::compute) and 183-201 (neuron_sigma): mean of the
// unembedding rows (f64 sums), the gain-weighted covariance of a strided subsample of at most 16384 rows (the
// centred rows scaled by 64 and rounded to f16 as the GEMM's weight operand), normalised to its largest magnitude
// and stored as f16; then sigma = sqrt(max(u . (M u) * m_scale, 1e-30)) for every down_proj column u (carried
// through the lens map of its layer first when a lens is set).
struct UnembedStats {
  std::vector<float> mean;
  std::vector<float> m;  // d x d, the f16 values widened
  float m_scale = 0.0f;
};
UnembedStats unembed_stats(const Model& m) {
  const Mat& w = m.lm_head;
  const size_t v = w.rows, d = w.cols;
  const float* g = m.final_norm.data();
  std::vector<double> sums(d, 0.0);
  for (size_t r = 0; r < v; r++)
    for (size_t i = 0; i < d; i++) sums[i] += (double)bf16_to_f32(w.p[r * d + i]);
  UnembedStats st;
  st.mean.resize(d);
  for (size_t i = 0; i < d; i++) st.mean[i] = (float)(sums[i] / (double)v);
  const size_t s = std::min<size_t>(16384, v), stride = v / s;
  std::vector<float> xt(d * s), xw(d * s);  // x^T (d x s) and its f16(64 x) widening, the GEMM weight
  for (size_t j = 0; j < s; j++)
    for (size_t i = 0; i < d; i++) {
      const float x = (bf16_to_f32(w.p[j * stride * d + i]) - st.mean[i]) * g[i];
      xt[i * s + j] = x;
      xw[i * s + j] = f16_to_f32(f32_to_f16(x * 64.0f));
    }
  std::vector<float> cov(d * d);
  packed_gemm(xw.data(), d, s, xt.data(), d, cov.data());
  const float norm = 1.0f / ((float)s * 64.0f);
  float mx = 0.0f;
  for (auto& c : cov) {
    c *= norm;
    mx = std::max(mx, std::fabs(c));
  }
  st.m_scale = std::max(mx, 1e-30f);
  st.m.resize(d * d);
  for (size_t i = 0; i < d * d; i++) st.m[i] = f16_to_f32(f32_to_f16(cov[i] / st.m_scale));
  return st;
}
// lens.rs:57-62 (map: none past the target layer or where the file has no map) and 64-73 (transport: J_l @ x for n
// row vectors, the identity without a map).
const float* lens_map(const Model& m, size_t layer) {
  if ((long)layer > m.lens_target || layer >= m.lens.size() || m.lens[layer].empty()) return nullptr;
  return m.lens[layer].data();
}
std::vector<float> transport(const Model& m, size_t layer, const float* x, size_t n) {
  const size_t d = m.cfg.hidden;
  const float* j = lens_map(m, layer);
  if (!j) return std::vector<float>(x, x + n * d);
  std::vector<float> y(n * d);
  matmul(j, d, d, x, n, y.data());
  return y;
}
// kernels.rs:525-552 (matvec_t): out[c] = sum over rows r (in order, rows with x[r] == 0 skipped) of x[r] w[r][c],
// each product and sum separately rounded.
template <typename WT>
void matvec_t(const WT* w, size_t rows, size_t cols, const float* x, float* out) {
  for (size_t c = 0; c < cols; c++) out[c] = 0.0f;
  for (size_t r = 0; r < rows; r++) {
    const float xr = x[r];
    if (xr == 0.0f) continue;
    const WT* row = w + r * cols;
    for (size_t c = 0; c < cols; c++) out[c] += xr * widen(row[c]);
  }
}
// lens.rs:76-82 (pullback: J_l^T a, the identity without a map)
std::vector<float> pullback(const Model& m, size_t layer, const float* a) {
  const size_t d = m.cfg.hidden;
  const float* j = lens_map(m, layer);
  if (!j) return std::vector<float>(a, a + d);
  std::vector<float> out(d);
  matvec_t(j, d, d, a, out.data());
  return out;
}
// model.rs:287-294 (unembed: final RMSNorm of each row, then the LM head)
std::vector<float> unembed(const Model& m, const float* x, size_t n) {
  const size_t d = m.cfg.hidden, v = m.lm_head.rows;
  std::vector<float> normed(n * d), out(n * v);
  rmsnorm_rows(x, m.final_norm.data(), m.cfg.eps, normed.data(), d, (long)n);
  matmul(m.lm_head.p, v, d, normed.data(), n, out.data());
  return out;
}

void neuron_sigma(const Model& m, const UnembedStats& st, float* sigma) {
  const size_t nl = m.layers.size(), n = m.cfg.intermediate, d = m.cfg.hidden;
  std::vector<float> u(n * d), mu(n * d);
  for (size_t l = 0; l < nl; l++) {
    const Mat& dn = m.layers[l].down;  // [d][n]
    for (size_t k = 0; k < d; k++)
      for (size_t i = 0; i < n; i++) u[i * d + k] = bf16_to_f32(dn.p[k * n + i]);  // transpose_to_f32
    if (lens_map(m, l)) u = transport(m, l, u.data(), n);                      // analysis.rs:188-191
    packed_gemm(st.m.data(), d, d, u.data(), n, mu.data());
    for (size_t i = 0; i < n; i++)
      sigma[l * n + i] = std::sqrt(std::max(dot(u.data() + i * d, mu.data() + i * d, d) * st.m_scale, 1e-30f));
  }
}
EXPORT float oracle_neuron_sigma(void* model, float* sigma, float* mean) {
  const Model& m = *(const Model*)model;
  UnembedStats st = unembed_stats(m);
  if (mean) memcpy(mean, st.mean.data(), st.mean.size() * sizeof(float));
  neuron_sigma(m, st, sigma);
  return st.m_scale;
}
// lens.rs:20-54 after the file is read: maps[l] = [d][d] 16-bit values (kind 0 = f16, 1 = bf16) or NULL.
EXPORT void oracle_lens_set(void* model, const uint16_t* const* maps, int n_layers, int kind, long target_layer) {
  Model& m = *(Model*)model;
  const size_t d = m.cfg.hidden;
  m.lens.assign(n_layers, {});
  for (int l = 0; l < n_layers; l++) {
    if (!maps[l]) continue;
    m.lens[l].resize(d * d);
    for (size_t i = 0; i < d * d; i++) m.lens[l][i] = kind == 0 ? f16_to_f32(maps[l][i]) : bf16_to_f32(maps[l][i]);
  }
  m.lens_target = target_layer;
}
EXPORT void oracle_lens_clear(void* model) {
  Model& m = *(Model*)model;
  m.lens.clear();
  m.lens_target = -1;
}
// analysis.rs:28-34 (lens_logits): [n][V] logits of n residual-basis vectors at `layer`
EXPORT void oracle_lens_logits(void* model, int layer, const float* vecs, long n, float* logits) {
  const Model& m = *(const Model*)model;
  const std::vector<float> t = transport(m, layer, vecs, n);
  const std::vector<float> out = unembed(m, t.data(), n);
  memcpy(logits, out.data(), out.size() * sizeof(float));
}
// analysis.rs:37-67 (write_dirs + neuron_logits): the write directions W_down[:, neuron] of each neuron's layer,
// transported in blocks of one layer (ascending layers), then unembedded in the given order.
EXPORT void oracle_neuron_logits(void* model, const int32_t* layers, const int32_t* neurons, long n, float* logits) {
  const Model& m = *(const Model*)model;
  const size_t d = m.cfg.hidden, ni = m.cfg.intermediate;
  std::vector<float> dirs(n * d), moved(n * d);
  for (long i = 0; i < n; i++) {
    const Mat& dn = m.layers[layers[i]].down;
    for (size_t k = 0; k < d; k++) dirs[i * d + k] = bf16_to_f32(dn.p[k * ni + neurons[i]]);  // col_to_f32
  }
  std::vector<int32_t> ls(layers, layers + n);
  std::sort(ls.begin(), ls.end());
  ls.erase(std::unique(ls.begin(), ls.end()), ls.end());
  for (int32_t l : ls) {
    std::vector<long> idx;
    for (long i = 0; i < n; i++)
      if (layers[i] == l) idx.push_back(i);
    std::vector<float> block;
    for (long i : idx) block.insert(block.end(), dirs.begin() + i * d, dirs.begin() + (i + 1) * d);
    const std::vector<float> t = transport(m, l, block.data(), idx.size());
    for (size_t j = 0; j < idx.size(); j++) memcpy(&moved[idx[j] * d], &t[j * d], d * sizeof(float));
  }
  const std::vector<float> out = unembed(m, moved.data(), n);
  memcpy(logits, out.data(), out.size() * sizeof(float));
}
// analysis.rs:213-251 (search): z scores of `tokens` for every neuron and pole against sigma, best token per
// (neuron, pole); per layer the hits sorted by z descending (stable) and cut to `limit`, then all layers merged the
// same way. Writes up to `limit` hits (layer, neuron, sign, z) and returns their count.
EXPORT long oracle_search(void* model, const uint32_t* tokens, long nt, const float* mean, const float* sigma,
                          long limit, int32_t* hit_layer, int32_t* hit_neuron, int32_t* hit_sign, float* hit_z) {
  const Model& m = *(const Model*)model;
  if (nt == 0) return 0;
  const size_t nl = m.layers.size(), n = m.cfg.intermediate, d = m.cfg.hidden;
  const float* g = m.final_norm.data();
  std::vector<std::vector<float>> a(nt, std::vector<float>(d));
  for (long t = 0; t < nt; t++)  // analysis.rs:173-179 (UnembedStats::centered)
    for (size_t i = 0; i < d; i++) a[t][i] = (bf16_to_f32(m.lm_head.p[(size_t)tokens[t] * d + i]) - mean[i]) * g[i];
  struct Hit {
    int32_t layer, neuron, sign;
    float z;
  };
  auto by_z = [](const Hit& x, const Hit& y) { return x.z > y.z; };
  std::vector<Hit> all;
  for (size_t l = 0; l < nl; l++) {
    const Mat& dn = m.layers[l].down;  // [d][n]
    std::vector<std::vector<float>> scores(nt, std::vector<float>(n));
    for (long t = 0; t < nt; t++) {
      const std::vector<float> pulled = pullback(m, l, a[t].data());
      matvec_t(dn.p, d, n, pulled.data(), scores[t].data());
    }
    std::vector<Hit> best;
    for (size_t i = 0; i < n; i++) {
      float up = -INFINITY, dnz = -INFINITY;
      for (long t = 0; t < nt; t++) {
        const float z = scores[t][i] / sigma[l * n + i];
        up = std::max(up, z);
        dnz = std::max(dnz, -z);
      }
      best.push_back({(int32_t)l, (int32_t)i, 1, up});
      best.push_back({(int32_t)l, (int32_t)i, -1, dnz});
    }
    std::stable_sort(best.begin(), best.end(), by_z);
    if ((long)best.size() > limit) best.resize(limit);
    all.insert(all.end(), best.begin(), best.end());
  }
  std::stable_sort(all.begin(), all.end(), by_z);
  if ((long)all.size() > limit) all.resize(limit);
  for (size_t i = 0; i < all.size(); i++) {
    hit_layer[i] = all[i].layer;
    hit_neuron[i] = all[i].neuron;
    hit_sign[i] = all[i].sign;
    hit_z[i] = all[i].z;
  }
  return (long)all.size();
}
EXPORT int oracle_topk(const float* v, long n, int k, uint32_t* idx, float* val) { return topk(v, n, k, idx, val); }
EXPORT void oracle_softmax(float* x, long n) { softmax_inplace(x, n); }
EXPORT float oracle_dot(const float* a, const float* b, long n) { return dot(a, b, n); }

// Gated DeltaNet single decode step over B*H independent heads (model.rs:374-376 + recur_body).
// S: [B][H][dk][dv] f32 (updated in place); q,k: [B][H][dk] bf16; v: [B][H][dv] bf16;
// g (log decay) and beta: [B][H] f32; o: [B][H][dv] f32 = S_new^T q.
EXPORT void oracle_gdn_decode(int B, int H, int dk, int dv, float* S, const uint16_t* q, const uint16_t* k,
                              const uint16_t* v, const float* g, const float* beta, float* o) {
  par_for((long)B * H, [&](long bh) {
    std::vector<float> qf(dk), kf(dk), vf(dv), kv(dv);
    for (int i = 0; i < dk; i++) qf[i] = bf16_to_f32(q[bh * dk + i]), kf[i] = bf16_to_f32(k[bh * dk + i]);
    for (int j = 0; j < dv; j++) vf[j] = bf16_to_f32(v[bh * dv + j]);
    recur_body(S + (size_t)bh * dk * dv, qf.data(), kf.data(), vf.data(), expf(g[bh]), beta[bh], kv.data(),
               o + (size_t)bh * dv, dk, dv);
  });
}

// Gated DeltaNet prefill, token-sequential exactly as evie-core runs it (it has no chunked form).
// q,k: [B][T][H][dk] bf16; v: [B][T][H][dv] bf16; g, beta: [B][T][H] f32; S: [B][H][dk][dv] (in: initial,
// out: final); o: [B][T][H][dv] f32.
EXPORT void oracle_gdn_prefill(int B, int T, int H, int dk, int dv, float* S, const uint16_t* q, const uint16_t* k,
                               const uint16_t* v, const float* g, const float* beta, float* o) {
  par_for((long)B * H, [&](long bh) {
    long b = bh / H, h = bh % H;
    std::vector<float> qf(dk), kf(dk), vf(dv), kv(dv);
    float* st = S + (size_t)bh * dk * dv;
    for (long t = 0; t < T; t++) {
      size_t row = ((size_t)b * T + t) * H + h;
      for (int i = 0; i < dk; i++) qf[i] = bf16_to_f32(q[row * dk + i]), kf[i] = bf16_to_f32(k[row * dk + i]);
      for (int j = 0; j < dv; j++) vf[j] = bf16_to_f32(v[row * dv + j]);
      recur_body(st, qf.data(), kf.data(), vf.data(), expf(g[row]), beta[row], kv.data(), o + row * dv, dk, dv);
    }
  });
}

// Gated GQA decode attention core (model.rs:445-464) over a paged KV cache.
// q, gate (logits): [B][Hq][hd] bf16; pages: [num_pages][Hkv][page_size][hd] bf16; page_table: [B][max_pages];
// ctx: [B]; out: [B][Hq][hd] f32 = softmax(q.K^T * scale) V * sigmoid(gate).
EXPORT void oracle_gqa_decode(int B, int Hq, int Hkv, int hd, int page_size, const uint16_t* q, const uint16_t* kp,
                              const uint16_t* vp, const int32_t* page_table, int max_pages, const int32_t* ctx,
                              const uint16_t* gate, float scale, float* out) {
  int group = Hq / Hkv;
  par_for((long)B * Hq, [&](long bh) {
    long b = bh / Hq;
    int head = (int)(bh % Hq), kvh = head / group;
    long n = ctx[b];
    std::vector<float> qf(hd), kf(hd), sc(n > 0 ? n : 1);
    for (int i = 0; i < hd; i++) qf[i] = bf16_to_f32(q[bh * hd + i]);
    auto row_of = [&](const uint16_t* pages, long j) {
      long page = page_table[b * max_pages + j / page_size];
      return pages + (((size_t)page * Hkv + kvh) * page_size + (size_t)(j % page_size)) * hd;
    };
    for (long j = 0; j < n; j++) {
      const uint16_t* kr = row_of(kp, j);
      for (int i = 0; i < hd; i++) kf[i] = bf16_to_f32(kr[i]);
      sc[j] = dot(qf.data(), kf.data(), hd) * scale;
    }
    float* oh = out + (size_t)bh * hd;
    for (int i = 0; i < hd; i++) oh[i] = 0.0f;
    if (n > 0) softmax_inplace(sc.data(), n);
    for (long j = 0; j < n; j++) {
      const uint16_t* vr = row_of(vp, j);
      float p = sc[j];
      for (int i = 0; i < hd; i++) oh[i] += p * bf16_to_f32(vr[i]);
    }
    for (int i = 0; i < hd; i++) oh[i] *= sigmoid(bf16_to_f32(gate[bh * hd + i]));
  });
}

// The attention core of Model::attention (model.rs:445-464) for prefill rows with f32 queries and gate logits over a
// paged bf16 cache: row r belongs to sequence row_seq[r] (its page-table row) and sits at position row_pos[r], so
// its context is positions 0..row_pos[r]. q, gate, out: [R][Hq][hd]; pages: [num_pages][Hkv][page_size][hd].
EXPORT void oracle_gqa_rows(int R, int Hq, int Hkv, int hd, int page_size, const float* q, const uint16_t* kp,
                            const uint16_t* vp, const int32_t* page_table, int max_pages, const int32_t* row_seq,
                            const int32_t* row_pos, const float* gate, float scale, float* out) {
  int group = Hq / Hkv;
  par_for((long)R * Hq, [&](long rh) {
    long r = rh / Hq;
    int head = (int)(rh % Hq), kvh = head / group;
    long s = row_seq[r], n = (long)row_pos[r] + 1;
    std::vector<float> kf(hd), sc(n);
    auto row_of = [&](const uint16_t* pages, long j) {
      long page = page_table[s * max_pages + j / page_size];
      return pages + (((size_t)page * Hkv + kvh) * page_size + (size_t)(j % page_size)) * hd;
    };
    const float* qr = q + (size_t)rh * hd;
    for (long j = 0; j < n; j++) {
      const uint16_t* kr = row_of(kp, j);
      for (int i = 0; i < hd; i++) kf[i] = bf16_to_f32(kr[i]);
      sc[j] = dot(qr, kf.data(), hd) * scale;
    }
    softmax_inplace(sc.data(), n);
    float* oh = out + (size_t)rh * hd;
    for (int i = 0; i < hd; i++) oh[i] = 0.0f;
    for (long j = 0; j < n; j++) {
      const uint16_t* vr = row_of(vp, j);
      float p = sc[j];
      for (int i = 0; i < hd; i++) oh[i] += p * bf16_to_f32(vr[i]);
    }
    for (int i = 0; i < hd; i++) oh[i] *= sigmoid(gate[(size_t)rh * hd + i]);
  });
}

// ---- model ----

struct oracle_cfg {
  int hidden, intermediate, n_layers, vocab;
  float eps;
  int n_heads, n_kv_heads, head_dim, rotary_dim;
  double rope_theta;
  int conv_kernel, lin_k_heads, lin_v_heads, lin_k_dim, lin_v_dim;
};

EXPORT void* oracle_model_new(const oracle_cfg* c, const int* kinds) {
  Model* m = new Model();
  m->cfg = Cfg{c->hidden,     c->intermediate, c->n_layers,    c->vocab,       c->eps,
               c->n_heads,    c->n_kv_heads,   c->head_dim,    c->rotary_dim,  c->rope_theta,
               c->conv_kernel, c->lin_k_heads, c->lin_v_heads, c->lin_k_dim,   c->lin_v_dim};
  m->layers.resize(c->n_layers);
  for (int i = 0; i < c->n_layers; i++) m->layers[i].kind = kinds[i];
  int half = c->rotary_dim / 2;
  for (int i = 0; i < half; i++)
    m->inv_freq.push_back(1.0f / powf((float)c->rope_theta, (float)(2 * i) / (float)c->rotary_dim));
  return m;
}
EXPORT void oracle_model_free(void* p) { delete (Model*)p; }
// Switches the bf16 rounding of appended keys and values (Model::kv_bf16) on or off, with the optional relative
// jitter before rounding (Model::kv_perturb).
EXPORT void oracle_model_kv_bf16(void* p, int on, float perturb) {
  ((Model*)p)->kv_bf16 = on != 0;
  ((Model*)p)->kv_perturb = perturb;
}

// Registers one tensor. Matrices are bf16 views (the caller keeps the memory alive); vectors are copied
// as f32 with the load-time transforms of model.rs:148,171 (1+w norms, -exp(A_log)).
// slot codes: matrices 1 embed, 2 lm_head, 10 qkv, 11 z, 12 b, 13 a, 14 out, 20 q, 21 k, 22 v, 23 o, 30 gate,
// 31 up, 32 down; vectors 40 ln1(+1), 41 ln2(+1), 42 final_norm(+1), 43 q_norm(+1), 44 k_norm(+1),
// 45 conv, 46 A_log(->-exp), 47 dt_bias, 48 gated norm (as is).
EXPORT int oracle_model_set(void* p, int layer, int slot, const void* data, int is_bf16, long rows, long cols) {
  Model* m = (Model*)p;
  if (slot < 40) {
    if (!is_bf16) return -1;
    Mat mat{(const uint16_t*)data, (size_t)rows, (size_t)cols};
    if (slot == 1) { m->embed = mat; return 0; }
    if (slot == 2) { m->lm_head = mat; return 0; }
    if (layer < 0 || layer >= (int)m->layers.size()) return -2;
    LayerW& L = m->layers[layer];
    switch (slot) {
      case 10: L.dn.qkv = mat; break;
      case 11: L.dn.z = mat; break;
      case 12: L.dn.b = mat; break;
      case 13: L.dn.a = mat; break;
      case 14: L.dn.out = mat; break;
      case 20: L.at.q = mat; break;
      case 21: L.at.k = mat; break;
      case 22: L.at.v = mat; break;
      case 23: L.at.o = mat; break;
      case 30: L.gate = mat; break;
      case 31: L.up = mat; break;
      case 32: L.down = mat; break;
      default: return -3;
    }
    return 0;
  }
  size_t n = (size_t)rows * (size_t)cols;
  std::vector<float> v(n);
  for (size_t i = 0; i < n; i++)
    v[i] = is_bf16 ? bf16_to_f32(((const uint16_t*)data)[i]) : ((const float*)data)[i];
  if (slot == 40 || slot == 41 || slot == 42 || slot == 43 || slot == 44)
    for (auto& x : v) x = 1.0f + x;
  if (slot == 46)
    for (auto& x : v) x = -expf(x);
  if (slot == 42) { m->final_norm = v; return 0; }
  if (layer < 0 || layer >= (int)m->layers.size()) return -2;
  LayerW& L = m->layers[layer];
  switch (slot) {
    case 40: L.ln1 = v; break;
    case 41: L.ln2 = v; break;
    case 43: L.at.q_norm = v; break;
    case 44: L.at.k_norm = v; break;
    case 45: L.dn.conv = v; break;
    case 46: L.dn.neg_a = v; break;
    case 47: L.dn.dt_bias = v; break;
    case 48: L.dn.norm = v; break;
    default: return -3;
  }
  return 0;
}

// model.rs:92-106
EXPORT void* oracle_cache_new(void* p) {
  Model* m = (Model*)p;
  const Cfg& c = m->cfg;
  Cache* cache = new Cache();
  cache->layers.resize(c.n_layers);
  for (int i = 0; i < c.n_layers; i++)
    if (m->layers[i].kind == 0) {
      cache->layers[i].conv.assign((size_t)(c.conv_kernel - 1) * c.conv_dim(), 0.0f);
      cache->layers[i].state.assign((size_t)c.lin_v_heads * c.lin_k_dim * c.lin_v_dim, 0.0f);
    }
  return cache;
}
EXPORT void oracle_cache_free(void* c) { delete (Cache*)c; }
// Timing aid: puts a cache at position `pos` without running a prefill. Every DeltaNet state and conv window and
// `pos` rows of every attention layer's keys and values are filled with values of a fixed generator (uniform in
// [-a, a], a = 0.1 for states and windows, 1 for keys and values), so that a decode step afterwards does the work
// of a step at that context length. The values carry no meaning; the CPU baseline uses this to time decode at the
// GPU's context without the hours-long prefill of the 4B-shaped model.
EXPORT void oracle_cache_seed(void* p, void* cp, long pos, uint64_t seed) {
  Model* m = (Model*)p;
  Cache* c = (Cache*)cp;
  const Cfg& cfg = m->cfg;
  uint64_t x = seed * 0x9E3779B97F4A7C15ull + 1;
  auto uni = [&x](float a) {
    x = x * 6364136223846793005ull + 1442695040888963407ull;
    return a * ((float)((x >> 40) & 0xffffff) / 8388608.0f - 1.0f);
  };
  for (int i = 0; i < cfg.n_layers; i++) {
    LayerCache& lc = c->layers[i];
    if (m->layers[i].kind == 0) {
      for (float& v : lc.conv) v = uni(0.1f);
      for (float& v : lc.state) v = uni(0.1f);
    } else {
      const size_t n = (size_t)pos * cfg.n_kv_heads * cfg.head_dim;
      lc.k.resize(n);
      lc.v.resize(n);
      for (size_t j = 0; j < n; j++) lc.k[j] = uni(1.0f), lc.v[j] = uni(1.0f);
    }
  }
  c->pos = (size_t)pos;
}
EXPORT void* oracle_cache_clone(void* c) { return new Cache(*(Cache*)c); }
EXPORT long oracle_cache_pos(void* c) { return (long)((Cache*)c)->pos; }
// Copies one linear layer's recurrent state ([hv][dk][dv] f32) or conv window out of a cache.
EXPORT long oracle_cache_read(void* c, int layer, int which, float* dst, long cap) {
  LayerCache& lc = ((Cache*)c)->layers[layer];
  std::vector<float>& v = which == 0 ? lc.state : which == 1 ? lc.conv : which == 2 ? lc.k : lc.v;
  long n = (long)v.size();
  if (dst && cap >= n) memcpy(dst, v.data(), sizeof(float) * n);
  return n;
}

EXPORT void* oracle_plan_new(int n_layers) {
  Plan* p = new Plan();
  p->ops.resize(n_layers);
  p->detectors.resize(n_layers);
  return p;
}
EXPORT void oracle_plan_free(void* p) { delete (Plan*)p; }
EXPORT void oracle_plan_add_op(void* p, int layer, int neuron, int kind, float value, int gate) {
  ((Plan*)p)->ops[layer].push_back(Op{neuron, kind, value, gate});
}
EXPORT int oracle_plan_add_gate(void* p, float threshold, int last_layer) {
  Plan* pl = (Plan*)p;
  pl->gates.push_back(GateSpec{threshold, last_layer});
  return (int)pl->gates.size() - 1;
}
EXPORT void oracle_plan_add_detector(void* p, int gate, int layer, int neuron, float weight) {
  ((Plan*)p)->detectors[layer].emplace_back(gate, neuron, weight);
}
EXPORT void* oracle_gate_state_new() { return new GateState(); }
EXPORT void oracle_gate_state_free(void* s) { delete (GateState*)s; }
EXPORT int oracle_gate_state_open(void* s, int g) {
  GateState* st = (GateState*)s;
  return g < (int)st->open.size() ? st->open[g] : 0;
}
EXPORT float oracle_gate_state_score(void* s, int g) {
  GateState* st = (GateState*)s;
  return g < (int)st->score.size() ? st->score[g] : 0.0f;
}
// The running detector sums of gate g over the rows of the latest pass (GateState::partial, steering.rs:112).
EXPORT long oracle_gate_state_partial(void* s, int g, float* dst, long cap) {
  GateState* st = (GateState*)s;
  if (g >= (int)st->partial.size()) return 0;
  long n = (long)st->partial[g].size();
  if (dst && cap >= n) memcpy(dst, st->partial[g].data(), sizeof(float) * n);
  return n;
}
// Runs Plan::begin + Plan::apply on a plain activation block (steering.rs unit tests).
EXPORT void oracle_plan_begin(void* p, void* s, long rows) { plan_begin(*(Plan*)p, *(GateState*)s, rows); }
EXPORT void oracle_plan_apply(void* p, int layer, float* acts, long n, long rows, void* s) {
  plan_apply(*(Plan*)p, layer, acts, n, rows, *(GateState*)s);
}

struct oracle_seq {
  void* cache;
  const uint32_t* tokens;
  long n;
  void* plan;
  void* gate;
  int8_t* frames;
  uint16_t* resid;
};

EXPORT void oracle_forward(void* p, oracle_seq* seqs, int nseq, const float* act_scale, float* track_max,
                           int want_logits, float* logits) {
  std::vector<SeqIO> io(nseq);
  for (int i = 0; i < nseq; i++)
    io[i] = SeqIO{(Cache*)seqs[i].cache, seqs[i].tokens, seqs[i].n, (const Plan*)seqs[i].plan,
                  (GateState*)seqs[i].gate, seqs[i].frames, seqs[i].resid};
  forward(*(Model*)p, io.data(), nseq, act_scale, track_max, want_logits, logits);
}

EXPORT int8_t oracle_compand(float v) { return compand(v); }
EXPORT uint16_t oracle_f32_to_f16(float v) { return f32_to_f16(v); }
