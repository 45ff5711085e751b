// Host runtime of the full-model path: the C ABI that mirrors evie-core's GpuModel (crates/evie-core/src/gpu/mod.rs).
//
//   evie_create   GpuModel::new (gpu/mod.rs:226-262): config.json + safetensors -> device weights, slot caches
//   evie_forward  GpuModel::forward (gpu/mod.rs:615-706) = Model::forward (model.rs:217-284) on device
//   evie_set_ops / evie_reset_slot / evie_set_scale / evie_track_max / evie_read_max  (gpu/mod.rs:549-593)
//
// Device memory (all owned by the context):
//   weights   bf16; per layer the projections that read the same input are fused row-wise into one matrix:
//             DeltaNet [qkv; z; b; a] x d, attention [q(+gate); k; v] x d, MLP [gate; up] x d
//   caches    conv window [slot][lin layer][K-1][conv_dim] f32, recurrent state [slot][lin layer][hv][dk][dv] f32,
//             KV pages [full layer][slot * pages_per_slot][nkv][256][hd] (bf16, or f32 with EVIE_KV_F32=1),
//             a fixed page table per slot (slot s owns pages s*pps .. s*pps+pps-1)
//   activations sized for max_rows: residual x f32, split operand planes X2 bf16, projection outputs Y2 f32
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <dirent.h>
#include <fstream>
#include <map>
#include <tuple>
#include <memory>
#include <sstream>
#include <string>
#include <vector>

#include "common.h"
#include "gqa_decode.h"
#include "json.h"
#include "analysis.h"
#include "gdn_chunk.h"
#include "model_kernels.h"
#include "proj_gemm.h"
#include "sampler.h"

using evie::RowInfo;
using evie::SegInfo;

namespace {

constexpr int kPage = 256;
constexpr int kMaxOps = 64;
constexpr int kMaxGates = 32;
constexpr int kMaxDets = 128;

struct Tensor {
  std::string dtype;
  std::vector<int64_t> shape;
  const char* data = nullptr;
  size_t bytes = 0;
};

// weights.rs:33-123: every *.safetensors in the directory, memory-mapped.
struct SafeTensors {
  struct Map {
    void* p = MAP_FAILED;
    size_t n = 0;
  };
  std::vector<Map> maps;
  std::map<std::string, Tensor> t;
  ~SafeTensors() {
    for (auto& m : maps)
      if (m.p != MAP_FAILED) munmap(m.p, m.n);
  }
  std::string open_dir(const std::string& dir) {
    DIR* d = opendir(dir.c_str());
    if (!d) return "cannot open " + dir;
    std::vector<std::string> files;
    while (dirent* e = readdir(d)) {
      std::string n = e->d_name;
      if (n.size() > 12 && n.substr(n.size() - 12) == ".safetensors") files.push_back(dir + "/" + n);
    }
    closedir(d);
    std::sort(files.begin(), files.end());
    if (files.empty()) return "no .safetensors files in " + dir;
    for (auto& f : files) {
      int fd = open(f.c_str(), O_RDONLY);
      if (fd < 0) return "cannot open " + f;
      struct stat st;
      fstat(fd, &st);
      Map m;
      m.n = (size_t)st.st_size;
      m.p = mmap(nullptr, m.n, PROT_READ, MAP_PRIVATE, fd, 0);
      close(fd);
      if (m.p == MAP_FAILED || m.n < 8) return f + " is too small or unmappable";
      maps.push_back(m);
      const char* base = (const char*)m.p;
      uint64_t hn;
      memcpy(&hn, base, 8);
      if (8 + hn > m.n) return f + ": bad header length";
      evie::json::Value h;
      try {
        h = evie::json::parse(base + 8, hn);
      } catch (std::exception& e) {
        return f + ": " + e.what();
      }
      const char* data = base + 8 + hn;
      for (auto& kv : h.obj) {
        if (kv.first == "__metadata__") continue;
        Tensor x;
        x.dtype = kv.second["dtype"].string();
        for (auto& s : kv.second["shape"].arr) x.shape.push_back(s.integer());
        const auto& off = kv.second["data_offsets"].arr;
        size_t a = (size_t)off[0].integer(), b = (size_t)off[1].integer();
        if (8 + hn + b > m.n) return f + ": tensor " + kv.first + " out of range";
        x.data = data + a;
        x.bytes = b - a;
        t[kv.first] = x;
      }
    }
    return "";
  }
  const Tensor* get(const std::string& n) const {
    auto it = t.find(n);
    return it == t.end() ? nullptr : &it->second;
  }
};

float bf16_bits_to_f32(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}
float half_bits_to_f32(uint16_t h) {
  const uint32_t s = (h >> 15) & 1, e = (h >> 10) & 31, m = h & 1023;
  float v;
  if (e == 0) v = std::ldexp((float)m, -24);
  else if (e == 31) v = m ? NAN : INFINITY;
  else v = std::ldexp((float)(m | 1024), (int)e - 25);
  return s ? -v : v;
}

struct Layer {
  int kind = 0;  // 0 DeltaNet, 1 full attention
  int idx = 0;   // index among layers of the same kind
  float* ln1 = nullptr;
  float* ln2 = nullptr;
  __nv_bfloat16* w_in = nullptr;   // fused input projection
  __nv_bfloat16* w_out = nullptr;  // out_proj / o_proj [d][vd or nh*hd]
  __nv_bfloat16* w_gu = nullptr;   // [2n][d]
  __nv_bfloat16* w_down = nullptr; // [d][n]
  float *conv = nullptr, *neg_a = nullptr, *dt_bias = nullptr, *norm = nullptr;  // DeltaNet
  float *q_norm = nullptr, *k_norm = nullptr;                                    // attention
};

}  // namespace

// Kernel groups timed by the optional profiling mode (evie_profile).
// The projections are one group per weight (each is its own cuBLAS kernel shape).
enum ProfCat {
  P_GEMM_LIN_IN = 0,
  P_GEMM_LIN_OUT,
  P_GEMM_ATT_IN,
  P_GEMM_ATT_OUT,
  P_GEMM_GATE_UP,
  P_GEMM_DOWN,
  P_LMHEAD,
  P_CONV,
  P_MIXER,
  P_ATTN_PREP,
  P_ATTN,
  P_NORM,
  P_SWIGLU,
  P_OTHER,
  P_COUNT
};
const char* const kProfNames[P_COUNT] = {"gemm_linear_in", "gemm_linear_out", "gemm_attn_in", "gemm_attn_out",
                                         "gemm_mlp_gate_up", "gemm_mlp_down", "lm_head_gemm", "conv", "gdn_mixer",
                                         "attn_prep", "gqa_attention", "add_norm", "swiglu", "other"};

struct evie_ctx {
  int device = 0;
  cudaStream_t stream = nullptr;
  // Capture read-back: per-layer copies of frames and residual rows to page-locked host buffers run on cstream,
  // forked from the compute stream after each layer and joined at the end of the call (cap_ev: one per layer + 1).
  cudaStream_t cstream = nullptr;
  std::vector<cudaEvent_t> cap_ev;
  evie::LensDev lens;  // evie_set_lens: the lens of the analysis calls
  evie::ModelShape s{};
  std::vector<int> kinds;
  int n_lin = 0, n_full = 0;
  int slots = 0, max_ctx = 0, max_rows = 0, pages_per_slot = 0;
  bool kv_f32 = false;
  std::vector<void*> allocs;
  size_t weight_bytes = 0, cache_bytes = 0;
  // weights
  __nv_bfloat16* embed = nullptr;  // [V][d] (also the LM head when tied)
  __nv_bfloat16* lm_head = nullptr;
  float* final_norm = nullptr;
  float* inv_freq = nullptr;
  std::vector<Layer> layers;
  // caches
  float* conv_state = nullptr;
  float* rec_state = nullptr;
  void* k_cache = nullptr;
  void* v_cache = nullptr;
  int* page_table = nullptr;
  // steering / capture
  evie_op* ops = nullptr;      // [slots][kMaxOps]
  int* op_range = nullptr;     // [slots][L][2]
  int* op_gate = nullptr;      // [slots][kMaxOps]
  evie::GateSpec* gates = nullptr;  // [slots][kMaxGates]
  int* n_gates = nullptr;           // [slots]
  evie::DetSpec* dets = nullptr;    // [slots][kMaxDets]
  int* det_range = nullptr;         // [slots][L][2]
  int* gate_open = nullptr;         // [slots][kMaxGates]
  float* gate_score = nullptr;      // [slots][kMaxGates]
  int* gate_from = nullptr;         // [slots][kMaxGates]
  float* gate_partial = nullptr;    // [max_rows][kMaxGates]
  std::vector<int> h_n_gates;                // [slots]
  std::vector<std::vector<char>> h_gate_layers;  // per slot: layers that hold a detector or a gate decision
  std::vector<char> gate_layers;             // [L]: some slot's plan needs the detector kernel at this layer
  // sampling (sampling.rs:21-93): per-slot parameters and generator state, bitmap of every token fed since reset
  evie::SamplerParams* samp = nullptr;  // [slots]
  uint64_t* samp_rng = nullptr;         // [slots]
  uint32_t* seen = nullptr;             // [slots][seen_words]
  int seen_words = 0;
  std::vector<char> h_samp_on;          // [slots]: not plain greedy
  bool samp_active = false;             // some slot is not plain greedy: the sampler kernel follows the argmax
  float* scale = nullptr;      // [L][n]
  uint32_t* maxbuf = nullptr;  // [L][n]
  bool track = false;
  // activations
  float* x = nullptr;
  __nv_bfloat16* X2 = nullptr;
  float* Y2 = nullptr;
  size_t y2_cols = 0;  // Y2 holds 2 * max_rows rows of y2_cols floats
  bool pdl = true;     // projection GEMMs use programmatic dependent launch (EVIE_NO_PDL=1 at creation: off)
  int max_planes = evie::YView::kMaxPlanes;  // K slices per projection at most (EVIE_GEMM_PLANES=1..16 at creation)
  size_t y2_cap() const { return (size_t)2 * max_rows * y2_cols; }
  bool attn_rowwise = false;  // EVIE_ATTN_ROWWISE=1 at creation: prefill rows use the per-row split-KV kernel too
  bool attn_prefill_mma = false;  // EVIE_ATTN_PREFILL_MMA=1 at creation: prefill attention on the mma.sync kernel
  bool gdn_seq = false;  // EVIE_GDN_SEQ=1 at creation: prefill DeltaNet on the token-sequential CUDA-core kernel
  bool no_graph = false;      // EVIE_NO_GRAPH=1 at creation: decode-shaped calls run eagerly
  // Captured decode-shaped forward calls, keyed by (sequences, want logits, head, capture, tracking, context bound).
  // The host capture destinations are part of the key: their copies are nodes of the graph.
  std::map<std::tuple<int, int, int, int, int, int, uintptr_t, uintptr_t>, cudaGraphExec_t> fwd_graphs;
  // Captured decode-loop steps, keyed by (sequences, capture, tracking, context bound).
  std::map<std::tuple<int, int, int, int>, cudaGraphExec_t> dec_graphs;
  float* act = nullptr;
  float* q_rot = nullptr;
  int8_t* frames = nullptr;
  int cap_rows = 0;             // rows the last capturing call left in `frames`
  int32_t* topk = nullptr;      // [max_rows][100] scratch of evie_read_top_active
  uint16_t* resid = nullptr;
  float* L2 = nullptr;
  float* logits = nullptr;
  unsigned long long* best = nullptr;
  uint32_t* next = nullptr;
  void* attn_scratch = nullptr;
  RowInfo* d_rows = nullptr;
  SegInfo* d_segs = nullptr;
  RowInfo* h_rows = nullptr;  // pinned
  SegInfo* h_segs = nullptr;  // pinned
  unsigned int* timeouts = nullptr;    // this device's give-up counter (tc.h)
  unsigned int* h_timeouts = nullptr;  // pinned copy, read after each call's synchronisation
  uint32_t* hist = nullptr;   // device token history of evie_decode_greedy
  size_t hist_cap = 0;
  // profiling: event pairs per kernel group, resolved after each synchronising call
  bool prof = false;
  std::vector<std::pair<int, std::pair<cudaEvent_t, cudaEvent_t>>> prof_pending;
  std::vector<cudaEvent_t> prof_free;
  double prof_ms[P_COUNT] = {0};
  int64_t prof_n[P_COUNT] = {0};
  bool prof_failed = false;  // an event could not be created, recorded or timed
  cudaEvent_t prof_event() {
    if (!prof_free.empty()) {
      cudaEvent_t e = prof_free.back();
      prof_free.pop_back();
      return e;
    }
    cudaEvent_t e = nullptr;
    if (cudaEventCreate(&e) != cudaSuccess) {
      cudaGetLastError();
      prof_failed = true;
      return nullptr;
    }
    return e;
  }
  // Creates events ahead of a stream capture, so that none is created while capturing.
  void prof_reserve(size_t n) {
    while (prof_free.size() < n) {
      cudaEvent_t e = nullptr;
      if (cudaEventCreate(&e) != cudaSuccess) {
        cudaGetLastError();
        prof_failed = true;
        return;
      }
      prof_free.push_back(e);
    }
  }
  std::string err;

  template <typename T>
  evie_status alloc(T** p, size_t count, bool zero = true) {
    void* q = nullptr;
    if (cudaMalloc(&q, std::max<size_t>(count * sizeof(T), 16)) != cudaSuccess) {
      cudaGetLastError();
      return evie::fail(EVIE_ERR_OOM, "cannot allocate %zu bytes on device %d", count * sizeof(T), device);
    }
    allocs.push_back(q);
    if (zero) EVIE_CUDA_TRY(cudaMemset(q, 0, std::max<size_t>(count * sizeof(T), 16)));
    *p = (T*)q;
    return EVIE_OK;
  }
};

namespace {

// Records a profiling event on the context's stream. Inside a stream capture the record becomes an event-record
// node of the graph (cudaEventRecordExternal), so the replayed graph timestamps the group where it runs.
void prof_record(evie_ctx* c, cudaEvent_t e) {
  if (!e) return;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  cudaError_t rc = cudaStreamIsCapturing(c->stream, &cs);
  if (rc == cudaSuccess)
    rc = cs == cudaStreamCaptureStatusActive ? cudaEventRecordWithFlags(e, c->stream, cudaEventRecordExternal)
                                             : cudaEventRecord(e, c->stream);
  if (rc != cudaSuccess) {
    cudaGetLastError();
    c->prof_failed = true;
  }
}

// Brackets one kernel group with CUDA events on the context's stream when profiling is on.
struct ProfScope {
  evie_ctx* c;
  int cat;
  cudaEvent_t a = nullptr;
  ProfScope(evie_ctx* c_, int cat_) : c(c_), cat(cat_) {
    if (c->prof) {
      a = c->prof_event();
      prof_record(c, a);
    }
  }
  ~ProfScope() {
    if (c->prof) {
      cudaEvent_t b = c->prof_event();
      prof_record(c, b);
      if (a && b) {
        c->prof_pending.push_back({cat, {a, b}});
      } else {  // one of the pair could not be created: return the other to the pool
        if (a) c->prof_free.push_back(a);
        if (b) c->prof_free.push_back(b);
      }
    }
  }
};

void prof_resolve(evie_ctx* c) {
  for (auto& p : c->prof_pending) {
    float ms = 0.f;
    if (cudaEventElapsedTime(&ms, p.second.first, p.second.second) == cudaSuccess) {
      c->prof_ms[p.first] += ms;
      c->prof_n[p.first] += 1;
    } else {
      cudaGetLastError();
      c->prof_failed = true;
    }
    c->prof_free.push_back(p.second.first);
    c->prof_free.push_back(p.second.second);
  }
  c->prof_pending.clear();
}

#define PROF(cat) ProfScope prof_scope_##__LINE__(c, cat)

#define TRY(expr)                        \
  do {                                   \
    evie_status rc_ = (expr);            \
    if (rc_ != EVIE_OK) return rc_;      \
  } while (0)

evie_status upload_f32(evie_ctx* c, const SafeTensors& st, const std::string& name, size_t expect, float** out,
                       float add = 0.0f, bool neg_exp = false) {
  const Tensor* t = st.get(name);
  if (!t) return evie::fail(EVIE_ERR_IO, "missing tensor %s", name.c_str());
  std::vector<float> v;
  if (t->dtype == "F32") {
    v.resize(t->bytes / 4);
    memcpy(v.data(), t->data, t->bytes);
  } else if (t->dtype == "BF16" || t->dtype == "F16") {
    v.resize(t->bytes / 2);
    for (size_t i = 0; i < v.size(); i++) {
      uint16_t b;
      memcpy(&b, t->data + 2 * i, 2);
      v[i] = t->dtype == "BF16" ? bf16_bits_to_f32(b) : half_bits_to_f32(b);
    }
  } else {
    return evie::fail(EVIE_ERR_IO, "%s: unsupported dtype %s", name.c_str(), t->dtype.c_str());
  }
  if (v.size() != expect) return evie::fail(EVIE_ERR_IO, "%s: %zu values, expected %zu", name.c_str(), v.size(), expect);
  for (auto& x : v) {
    x = x + add;
    if (neg_exp) x = -expf(x);  // model.rs:171: A_log -> -exp(A_log)
  }
  TRY(c->alloc(out, v.size(), false));
  EVIE_CUDA_TRY(cudaMemcpy(*out, v.data(), v.size() * 4, cudaMemcpyHostToDevice));
  c->weight_bytes += v.size() * 4;
  return EVIE_OK;
}

// Concatenates bf16 matrices row-wise into one device matrix of `cols` columns.
evie_status upload_rows(evie_ctx* c, const SafeTensors& st, const std::vector<std::pair<std::string, int64_t>>& parts,
                        int64_t cols, __nv_bfloat16** out) {
  int64_t rows = 0;
  for (auto& p : parts) rows += p.second;
  TRY(c->alloc(out, (size_t)rows * cols, false));
  int64_t r0 = 0;
  for (auto& p : parts) {
    const Tensor* t = st.get(p.first);
    if (!t) return evie::fail(EVIE_ERR_IO, "missing tensor %s", p.first.c_str());
    if (t->dtype != "BF16") return evie::fail(EVIE_ERR_IO, "%s: expected BF16, got %s", p.first.c_str(), t->dtype.c_str());
    if ((int64_t)t->bytes != p.second * cols * 2)
      return evie::fail(EVIE_ERR_IO, "%s: size %zu does not match %lld x %lld", p.first.c_str(), t->bytes,
                        (long long)p.second, (long long)cols);
    EVIE_CUDA_TRY(cudaMemcpy(*out + r0 * cols, t->data, t->bytes, cudaMemcpyHostToDevice));
    r0 += p.second;
  }
  c->weight_bytes += (size_t)rows * cols * 2;
  return EVIE_OK;
}

evie_status read_config(evie_ctx* c, const std::string& dir) {
  std::ifstream f(dir + "/config.json");
  if (!f) return evie::fail(EVIE_ERR_IO, "cannot read %s/config.json", dir.c_str());
  std::stringstream ss;
  ss << f.rdbuf();
  try {
    evie::json::Value root = evie::json::parse(ss.str());
    const evie::json::Value& t = root.has("text_config") ? root["text_config"] : root;  // config.rs:82
    auto I = [&](const char* k) {
      if (!t.has(k)) throw std::runtime_error(std::string("missing ") + k);
      return (int)t[k].integer();
    };
    auto& s = c->s;
    s.d = I("hidden_size");
    s.n = I("intermediate_size");
    s.L = I("num_hidden_layers");
    s.V = I("vocab_size");
    s.eps = (float)t["rms_norm_eps"].number();
    s.nh = I("num_attention_heads");
    s.nkv = I("num_key_value_heads");
    s.hd = I("head_dim");
    s.K = I("linear_conv_kernel_dim");
    s.dk = I("linear_key_head_dim");
    s.hk = I("linear_num_key_heads");
    s.hv = I("linear_num_value_heads");
    s.dv = I("linear_value_head_dim");
    double theta = 10000000.0, partial = 1.0;  // config.rs:85-88
    if (t.has("rope_parameters")) {
      theta = t["rope_parameters"]["rope_theta"].number();
      if (t["rope_parameters"].has("partial_rotary_factor")) partial = t["rope_parameters"]["partial_rotary_factor"].number();
    } else {
      if (t.has("rope_theta")) theta = t["rope_theta"].number();
      if (t.has("partial_rotary_factor")) partial = t["partial_rotary_factor"].number();
    }
    s.rot = (int)std::round(s.hd * partial);  // config.rs:116
    for (auto& lt : t["layer_types"].arr) {
      if (lt.string() == "linear_attention") c->kinds.push_back(0);
      else if (lt.string() == "full_attention") c->kinds.push_back(1);
      else throw std::runtime_error("unsupported layer type " + lt.string());
    }
    if ((int)c->kinds.size() != s.L) throw std::runtime_error("layer_types does not match num_hidden_layers");
    s.conv_dim = 2 * s.hk * s.dk + s.hv * s.dv;  // config.rs:144-146
    s.vd = s.hv * s.dv;
    s.key_dim = s.hk * s.dk;
    s.in_dn = s.conv_dim + s.vd + 2 * s.hv;
    s.in_at = (2 * s.nh + 2 * s.nkv) * s.hd;
    std::vector<float> inv(s.rot / 2);
    for (int i = 0; i < s.rot / 2; i++) inv[i] = 1.0f / powf((float)theta, (float)(2 * i) / (float)s.rot);  // model.rs:198-201
    TRY(c->alloc(&c->inv_freq, inv.size() + 1, false));
    EVIE_CUDA_TRY(cudaMemcpy(c->inv_freq, inv.data(), inv.size() * 4, cudaMemcpyHostToDevice));
  } catch (std::exception& e) {
    return evie::fail(EVIE_ERR_IO, "config.json: %s", e.what());
  }
  // Limits of these kernels (gpu/mod.rs:267-269 states the same shape limits for the wgpu backend).
  auto& s = c->s;
  if (s.dk != 128 || s.dv != 128) return evie::fail(EVIE_ERR_ARG, "DeltaNet heads must be 128 wide");
  if (s.hd != 256) return evie::fail(EVIE_ERR_ARG, "attention head_dim must be 256");
  if (s.rot > s.hd || s.rot % 2) return evie::fail(EVIE_ERR_ARG, "bad rotary dim %d", s.rot);
  if (s.nh % s.nkv || (s.nh / s.nkv != 2 && s.nh / s.nkv != 4)) return evie::fail(EVIE_ERR_ARG, "GQA group must be 2 or 4");
  if (s.hv % s.hk) return evie::fail(EVIE_ERR_ARG, "value heads must be a multiple of key heads");
  if (s.K < 1 || s.K > 16) return evie::fail(EVIE_ERR_ARG, "conv kernel %d out of range", s.K);
  if (s.d % 4 || s.d > 8192 || s.n % 4)
    return evie::fail(EVIE_ERR_ARG, "hidden and MLP sizes must be multiples of 4 (hidden <= 8192)");
  return EVIE_OK;
}

evie_status load_weights(evie_ctx* c, const std::string& dir) {
  SafeTensors st;
  std::string e = st.open_dir(dir);
  if (!e.empty()) return evie::fail(EVIE_ERR_IO, "%s", e.c_str());
  std::string p;  // model.rs:140-146
  if (st.get("model.language_model.embed_tokens.weight")) p = "model.language_model.";
  else if (st.get("model.embed_tokens.weight")) p = "model.";
  else return evie::fail(EVIE_ERR_IO, "unrecognised checkpoint layout in %s", dir.c_str());
  auto& s = c->s;
  const Tensor* emb = st.get(p + "embed_tokens.weight");
  if (emb->shape.size() != 2 || emb->shape[0] < s.V || emb->shape[1] != s.d)
    return evie::fail(EVIE_ERR_IO, "embedding shape does not match config");
  s.V = (int)emb->shape[0];  // the LM head has as many rows as the embedding (model.rs:279)
  TRY(upload_rows(c, st, {{p + "embed_tokens.weight", s.V}}, s.d, &c->embed));
  c->lm_head = c->embed;
  {
    // config.rs:101-104 + model.rs:151: a separate lm_head only when present and embeddings are not tied
    std::ifstream f(dir + "/config.json");
    std::stringstream ss;
    ss << f.rdbuf();
    evie::json::Value root = evie::json::parse(ss.str());
    const evie::json::Value& t = root.has("text_config") ? root["text_config"] : root;
    bool tie = false;
    if (t["tie_word_embeddings"].kind == evie::json::Value::Bool) tie = t["tie_word_embeddings"].b;
    else if (root["tie_word_embeddings"].kind == evie::json::Value::Bool) tie = root["tie_word_embeddings"].b;
    if (st.get("lm_head.weight") && !tie) TRY(upload_rows(c, st, {{"lm_head.weight", s.V}}, s.d, &c->lm_head));
  }
  c->layers.resize(s.L);
  for (int i = 0; i < s.L; i++) {
    Layer& L = c->layers[i];
    const std::string l = p + "layers." + std::to_string(i) + ".";
    L.kind = c->kinds[i];
    L.idx = L.kind == 0 ? c->n_lin++ : c->n_full++;
    TRY(upload_f32(c, st, l + "input_layernorm.weight", s.d, &L.ln1, 1.0f));
    TRY(upload_f32(c, st, l + "post_attention_layernorm.weight", s.d, &L.ln2, 1.0f));
    if (L.kind == 0) {
      const std::string a = l + "linear_attn.";
      TRY(upload_rows(c, st,
                      {{a + "in_proj_qkv.weight", s.conv_dim}, {a + "in_proj_z.weight", s.vd},
                       {a + "in_proj_b.weight", s.hv}, {a + "in_proj_a.weight", s.hv}},
                      s.d, &L.w_in));
      TRY(upload_rows(c, st, {{a + "out_proj.weight", s.d}}, s.vd, &L.w_out));
      TRY(upload_f32(c, st, a + "conv1d.weight", (size_t)s.conv_dim * s.K, &L.conv));
      TRY(upload_f32(c, st, a + "A_log", s.hv, &L.neg_a, 0.0f, true));
      TRY(upload_f32(c, st, a + "dt_bias", s.hv, &L.dt_bias));
      TRY(upload_f32(c, st, a + "norm.weight", s.dv, &L.norm));  // gated norm gain used as is (model.rs:173)
    } else {
      const std::string a = l + "self_attn.";
      TRY(upload_rows(c, st,
                      {{a + "q_proj.weight", 2 * s.nh * s.hd}, {a + "k_proj.weight", s.nkv * s.hd},
                       {a + "v_proj.weight", s.nkv * s.hd}},
                      s.d, &L.w_in));
      TRY(upload_rows(c, st, {{a + "o_proj.weight", s.d}}, s.nh * s.hd, &L.w_out));
      TRY(upload_f32(c, st, a + "q_norm.weight", s.hd, &L.q_norm, 1.0f));
      TRY(upload_f32(c, st, a + "k_norm.weight", s.hd, &L.k_norm, 1.0f));
    }
    TRY(upload_rows(c, st, {{l + "mlp.gate_proj.weight", s.n}, {l + "mlp.up_proj.weight", s.n}}, s.d, &L.w_gu));
    TRY(upload_rows(c, st, {{l + "mlp.down_proj.weight", s.d}}, s.n, &L.w_down));
  }
  TRY(upload_f32(c, st, p + "norm.weight", s.d, &c->final_norm, 1.0f));
  return EVIE_OK;
}

evie_status allocate_state(evie_ctx* c) {
  auto& s = c->s;
  const size_t S = c->slots, R = c->max_rows;
  c->pages_per_slot = (c->max_ctx + kPage - 1) / kPage;
  const size_t kv_elems = (size_t)std::max(c->n_full, 1) * S * c->pages_per_slot * s.nkv * kPage * s.hd;
  TRY(c->alloc(&c->conv_state, S * std::max(c->n_lin, 1) * (s.K - 1) * s.conv_dim + 1));
  TRY(c->alloc(&c->rec_state, S * std::max(c->n_lin, 1) * (size_t)s.hv * s.dk * s.dv));
  if (c->kv_f32) {
    float *k, *v;
    TRY(c->alloc(&k, kv_elems, false));
    TRY(c->alloc(&v, kv_elems, false));
    c->k_cache = k;
    c->v_cache = v;
  } else {
    __nv_bfloat16 *k, *v;
    TRY(c->alloc(&k, kv_elems, false));
    TRY(c->alloc(&v, kv_elems, false));
    c->k_cache = k;
    c->v_cache = v;
  }
  c->cache_bytes = (S * std::max(c->n_lin, 1) * ((s.K - 1) * (size_t)s.conv_dim + (size_t)s.hv * s.dk * s.dv)) * 4 +
                   2 * kv_elems * (c->kv_f32 ? 4 : 2);
  std::vector<int> pt(S * c->pages_per_slot);
  for (size_t i = 0; i < pt.size(); i++) pt[i] = (int)i;
  TRY(c->alloc(&c->page_table, pt.size()));
  EVIE_CUDA_TRY(cudaMemcpy(c->page_table, pt.data(), pt.size() * 4, cudaMemcpyHostToDevice));
  TRY(c->alloc(&c->ops, S * kMaxOps));
  TRY(c->alloc(&c->op_range, S * s.L * 2));
  TRY(c->alloc(&c->op_gate, S * kMaxOps));
  TRY(c->alloc(&c->gates, S * kMaxGates));
  TRY(c->alloc(&c->n_gates, S));
  TRY(c->alloc(&c->dets, S * kMaxDets));
  TRY(c->alloc(&c->det_range, S * s.L * 2));
  TRY(c->alloc(&c->gate_open, S * kMaxGates));
  TRY(c->alloc(&c->gate_score, S * kMaxGates));
  TRY(c->alloc(&c->gate_from, S * kMaxGates));
  TRY(c->alloc(&c->gate_partial, R * kMaxGates));
  c->h_n_gates.assign(S, 0);
  c->seen_words = (s.V + 31) / 32;
  TRY(c->alloc(&c->samp, S));
  TRY(c->alloc(&c->samp_rng, S));
  TRY(c->alloc(&c->seen, S * c->seen_words));
  {
    std::vector<evie::SamplerParams> dflt(S, evie::SamplerParams{0.0f, 1.0f, 0.0f, 1.0f});  // SampleParams::default
    EVIE_CUDA_TRY(cudaMemcpy(c->samp, dflt.data(), S * sizeof(evie::SamplerParams), cudaMemcpyHostToDevice));
    std::vector<uint64_t> rng(S, evie::sampler_seed_state(0));
    EVIE_CUDA_TRY(cudaMemcpy(c->samp_rng, rng.data(), S * 8, cudaMemcpyHostToDevice));
  }
  c->h_samp_on.assign(S, 0);
  c->cap_ev.assign(s.L + 1, nullptr);
  for (auto& e : c->cap_ev) EVIE_CUDA_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  c->h_gate_layers.assign(S, std::vector<char>(s.L, 0));
  c->gate_layers.assign(s.L, 0);
  TRY(c->alloc(&c->scale, (size_t)s.L * s.n, false));
  {
    std::vector<float> one((size_t)s.L * s.n, 1.0f);  // gpu/mod.rs:367: scales start at 1
    EVIE_CUDA_TRY(cudaMemcpy(c->scale, one.data(), one.size() * 4, cudaMemcpyHostToDevice));
  }
  TRY(c->alloc(&c->maxbuf, (size_t)s.L * s.n));
  const size_t kmax = std::max({(size_t)s.d, (size_t)s.vd, (size_t)s.nh * s.hd, (size_t)s.n});
  const size_t mmax = std::max({(size_t)s.in_dn, (size_t)s.in_at, (size_t)2 * s.n, (size_t)s.d});
  TRY(c->alloc(&c->x, R * s.d));
  TRY(c->alloc(&c->X2, 2 * R * kmax));
  TRY(c->alloc(&c->Y2, 2 * R * mmax));
  c->y2_cols = mmax;
  if (const char* e = getenv("EVIE_NO_PDL")) c->pdl = e[0] != '1';
  if (const char* e = getenv("EVIE_GEMM_PLANES")) c->max_planes = std::min(evie::YView::kMaxPlanes, std::max(1, atoi(e)));
  if (const char* e = getenv("EVIE_ATTN_ROWWISE")) c->attn_rowwise = e[0] == '1';
  if (const char* e = getenv("EVIE_ATTN_PREFILL_MMA")) c->attn_prefill_mma = e[0] == '1';
  if (const char* e = getenv("EVIE_GDN_SEQ")) c->gdn_seq = e[0] == '1';
  if (const char* e = getenv("EVIE_NO_GRAPH")) c->no_graph = e[0] == '1';
  TRY(c->alloc(&c->act, R * s.conv_dim));
  TRY(c->alloc(&c->q_rot, R * s.nh * s.hd));
  TRY(c->alloc(&c->frames, R * s.L * (size_t)s.n, false));
  TRY(c->alloc(&c->topk, R * 100, false));
  TRY(c->alloc(&c->resid, R * s.L * (size_t)s.d, false));
  TRY(c->alloc(&c->L2, 2 * S * (size_t)s.V, false));
  TRY(c->alloc(&c->logits, S * (size_t)s.V, false));
  TRY(c->alloc(&c->best, S));
  TRY(c->alloc(&c->next, S));
  {
    char* p = nullptr;
    TRY(c->alloc(&p, evie::gqa_scratch_bytes((int)R, s.nkv, s.nh / s.nkv, c->pages_per_slot * kPage)));
    c->attn_scratch = p;
  }
  TRY(c->alloc(&c->d_rows, R));
  TRY(c->alloc(&c->d_segs, S));
  EVIE_CUDA_TRY(cudaMallocHost(&c->h_rows, R * sizeof(RowInfo)));
  EVIE_CUDA_TRY(cudaMallocHost(&c->h_segs, S * sizeof(SegInfo)));
  EVIE_CUDA_TRY(cudaMallocHost(&c->h_timeouts, sizeof(unsigned int)));
  *c->h_timeouts = 0;
  return EVIE_OK;
}

// Y = X . W^T for the R rows of the split operand X2 ([2][R][K] bf16) on the tcgen05 projection GEMM (proj_gemm.cu):
// the hi and lo products accumulate in one f32 accumulator, so each K slice leaves one plane; decode-shaped calls cut
// K into as many slices as fill the SMs, and the consumer adds the planes in slice order (the split-K reduction).
// `cap` is the number of floats at Y2. Launched with programmatic stream serialisation (unless EVIE_NO_PDL=1), so
// that its first weight tiles stream while the previous kernel finishes.
evie_status gemm(evie_ctx* c, const __nv_bfloat16* W, int M, int K, const __nv_bfloat16* X2, int R, float* Y2,
                 size_t cap, evie::YView* out) {
  int planes = 0;
  TRY(evie::launch_proj_gemm(W, M, K, X2, R, Y2, cap, c->max_planes, c->pdl, c->stream, &planes));
  *out = evie::YView{Y2, (size_t)R * M, planes};
  return EVIE_OK;
}

// gpu/mod.rs:616-634: limits, then the row and segment tables uploaded for the kernels.
evie_status upload_rows(evie_ctx* c, int R, int nseq) {
  EVIE_CUDA_TRY(cudaMemcpyAsync(c->d_rows, c->h_rows, R * sizeof(RowInfo), cudaMemcpyHostToDevice, c->stream));
  EVIE_CUDA_TRY(cudaMemcpyAsync(c->d_segs, c->h_segs, nseq * sizeof(SegInfo), cudaMemcpyHostToDevice, c->stream));
  return EVIE_OK;
}

evie_status prepare_rows(evie_ctx* c, const evie_seq* seqs, int nseq, int* R_out, int* max_ctx_out,
                         bool upload = true) {
  auto& s = c->s;
  EVIE_ARG(nseq >= 1 && nseq <= c->slots, "forward: 1..=%d sequences per call, got %d", c->slots, nseq);
  int R = 0, max_ctx_rows = 0;
  std::vector<char> used(c->slots, 0);
  for (int i = 0; i < nseq; i++) {
    const evie_seq& q = seqs[i];
    EVIE_ARG(q.slot >= 0 && q.slot < c->slots, "forward: bad slot %d", q.slot);
    EVIE_ARG(!used[q.slot], "forward: slot %d appears twice", q.slot);
    used[q.slot] = 1;
    EVIE_ARG(q.n_tokens >= 1 && q.tokens, "forward: sequence %d has no tokens", i);
    EVIE_ARG(q.pos0 >= 0 && (long)q.pos0 + q.n_tokens <= c->max_ctx, "forward: context longer than %d tokens", c->max_ctx);
    R += q.n_tokens;
    EVIE_ARG(R <= c->max_rows, "forward: needs 1..=%d rows, got more", c->max_rows);
    max_ctx_rows = std::max(max_ctx_rows, q.pos0 + q.n_tokens);
  }
  int r = 0;
  for (int i = 0; i < nseq; i++) {
    const evie_seq& q = seqs[i];
    c->h_segs[i] = SegInfo{q.slot, r, q.n_tokens, q.pos0};
    for (int t = 0; t < q.n_tokens; t++) {
      EVIE_ARG(q.tokens[t] < (uint32_t)s.V, "forward: token id %u out of range", q.tokens[t]);
      c->h_rows[r++] = RowInfo{q.slot, q.pos0 + t, (int)q.tokens[t], i};
    }
  }
  if (upload) TRY(upload_rows(c, R, nseq));
  *R_out = R;
  *max_ctx_out = max_ctx_rows;
  return EVIE_OK;
}

// model.rs:230-267: embedding, every layer, and the final norm of each sequence's last row (into X2).
// Page-locked host destinations of a call's captures ([R][L][n] i8 frames, [R][L][d] f16 residual rows).
struct CapHost {
  int8_t* frames;
  uint16_t* resid;
};

// True when [p, p + bytes) lies in page-locked (pinned or registered) host memory, so copies into it can run
// asynchronously on a second stream.
bool page_locked(const void* p, size_t bytes) {
  if (!p || !bytes) return false;
  for (const char* q : {(const char*)p, (const char*)p + bytes - 1}) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, q) != cudaSuccess) {
      cudaGetLastError();
      return false;
    }
    if (a.type != cudaMemoryTypeHost) return false;
  }
  return true;
}

evie_status enqueue_layers(evie_ctx* c, int R, int nseq, int max_ctx_rows, int capture, const CapHost* ch = nullptr) {
  auto& s = c->s;
  cudaStream_t st = c->stream;
  int8_t* fr = capture ? c->frames : nullptr;
  uint16_t* rs = capture ? c->resid : nullptr;
  const size_t cs_slot = (size_t)std::max(c->n_lin, 1) * (s.K - 1) * s.conv_dim;
  const size_t rs_slot = (size_t)std::max(c->n_lin, 1) * s.hv * s.dk * s.dv;
  const size_t kv_layer = (size_t)c->slots * c->pages_per_slot * s.nkv * kPage * s.hd;
  evie::SteerTables steer{c->ops, c->op_range, kMaxOps, c->op_gate, c->gates, c->gate_open, c->gate_from, kMaxGates};
  const evie::GateTables gt{c->gates,    c->n_gates,    c->dets,      c->det_range, kMaxGates,
                            kMaxDets,    c->gate_open,  c->gate_score, c->gate_from, c->gate_partial};

  {
    PROF(P_NORM);
    TRY(evie::k_embed_norm(c->d_rows, R, c->embed, c->x, c->layers[0].ln1, s.eps, s.d, c->X2, c->seen,
                           c->seen_words, st));
  }
  for (int li = 0; li < s.L; li++) {
    Layer& L = c->layers[li];
    evie::YView yo;  // output projection of the mixer
    if (L.kind == 0) {
      evie::YView y;
      { PROF(P_GEMM_LIN_IN); TRY(gemm(c, L.w_in, s.in_dn, s.d, c->X2, R, c->Y2, c->y2_cap(), &y)); }
      float* cs = c->conv_state + (size_t)L.idx * (s.K - 1) * s.conv_dim;
      const bool single_rows = R == nseq && s.K <= 8;  // decode: one row per segment, the conv kernel shifts the window
      int max_seg_rows = 1;
      if (!single_rows)
        for (int i = 0; i < nseq; i++) max_seg_rows = std::max(max_seg_rows, c->h_segs[i].count);
      // Prefill calls run the recurrence chunked on tensor cores (gdn_chunk.cu); the conv then writes q and k as
      // split bf16 planes, the chunk kernel's operand format.
      const bool chunked = !c->gdn_seq && max_seg_rows > 1 && s.K == 4 && s.dk == 128 && s.dv == 128;
      {
        PROF(P_CONV);
        TRY(evie::k_conv_silu_norm(y, s.in_dn, R, c->d_rows, c->d_segs, cs, cs_slot, L.conv, s, c->act, st,
                                   single_rows, nseq, max_seg_rows, chunked));
        if (!single_rows) TRY(evie::k_conv_state_update(y, s.in_dn, R, c->d_segs, nseq, cs, cs_slot, s, st));
      }
      float* rsb = c->rec_state + (size_t)L.idx * s.hv * s.dk * s.dv;
      {
        PROF(P_MIXER);
        if (chunked) {
          TRY(evie::launch_gdn_chunk_model(c->act, y, s.in_dn, R, c->d_segs, nseq, rsb, rs_slot, L.neg_a,
                                           L.dt_bias, s.conv_dim, s.key_dim, s.vd, s.hv, s.hk, st));
          TRY(evie::k_gdn_gated_norm(c->act, y, s.in_dn, R, L.norm, s, c->X2, st));
        } else {
          TRY(evie::k_gdn_mixer(c->act, y, s.in_dn, R, c->d_segs, nseq, rsb, rs_slot, L.neg_a, L.dt_bias, L.norm,
                                s, c->X2, st));
        }
      }
      { PROF(P_GEMM_LIN_OUT); TRY(gemm(c, L.w_out, s.d, s.vd, c->X2, R, c->Y2, c->y2_cap(), &yo)); }
    } else {
      evie::YView y;
      { PROF(P_GEMM_ATT_IN); TRY(gemm(c, L.w_in, s.in_at, s.d, c->X2, R, c->Y2, c->y2_cap(), &y)); }
      const float scale = 1.0f / sqrtf((float)s.hd);
      if (c->kv_f32) {
        float* kc = (float*)c->k_cache + (size_t)L.idx * kv_layer;
        float* vc = (float*)c->v_cache + (size_t)L.idx * kv_layer;
        {
          PROF(P_ATTN_PREP);
          TRY(evie::k_attn_prep<float>(y, s.in_at, R, c->d_rows, L.q_norm, L.k_norm, c->inv_freq, s, c->q_rot,
                                       kc, vc, c->page_table, c->pages_per_slot, kPage, st));
        }
        PROF(P_ATTN);
        TRY(evie::launch_gqa_model<float>(c->q_rot, y, s.in_at, c->X2,
                                          (size_t)R * s.nh * s.hd, c->d_rows, R, c->page_table, c->pages_per_slot,
                                          kc, vc, s.nh, s.nkv, kPage, max_ctx_rows, scale, c->attn_scratch, c->max_rows,
                                          st));
      } else {
        auto* kc = (__nv_bfloat16*)c->k_cache + (size_t)L.idx * kv_layer;
        auto* vc = (__nv_bfloat16*)c->v_cache + (size_t)L.idx * kv_layer;
        {
          PROF(P_ATTN_PREP);
          TRY(evie::k_attn_prep<__nv_bfloat16>(y, s.in_at, R, c->d_rows, L.q_norm, L.k_norm, c->inv_freq, s,
                                               c->q_rot, kc, vc, c->page_table, c->pages_per_slot, kPage, st));
        }
        PROF(P_ATTN);
        if (R > nseq && !c->attn_rowwise && s.nh == 4 * s.nkv) {
          // prefill: blocks of 16 rows of a segment share every K/V tile (gqa_prefill.cu)
          int max_seg_rows = 0;
          for (int i = 0; i < nseq; i++) max_seg_rows = std::max(max_seg_rows, c->h_segs[i].count);
          if (c->attn_prefill_mma)
            TRY(evie::launch_gqa_prefill_model(c->q_rot, y, s.in_at, c->X2, (size_t)R * s.nh * s.hd, c->d_rows,
                                               c->d_segs, nseq, max_seg_rows, c->page_table, c->pages_per_slot, kc,
                                               vc, s.nh, s.nkv, kPage, scale, st));
          else
            TRY(evie::launch_gqa_prefill_tc_model(c->q_rot, y, s.in_at, c->X2, (size_t)R * s.nh * s.hd, c->d_segs,
                                                  nseq, max_seg_rows, c->page_table, c->pages_per_slot, kc, vc,
                                                  (long)c->slots * c->pages_per_slot * s.nkv * kPage, s.nh, s.nkv,
                                                  kPage, scale, st));
        } else {
          TRY(evie::launch_gqa_model<__nv_bfloat16>(c->q_rot, y, s.in_at, c->X2,
                                                    (size_t)R * s.nh * s.hd, c->d_rows, R, c->page_table,
                                                    c->pages_per_slot, kc, vc, s.nh, s.nkv, kPage, max_ctx_rows,
                                                    scale, c->attn_scratch, c->max_rows, st));
        }
      }
      { PROF(P_GEMM_ATT_OUT); TRY(gemm(c, L.w_out, s.d, s.nh * s.hd, c->X2, R, c->Y2, c->y2_cap(), &yo)); }
    }
    // model.rs:246-248: residual add after the mixer, then the pre-MLP norm
    { PROF(P_NORM); TRY(evie::k_add_norm(c->x, yo, s.d, R, L.ln2, s.eps, s.d, c->X2, nullptr, 0, s.L, st)); }
    evie::YView yg, yd;
    { PROF(P_GEMM_GATE_UP); TRY(gemm(c, L.w_gu, 2 * s.n, s.d, c->X2, R, c->Y2, c->y2_cap(), &yg)); }
    {
      PROF(P_SWIGLU);
      if (c->gate_layers[li]) TRY(evie::k_gate_detect(yg, 2 * s.n, c->d_segs, nseq, li, s, gt, st));
      TRY(evie::k_swiglu(yg, 2 * s.n, R, c->d_rows, li, s, steer, c->scale, fr, c->track ? c->maxbuf : nullptr,
                         c->X2, st));
    }
    { PROF(P_GEMM_DOWN); TRY(gemm(c, L.w_down, s.d, s.n, c->X2, R, c->Y2, c->y2_cap(), &yd)); }
    {
      PROF(P_NORM);
      if (li + 1 < s.L) {
        TRY(evie::k_add_norm(c->x, yd, s.d, R, c->layers[li + 1].ln1, s.eps, s.d, c->X2, rs, li, s.L, st));
      } else {
        TRY(evie::k_add_final(c->x, yd, s.d, R, c->d_rows, c->d_segs, nseq, c->final_norm, s.eps, s.d, c->X2, rs,
                              li, s.L, st));
      }
    }
    if (ch) {  // this layer's frames and residual rows are final: copy them out while later layers run
      EVIE_CUDA_TRY(cudaEventRecord(c->cap_ev[li], st));
      EVIE_CUDA_TRY(cudaStreamWaitEvent(c->cstream, c->cap_ev[li], 0));
      if (ch->frames)
        EVIE_CUDA_TRY(cudaMemcpy2DAsync(ch->frames + (size_t)li * s.n, (size_t)s.L * s.n, c->frames + (size_t)li * s.n,
                                        (size_t)s.L * s.n, s.n, R, cudaMemcpyDeviceToHost, c->cstream));
      if (ch->resid)
        EVIE_CUDA_TRY(cudaMemcpy2DAsync(ch->resid + (size_t)li * s.d, (size_t)s.L * s.d * 2,
                                        c->resid + (size_t)li * s.d, (size_t)s.L * s.d * 2, (size_t)s.d * 2, R,
                                        cudaMemcpyDeviceToHost, c->cstream));
    }
  }
  return EVIE_OK;
}

// Joins the capture copy stream back into the compute stream (after the head, which overlaps the last copies).
evie_status join_captures(evie_ctx* c) {
  EVIE_CUDA_TRY(cudaEventRecord(c->cap_ev[c->s.L], c->cstream));
  EVIE_CUDA_TRY(cudaStreamWaitEvent(c->stream, c->cap_ev[c->s.L], 0));
  return EVIE_OK;
}

// model.rs:271-283: LM head on the last row of every sequence; greedy id (sampling.rs:60-62) on device.
evie_status enqueue_head(evie_ctx* c, int nseq, bool want_logits) {
  evie::YView yl;
  { PROF(P_LMHEAD); TRY(gemm(c, c->lm_head, c->s.V, c->s.d, c->X2, nseq, c->L2, (size_t)2 * c->slots * c->s.V, &yl)); }
  PROF(P_OTHER);
  TRY(evie::k_logits_argmax(yl, nseq, c->s.V, want_logits ? c->logits : nullptr, c->best, c->next, c->stream));
  if (!c->samp_active) return EVIE_OK;
  // some slot samples (or penalises repeats): every sequence's token comes from its slot's sampler
  const evie::SampleArgs a{yl, c->s.V, c->d_segs, c->samp, c->samp_rng, c->seen, c->seen_words, nullptr, nullptr,
                           c->next};
  return evie::k_sample(a, nseq, c->stream);
}

// The device's count of bounded waits that gave up (tc.h) is copied to page-locked memory behind a call's work, so
// that the call can report a give-up among its own kernels with its status. The count is per device: a give-up in
// another kernel on the device since the last check (or evie_poll_device_errors) is reported here as well.
evie_status enqueue_timeout_read(evie_ctx* c) {
  if (!c->timeouts) {
    c->timeouts = evie::device_timeout_counter();
    if (!c->timeouts) return evie::fail(EVIE_ERR_CUDA, "device timeout counter unavailable");
  }
  EVIE_CUDA_TRY(cudaMemcpyAsync(c->h_timeouts, c->timeouts, sizeof(unsigned int), cudaMemcpyDeviceToHost, c->stream));
  return EVIE_OK;
}
// After the call's synchronisation: EVIE_ERR_TIMEOUT (and the count restarts) when a kernel gave up a wait.
evie_status check_timeouts(evie_ctx* c, const char* what) {
  const unsigned int n = *c->h_timeouts;
  if (!n) return EVIE_OK;
  *c->h_timeouts = 0;
  EVIE_CUDA_TRY(cudaMemsetAsync(c->timeouts, 0, sizeof(unsigned int), c->stream));
  EVIE_CUDA_TRY(cudaStreamSynchronize(c->stream));
  return evie::fail(EVIE_ERR_TIMEOUT, "%s: %u thread(s) gave up a bounded device-side wait; outputs are incomplete",
                    what, n);
}

evie_status forward_impl(evie_ctx* c, const evie_seq* seqs, int nseq, int want_logits, int capture, float* logits,
                         int8_t* frames, uint16_t* resid, uint32_t* next_tokens) {
  auto& s = c->s;
  int R = 0, max_ctx_rows = 0;
  TRY(prepare_rows(c, seqs, nseq, &R, &max_ctx_rows, false));
  cudaStream_t st = c->stream;
  const bool head = want_logits || next_tokens;
  // Captures into page-locked host buffers are copied layer by layer on the copy stream while later layers run;
  // other destinations get one copy at the end.
  CapHost chv{nullptr, nullptr};
  if (capture && !c->prof) {
    if (frames && page_locked(frames, (size_t)R * s.L * s.n)) chv.frames = frames;
    if (resid && page_locked(resid, (size_t)R * s.L * s.d * 2)) chv.resid = resid;
  }
  const CapHost* ch = (chv.frames || chv.resid) ? &chv : nullptr;
  if (R == nseq && !c->prof && !c->no_graph) {
    // Decode-shaped call (one token per sequence): replay a captured graph of (row-table upload, layers, head).
    // The tables are copied from the same pinned host arrays each replay; the attention's split count uses a
    // context bound rounded up to a multiple of 2048, so a graph serves every call until the context passes it.
    const int bound = std::min(c->max_ctx, (max_ctx_rows + 2047) / 2048 * 2048);
    const auto key = std::make_tuple(nseq, want_logits != 0, (int)head, capture != 0, (int)c->track, bound,
                                     (uintptr_t)chv.frames, (uintptr_t)chv.resid);
    auto it = c->fwd_graphs.find(key);
    if (it == c->fwd_graphs.end()) {
      if (c->fwd_graphs.size() >= 32) {  // callers that rotate capture buffers: start over rather than grow
        EVIE_CUDA_TRY(cudaStreamSynchronize(st));
        for (auto& g : c->fwd_graphs) cudaGraphExecDestroy(g.second);
        c->fwd_graphs.clear();
      }
      cudaGraph_t g = nullptr;
      EVIE_CUDA_TRY(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
      evie_status rc = upload_rows(c, R, nseq);
      if (rc == EVIE_OK) rc = enqueue_layers(c, R, nseq, bound, capture, ch);
      if (rc == EVIE_OK && head) rc = enqueue_head(c, nseq, want_logits != 0);
      if (rc == EVIE_OK && ch) rc = join_captures(c);
      const cudaError_t ce = cudaStreamEndCapture(st, &g);
      if (rc != EVIE_OK) {
        if (g) cudaGraphDestroy(g);
        return rc;
      }
      EVIE_CUDA_TRY(ce);
      cudaGraphExec_t exec = nullptr;
      const cudaError_t ie = cudaGraphInstantiate(&exec, g, 0);
      cudaGraphDestroy(g);
      EVIE_CUDA_TRY(ie);
      it = c->fwd_graphs.emplace(key, exec).first;
    }
    EVIE_CUDA_TRY(cudaGraphLaunch(it->second, st));
  } else {
    TRY(upload_rows(c, R, nseq));
    TRY(enqueue_layers(c, R, nseq, max_ctx_rows, capture, ch));
    if (head) TRY(enqueue_head(c, nseq, want_logits != 0));
    if (ch) TRY(join_captures(c));
  }
  if (want_logits && logits)
    EVIE_CUDA_TRY(cudaMemcpyAsync(logits, c->logits, (size_t)nseq * s.V * 4, cudaMemcpyDeviceToHost, st));
  if (next_tokens) EVIE_CUDA_TRY(cudaMemcpyAsync(next_tokens, c->next, nseq * 4, cudaMemcpyDeviceToHost, st));
  if (capture && frames && !chv.frames)
    EVIE_CUDA_TRY(cudaMemcpyAsync(frames, c->frames, (size_t)R * s.L * s.n, cudaMemcpyDeviceToHost, st));
  if (capture && resid && !chv.resid)
    EVIE_CUDA_TRY(cudaMemcpyAsync(resid, c->resid, (size_t)R * s.L * s.d * 2, cudaMemcpyDeviceToHost, st));
  TRY(enqueue_timeout_read(c));
  EVIE_CUDA_TRY(cudaStreamSynchronize(st));
  prof_resolve(c);
  TRY(check_timeouts(c, "forward"));
  if (c->prof && c->prof_failed)
    return evie::fail(EVIE_ERR_CUDA, "forward: the profiling events could not be recorded or timed");
  if (capture) c->cap_rows = R;
  return EVIE_OK;
}

// The decode loop of worker.rs:442-526 with greedy sampling, kept on the device: each step feeds every sequence the
// greedy token of the previous step at the next position, with no host round trip between steps.
evie_status decode_greedy_impl(evie_ctx* c, const evie_seq* seqs, int nseq, int steps, uint32_t* out_tokens,
                               int capture, int8_t* frames, uint16_t* resid) {
  auto& s = c->s;
  EVIE_ARG(steps >= 1, "decode: steps must be >= 1");
  for (int i = 0; i < nseq; i++) {
    EVIE_ARG(seqs[i].n_tokens == 1, "decode: every sequence carries exactly one (first) token");
    EVIE_ARG((long)seqs[i].pos0 + steps <= c->max_ctx, "decode: %d steps from position %d exceed max_ctx %d", steps,
             seqs[i].pos0, c->max_ctx);
  }
  int R = 0, max_ctx_rows = 0;
  TRY(prepare_rows(c, seqs, nseq, &R, &max_ctx_rows));
  const size_t need = (size_t)steps * nseq;
  if (c->hist_cap < need) {
    if (c->hist) {
      EVIE_CUDA_TRY(cudaStreamSynchronize(c->stream));
      cudaFree(c->hist);
      c->hist = nullptr;
    }
    if (cudaMalloc(&c->hist, need * 4) != cudaSuccess) {
      cudaGetLastError();
      return evie::fail(EVIE_ERR_OOM, "decode: cannot allocate the token history");
    }
    c->hist_cap = need;
  }
  cudaStream_t st = c->stream;
  // Every step is (layers, head, advance rows): the advance moves each sequence to its next position and token, so
  // all steps, the first included, are the same work on device-resident inputs. They replay one captured CUDA
  // graph, cached across calls like the forward graphs (key: sequences, capture, tracking, and a context bound
  // that covers every step, rounded up to a multiple of 2048, from which the attention takes its split count).
  // The profiling mode (events around kernel groups) captures each step into a graph of its own, the events as
  // event-record nodes between the groups, so that every group is timed as the replayed step runs it (no host
  // launch gaps inside an event pair). A context created with EVIE_NO_GRAPH=1 runs the steps eagerly.
  const bool use_graph = !c->prof && !c->no_graph;
  const bool prof_graph = c->prof && !c->no_graph;
  const int bound = std::min(c->max_ctx, (max_ctx_rows + steps - 1 + 2047) / 2048 * 2048);
  cudaGraphExec_t exec = nullptr;
  if (use_graph) {
    const auto key = std::make_tuple(nseq, capture != 0, (int)c->track, bound);
    auto it = c->dec_graphs.find(key);
    if (it == c->dec_graphs.end()) {
      if (c->dec_graphs.size() >= 32) {
        EVIE_CUDA_TRY(cudaStreamSynchronize(st));
        for (auto& g : c->dec_graphs) cudaGraphExecDestroy(g.second);
        c->dec_graphs.clear();
      }
      cudaGraph_t g = nullptr;
      EVIE_CUDA_TRY(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
      evie_status rc = enqueue_layers(c, R, nseq, bound, capture);
      if (rc == EVIE_OK) rc = enqueue_head(c, nseq, false);
      if (rc == EVIE_OK) rc = evie::k_advance_rows(c->d_rows, nseq, c->next, st);
      const cudaError_t ce = cudaStreamEndCapture(st, &g);
      if (rc != EVIE_OK) {
        if (g) cudaGraphDestroy(g);
        return rc;
      }
      EVIE_CUDA_TRY(ce);
      cudaGraphExec_t e = nullptr;
      const cudaError_t ie = cudaGraphInstantiate(&e, g, 0);
      cudaGraphDestroy(g);
      EVIE_CUDA_TRY(ie);
      it = c->dec_graphs.emplace(key, e).first;
    }
    exec = it->second;
  }
  struct StepExec {  // the profiling mode's per-step graph, released once its replay has finished
    cudaStream_t st;
    cudaGraphExec_t e = nullptr;
    ~StepExec() { reset(); }
    void reset() {
      if (!e) return;
      cudaStreamSynchronize(st);
      cudaGraphExecDestroy(e);
      e = nullptr;
    }
  } pexec{st};
  for (int i = 0; i < steps; i++) {
    if (exec) {
      EVIE_CUDA_TRY(cudaGraphLaunch(exec, st));
    } else if (prof_graph) {
      c->prof_reserve(2048);
      cudaGraph_t g = nullptr;
      EVIE_CUDA_TRY(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
      evie_status rc = enqueue_layers(c, R, nseq, bound, capture);
      if (rc == EVIE_OK) rc = enqueue_head(c, nseq, false);
      if (rc == EVIE_OK) {
        PROF(P_OTHER);
        rc = evie::k_advance_rows(c->d_rows, nseq, c->next, st);
      }
      const cudaError_t ce = cudaStreamEndCapture(st, &g);
      if (rc != EVIE_OK) {
        if (g) cudaGraphDestroy(g);
        return rc;
      }
      EVIE_CUDA_TRY(ce);
      const cudaError_t ie = cudaGraphInstantiate(&pexec.e, g, 0);
      cudaGraphDestroy(g);
      EVIE_CUDA_TRY(ie);
      EVIE_CUDA_TRY(cudaGraphLaunch(pexec.e, st));
    } else {
      TRY(enqueue_layers(c, R, nseq, max_ctx_rows + i, capture));
      TRY(enqueue_head(c, nseq, false));
      PROF(P_OTHER);
      TRY(evie::k_advance_rows(c->d_rows, nseq, c->next, st));
    }
    EVIE_CUDA_TRY(cudaMemcpyAsync(c->hist + (size_t)i * nseq, c->next, nseq * 4, cudaMemcpyDeviceToDevice, st));
    if (capture && frames)
      EVIE_CUDA_TRY(cudaMemcpyAsync(frames + (size_t)i * nseq * s.L * s.n, c->frames, (size_t)nseq * s.L * s.n,
                                    cudaMemcpyDeviceToHost, st));
    if (capture && resid)
      EVIE_CUDA_TRY(cudaMemcpyAsync(resid + (size_t)i * nseq * s.L * s.d, c->resid, (size_t)nseq * s.L * s.d * 2,
                                    cudaMemcpyDeviceToHost, st));
    if (pexec.e) {
      pexec.reset();
      prof_resolve(c);
    }
  }
  if (out_tokens) EVIE_CUDA_TRY(cudaMemcpyAsync(out_tokens, c->hist, need * 4, cudaMemcpyDeviceToHost, st));
  TRY(enqueue_timeout_read(c));
  EVIE_CUDA_TRY(cudaStreamSynchronize(st));
  prof_resolve(c);
  TRY(check_timeouts(c, "decode"));
  if (c->prof && c->prof_failed)
    return evie::fail(EVIE_ERR_CUDA, "decode: the profiling events could not be recorded or timed");
  if (capture) c->cap_rows = nseq;
  return EVIE_OK;
}

void destroy(evie_ctx* c) {
  if (!c) return;
  cudaSetDevice(c->device);
  if (c->stream) cudaStreamSynchronize(c->stream);
  for (auto& g : c->fwd_graphs) cudaGraphExecDestroy(g.second);
  for (auto& g : c->dec_graphs) cudaGraphExecDestroy(g.second);
  for (void* p : c->allocs) cudaFree(p);
  if (c->hist) cudaFree(c->hist);
  for (auto& p : c->prof_pending) {
    cudaEventDestroy(p.second.first);
    cudaEventDestroy(p.second.second);
  }
  for (auto e : c->prof_free) cudaEventDestroy(e);
  if (c->h_rows) cudaFreeHost(c->h_rows);
  if (c->h_segs) cudaFreeHost(c->h_segs);
  if (c->h_timeouts) cudaFreeHost(c->h_timeouts);
  evie::lens_free(c->lens);
  for (auto e : c->cap_ev) cudaEventDestroy(e);
  if (c->cstream) cudaStreamDestroy(c->cstream);
  if (c->stream) cudaStreamDestroy(c->stream);
  delete c;
}

// Destroys every cached graph (the caller has synchronised the stream): their launch sets no longer match.
void drop_graphs(evie_ctx* c) {
  for (auto& g : c->fwd_graphs) cudaGraphExecDestroy(g.second);
  for (auto& g : c->dec_graphs) cudaGraphExecDestroy(g.second);
  c->fwd_graphs.clear();
  c->dec_graphs.clear();
}

// gpu/mod.rs:555-565 extended with the gates of Plan (steering.rs:97-139): ops and detectors are kept in the
// caller's order within each layer (Plan::apply order); out-of-range ones are dropped as Plan::compile drops them.
evie_status set_plan_impl(evie_ctx* c, int slot, const evie_plan_op* ops, int n_ops, const float* thresholds,
                          int n_gates, const evie_detector* dets, int n_dets) {
  auto& s = c->s;
  EVIE_ARG(slot >= 0 && slot < c->slots, "set_plan: bad slot %d", slot);
  EVIE_ARG(n_ops >= 0 && (n_ops == 0 || ops), "set_plan: bad op list");
  EVIE_ARG(n_gates >= 0 && n_gates <= kMaxGates, "set_plan: at most %d gates per slot (got %d)", kMaxGates, n_gates);
  EVIE_ARG(n_gates == 0 || thresholds, "set_plan: null thresholds");
  EVIE_ARG(n_dets >= 0 && (n_dets == 0 || dets), "set_plan: bad detector list");
  std::vector<evie_op> kept;
  std::vector<int> kept_gate;
  std::vector<int> idx;
  for (int i = 0; i < n_ops; i++) {
    const evie_plan_op& o = ops[i];
    if (o.layer < 0 || o.layer >= s.L || o.neuron < 0 || o.neuron >= s.n) continue;  // as gpu/mod.rs:559
    EVIE_ARG(o.mode >= 1 && o.mode <= 3, "set_plan: mode %d (1 add, 2 mul, 3 set)", o.mode);
    EVIE_ARG(o.gate >= -1 && o.gate < n_gates, "set_plan: op %d names gate %d of %d", i, o.gate, n_gates);
    idx.push_back(i);
  }
  std::stable_sort(idx.begin(), idx.end(), [&](int a, int b) { return ops[a].layer < ops[b].layer; });
  EVIE_ARG((int)idx.size() <= kMaxOps, "set_plan: at most %d ops per slot (got %zu)", kMaxOps, idx.size());
  std::vector<int> range((size_t)s.L * 2, 0);
  for (size_t i = 0; i < idx.size(); i++) {
    const evie_plan_op& o = ops[idx[i]];
    kept.push_back(evie_op{o.layer, o.neuron, o.mode, o.value});
    kept_gate.push_back(o.gate);
    if (range[o.layer * 2 + 1] == 0) range[o.layer * 2] = (int)i;
    range[o.layer * 2 + 1]++;
  }
  // detectors: steering.rs:128-131 (filtered, per-layer lists in push order); gate layers: steering.rs:129-133
  std::vector<int> didx;
  std::vector<evie::GateSpec> gspec(n_gates, evie::GateSpec{0.f, 0, 0, 0});
  std::vector<char> has_det(n_gates, 0);
  for (int g = 0; g < n_gates; g++) gspec[g].threshold = thresholds[g];
  for (int i = 0; i < n_dets; i++) {
    const evie_detector& d = dets[i];
    EVIE_ARG(d.gate >= 0 && d.gate < n_gates, "set_plan: detector %d names gate %d of %d", i, d.gate, n_gates);
    if (d.layer < 0 || d.layer >= s.L || d.neuron < 0 || d.neuron >= s.n) continue;
    didx.push_back(i);
    evie::GateSpec& gs = gspec[d.gate];
    gs.first_layer = has_det[d.gate] ? std::min(gs.first_layer, d.layer) : d.layer;
    gs.last_layer = has_det[d.gate] ? std::max(gs.last_layer, d.layer) : d.layer;
    has_det[d.gate] = 1;
  }
  EVIE_ARG((int)didx.size() <= kMaxDets, "set_plan: at most %d detectors per slot (got %zu)", kMaxDets, didx.size());
  std::stable_sort(didx.begin(), didx.end(), [&](int a, int b) { return dets[a].layer < dets[b].layer; });
  std::vector<evie::DetSpec> dk;
  std::vector<int> drange((size_t)s.L * 2, 0);
  for (size_t i = 0; i < didx.size(); i++) {
    const evie_detector& d = dets[didx[i]];
    dk.push_back(evie::DetSpec{d.gate, d.neuron, d.weight, 0});
    if (drange[d.layer * 2 + 1] == 0) drange[d.layer * 2] = (int)i;
    drange[d.layer * 2 + 1]++;
  }
  std::vector<char> layers(s.L, 0);
  for (size_t i = 0; i < didx.size(); i++) layers[dets[didx[i]].layer] = 1;
  for (int g = 0; g < n_gates; g++) layers[gspec[g].last_layer] = 1;

  EVIE_CUDA_TRY(cudaSetDevice(c->device));
  EVIE_CUDA_TRY(cudaStreamSynchronize(c->stream));
  const size_t so = (size_t)slot * kMaxOps, sg = (size_t)slot * kMaxGates, sd = (size_t)slot * kMaxDets;
  const size_t sr = (size_t)slot * s.L * 2;
  if (!kept.empty()) {
    EVIE_CUDA_TRY(cudaMemcpy(c->ops + so, kept.data(), kept.size() * sizeof(evie_op), cudaMemcpyHostToDevice));
    EVIE_CUDA_TRY(cudaMemcpy(c->op_gate + so, kept_gate.data(), kept_gate.size() * 4, cudaMemcpyHostToDevice));
  }
  EVIE_CUDA_TRY(cudaMemcpy(c->op_range + sr, range.data(), range.size() * 4, cudaMemcpyHostToDevice));
  if (n_gates)
    EVIE_CUDA_TRY(cudaMemcpy(c->gates + sg, gspec.data(), gspec.size() * sizeof(evie::GateSpec), cudaMemcpyHostToDevice));
  if (!dk.empty())
    EVIE_CUDA_TRY(cudaMemcpy(c->dets + sd, dk.data(), dk.size() * sizeof(evie::DetSpec), cudaMemcpyHostToDevice));
  EVIE_CUDA_TRY(cudaMemcpy(c->det_range + sr, drange.data(), drange.size() * 4, cudaMemcpyHostToDevice));
  EVIE_CUDA_TRY(cudaMemcpy(c->n_gates + slot, &n_gates, 4, cudaMemcpyHostToDevice));
  EVIE_CUDA_TRY(cudaMemset(c->gate_open + sg, 0, kMaxGates * 4));  // Plan::new_state, steering.rs:145-148
  EVIE_CUDA_TRY(cudaMemset(c->gate_score + sg, 0, kMaxGates * 4));
  EVIE_CUDA_TRY(cudaMemset(c->gate_from + sg, 0, kMaxGates * 4));
  c->h_n_gates[slot] = n_gates;
  c->h_gate_layers[slot] = layers;
  // The set of layers that launch the detector kernel is part of every captured forward graph: a change drops them.
  std::vector<char> all(s.L, 0);
  for (int i = 0; i < c->slots; i++)
    for (int l = 0; l < s.L; l++) all[l] |= c->h_gate_layers[i][l];
  if (all != c->gate_layers) {
    drop_graphs(c);
    c->gate_layers = all;
  }
  return EVIE_OK;
}
// Records the thread-local message of a failed call into the context.
evie_status remember(evie_ctx* c, evie_status rc) {
  if (rc != EVIE_OK && c) c->err = evie::thread_error();
  return rc;
}

}  // namespace

extern "C" {

evie_status evie_create(const char* ckpt_dir, int device, int slots, int max_ctx, int max_rows, evie_ctx** out) {
  if (!out) return evie::fail(EVIE_ERR_ARG, "evie_create: out is null");
  *out = nullptr;
  EVIE_ARG(ckpt_dir != nullptr, "evie_create: null checkpoint directory");
  EVIE_ARG(slots >= 1 && slots <= 4096, "evie_create: slots must be in 1..4096");
  EVIE_ARG(max_ctx >= 1 && max_ctx <= (int)evie::kGqaMaxContext, "evie_create: max_ctx must be in 1..%ld",
           (long)evie::kGqaMaxContext);
  EVIE_ARG(max_rows >= 1 && max_rows <= 65535, "evie_create: max_rows must be in 1..65535");
  int ndev = 0;
  EVIE_CUDA_TRY(cudaGetDeviceCount(&ndev));
  EVIE_ARG(device >= 0 && device < ndev, "evie_create: device %d not present (%d devices)", device, ndev);
  evie_ctx* c = new evie_ctx();
  c->device = device;
  c->slots = slots;
  c->max_ctx = max_ctx;
  c->max_rows = max_rows;
  const char* kvf = getenv("EVIE_KV_F32");
  c->kv_f32 = kvf && kvf[0] == '1';
  evie_status rc = EVIE_OK;
  do {
    if (cudaSetDevice(device) != cudaSuccess) { rc = evie::fail(EVIE_ERR_CUDA, "cudaSetDevice(%d) failed", device); break; }
    if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess) { rc = evie::fail(EVIE_ERR_CUDA, "stream creation failed"); break; }
    if (cudaStreamCreateWithFlags(&c->cstream, cudaStreamNonBlocking) != cudaSuccess) { rc = evie::fail(EVIE_ERR_CUDA, "stream creation failed"); break; }
    // the device's timeout counter of the bounded-wait kernels, looked up now rather than inside a graph capture
    if (!evie::device_timeout_counter()) { rc = evie::fail(EVIE_ERR_CUDA, "device timeout counter unavailable"); break; }
    if ((rc = read_config(c, ckpt_dir)) != EVIE_OK) break;
    if ((rc = load_weights(c, ckpt_dir)) != EVIE_OK) break;
    if ((rc = allocate_state(c)) != EVIE_OK) break;
    if (cudaDeviceSynchronize() != cudaSuccess) { rc = evie::fail(EVIE_ERR_CUDA, "initialisation failed"); break; }
  } while (0);
  if (rc != EVIE_OK) {
    destroy(c);
    return rc;
  }
  *out = c;
  return EVIE_OK;
}

void evie_destroy(evie_ctx* c) { destroy(c); }

const char* evie_last_error(const evie_ctx* c) { return c ? c->err.c_str() : evie::thread_error().c_str(); }

evie_status evie_info(const evie_ctx* c, evie_model_info* out) {
  EVIE_ARG(c && out, "evie_info: null argument");
  auto& s = c->s;
  *out = evie_model_info{s.d, s.n, s.L, s.V, c->n_lin, c->n_full, c->slots, c->max_ctx, c->max_rows, kMaxOps,
                         (int64_t)c->weight_bytes, (int64_t)c->cache_bytes};
  return EVIE_OK;
}

evie_status evie_forward(evie_ctx* c, const evie_seq* seqs, int n_seqs, int want_logits, int capture, float* logits,
                         int8_t* frames, uint16_t* resid, uint32_t* next_tokens) {
  if (!c) return evie::fail(EVIE_ERR_ARG, "evie_forward: null context");
  if (!seqs) return remember(c, evie::fail(EVIE_ERR_ARG, "evie_forward: null sequences"));
  if (cudaSetDevice(c->device) != cudaSuccess) return remember(c, evie::fail(EVIE_ERR_CUDA, "cudaSetDevice failed"));
  return remember(c, forward_impl(c, seqs, n_seqs, want_logits, capture, logits, frames, resid, next_tokens));
}

evie_status evie_decode_greedy(evie_ctx* c, const evie_seq* seqs, int n_seqs, int steps, uint32_t* out_tokens,
                               int capture, int8_t* frames, uint16_t* resid) {
  if (!c) return evie::fail(EVIE_ERR_ARG, "evie_decode_greedy: null context");
  if (!seqs) return remember(c, evie::fail(EVIE_ERR_ARG, "evie_decode_greedy: null sequences"));
  if (cudaSetDevice(c->device) != cudaSuccess) return remember(c, evie::fail(EVIE_ERR_CUDA, "cudaSetDevice failed"));
  return remember(c, decode_greedy_impl(c, seqs, n_seqs, steps, out_tokens, capture, frames, resid));
}

void* evie_stream(const evie_ctx* c) { return c ? (void*)c->stream : nullptr; }

evie_status evie_profile(evie_ctx* c, int on) {
  if (!c) return evie::fail(EVIE_ERR_ARG, "evie_profile: null context");
  c->prof = on != 0;
  c->prof_failed = false;
  for (int i = 0; i < P_COUNT; i++) c->prof_ms[i] = 0.0, c->prof_n[i] = 0;
  return EVIE_OK;
}

int evie_profile_read(const evie_ctx* c, int i, const char** name, double* ms, int64_t* launches) {
  if (!c || i < 0 || i >= P_COUNT) return 0;
  if (name) *name = kProfNames[i];
  if (ms) *ms = c->prof_ms[i];
  if (launches) *launches = c->prof_n[i];
  return P_COUNT;
}

evie_status evie_set_ops(evie_ctx* c, int slot, const evie_op* ops, int n_ops) {
  if (!c) return evie::fail(EVIE_ERR_ARG, "evie_set_ops: null context");
  if (n_ops < 0 || (n_ops > 0 && !ops)) return remember(c, evie::fail(EVIE_ERR_ARG, "evie_set_ops: bad op list"));
  std::vector<evie_plan_op> p(n_ops);
  for (int i = 0; i < n_ops; i++) p[i] = evie_plan_op{ops[i].layer, ops[i].neuron, ops[i].mode, ops[i].value, -1};
  return remember(c, set_plan_impl(c, slot, p.data(), n_ops, nullptr, 0, nullptr, 0));
}

evie_status evie_set_plan(evie_ctx* c, int slot, const evie_plan_op* ops, int n_ops, const float* thresholds,
                          int n_gates, const evie_detector* dets, int n_dets) {
  if (!c) return evie::fail(EVIE_ERR_ARG, "evie_set_plan: null context");
  return remember(c, set_plan_impl(c, slot, ops, n_ops, thresholds, n_gates, dets, n_dets));
}

evie_status evie_gate_state(evie_ctx* c, int slot, int32_t* open, float* score, int n_gates) {
  if (!c) return evie::fail(EVIE_ERR_ARG, "evie_gate_state: null context");
  if (slot < 0 || slot >= c->slots) return remember(c, evie::fail(EVIE_ERR_ARG, "evie_gate_state: bad slot %d", slot));
  const int ng = c->h_n_gates[slot];
  if (n_gates < ng)
    return remember(c, evie::fail(EVIE_ERR_ARG, "evie_gate_state: slot %d has %d gates, room for %d", slot, ng, n_gates));
  if (cudaSetDevice(c->device) != cudaSuccess) return remember(c, evie::fail(EVIE_ERR_CUDA, "cudaSetDevice failed"));
  const size_t sg = (size_t)slot * kMaxGates;
  cudaError_t e = cudaStreamSynchronize(c->stream);
  if (e == cudaSuccess && open && ng) e = cudaMemcpy(open, c->gate_open + sg, ng * 4, cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && score && ng) e = cudaMemcpy(score, c->gate_score + sg, ng * 4, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return remember(c, evie::fail(EVIE_ERR_CUDA, "evie_gate_state: %s", cudaGetErrorString(e)));
  return EVIE_OK;
}

evie_status evie_reset_gates(evie_ctx* c, int slot) {
  if (!c) return evie::fail(EVIE_ERR_ARG, "evie_reset_gates: null context");
  if (slot < 0 || slot >= c->slots) return remember(c, evie::fail(EVIE_ERR_ARG, "evie_reset_gates: bad slot %d", slot));
  if (cudaSetDevice(c->device) != cudaSuccess) return remember(c, evie::fail(EVIE_ERR_CUDA, "cudaSetDevice failed"));
  const size_t sg = (size_t)slot * kMaxGates;
  cudaError_t e = cudaMemsetAsync(c->gate_open + sg, 0, kMaxGates * 4, c->stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(c->gate_score + sg, 0, kMaxGates * 4, c->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
  if (e != cudaSuccess) return remember(c, evie::fail(EVIE_ERR_CUDA, "evie_reset_gates: %s", cudaGetErrorString(e)));
  return EVIE_OK;
}

namespace {
evie::AnalysisModel analysis_model(evie_ctx* c) {
  evie::AnalysisModel am;
  am.lm_head = c->lm_head;
  am.V = c->s.V;
  am.d = c->s.d;
  am.n = c->s.n;
  am.final_norm = c->final_norm;
  am.eps = c->s.eps;
  for (const Layer& L : c->layers) am.w_down.push_back(L.w_down);
  am.lens = &c->lens;
  am.st = c->stream;
  return am;
}
}  // namespace

// analysis.rs:129-201 on the context's weights, through the lens set by evie_set_lens (if any).
evie_status evie_neuron_sigma(evie_ctx* c, float* sigma, size_t n, float* mean, float* m_scale) {
  if (!c) return evie::fail(EVIE_ERR_ARG, "evie_neuron_sigma: null context");
  auto& s = c->s;
  if (!sigma || n != (size_t)s.L * s.n)
    return remember(c, evie::fail(EVIE_ERR_ARG, "evie_neuron_sigma: expected %zu outputs, got %zu",
                                  (size_t)s.L * s.n, n));
  if (cudaSetDevice(c->device) != cudaSuccess) return remember(c, evie::fail(EVIE_ERR_CUDA, "cudaSetDevice failed"));
  return remember(c, evie::neuron_sigma_run(analysis_model(c), sigma, mean, m_scale));
}

// lens.rs:20-54 once the file is read: maps[l] = [hidden][hidden] 16-bit values or NULL.
evie_status evie_set_lens(evie_ctx* c, const uint16_t* const* maps, int n_layers, int kind, int target_layer) {
  if (!c) return evie::fail(EVIE_ERR_ARG, "evie_set_lens: null context");
  if (!maps || n_layers != c->s.L)
    return remember(c, evie::fail(EVIE_ERR_ARG, "evie_set_lens: expected %d layer maps, got %d", c->s.L, n_layers));
  if (target_layer < 0 || target_layer >= c->s.L)
    return remember(c, evie::fail(EVIE_ERR_ARG, "evie_set_lens: target layer %d out of range", target_layer));
  if (cudaSetDevice(c->device) != cudaSuccess) return remember(c, evie::fail(EVIE_ERR_CUDA, "cudaSetDevice failed"));
  return remember(c, evie::lens_upload(c->lens, maps, n_layers, c->s.d, kind, target_layer, c->stream));
}

evie_status evie_clear_lens(evie_ctx* c) {
  if (!c) return evie::fail(EVIE_ERR_ARG, "evie_clear_lens: null context");
  if (cudaSetDevice(c->device) != cudaSuccess) return remember(c, evie::fail(EVIE_ERR_CUDA, "cudaSetDevice failed"));
  evie::lens_free(c->lens);
  return EVIE_OK;
}

// analysis.rs:28-34
evie_status evie_lens_logits(evie_ctx* c, int layer, const float* vecs, int n, float* logits) {
  if (!c) return evie::fail(EVIE_ERR_ARG, "evie_lens_logits: null context");
  if (n < 0 || (n > 0 && (!vecs || !logits))) return remember(c, evie::fail(EVIE_ERR_ARG, "evie_lens_logits: bad buffers"));
  if (cudaSetDevice(c->device) != cudaSuccess) return remember(c, evie::fail(EVIE_ERR_CUDA, "cudaSetDevice failed"));
  return remember(c, evie::lens_logits_run(analysis_model(c), layer, vecs, n, logits));
}

// analysis.rs:37-67
evie_status evie_neuron_logits(evie_ctx* c, const int32_t* layers, const int32_t* neurons, int n, float* logits) {
  if (!c) return evie::fail(EVIE_ERR_ARG, "evie_neuron_logits: null context");
  if (n < 0 || (n > 0 && (!layers || !neurons || !logits)))
    return remember(c, evie::fail(EVIE_ERR_ARG, "evie_neuron_logits: bad buffers"));
  if (cudaSetDevice(c->device) != cudaSuccess) return remember(c, evie::fail(EVIE_ERR_CUDA, "cudaSetDevice failed"));
  return remember(c, evie::neuron_logits_run(analysis_model(c), layers, neurons, n, logits));
}

// analysis.rs:213-240 (the per-neuron best z of both poles; the ranking is the caller's)
evie_status evie_search_scores(evie_ctx* c, const uint32_t* tokens, int n_tokens, const float* mean,
                               const float* sigma, float* z_up, float* z_dn) {
  if (!c) return evie::fail(EVIE_ERR_ARG, "evie_search_scores: null context");
  if (n_tokens < 1 || !tokens || !mean || !sigma || !z_up || !z_dn)
    return remember(c, evie::fail(EVIE_ERR_ARG, "evie_search_scores: bad buffers"));
  if (cudaSetDevice(c->device) != cudaSuccess) return remember(c, evie::fail(EVIE_ERR_CUDA, "cudaSetDevice failed"));
  return remember(c, evie::search_scores_run(analysis_model(c), tokens, n_tokens, mean, sigma, z_up, z_dn));
}

// mcp.rs:242-256 over the frames the last capturing call left on the device.
evie_status evie_read_top_active(evie_ctx* c, int k, int32_t* out, int* rows) {
  if (!c) return evie::fail(EVIE_ERR_ARG, "evie_read_top_active: null context");
  if (k < 1 || k > 100) return remember(c, evie::fail(EVIE_ERR_ARG, "evie_read_top_active: k must be in 1..100"));
  if (c->cap_rows == 0) return remember(c, evie::fail(EVIE_ERR_ARG, "evie_read_top_active: no captured rows yet"));
  if (!out) return remember(c, evie::fail(EVIE_ERR_ARG, "evie_read_top_active: null output"));
  if (cudaSetDevice(c->device) != cudaSuccess) return remember(c, evie::fail(EVIE_ERR_CUDA, "cudaSetDevice failed"));
  const long long width = (long long)c->s.L * c->s.n;
  evie_status rc = evie::k_top_active(c->frames, c->cap_rows, width, k, c->topk, c->stream);
  if (rc != EVIE_OK) return remember(c, rc);
  cudaError_t e = cudaMemcpyAsync(out, c->topk, (size_t)c->cap_rows * k * 4, cudaMemcpyDeviceToHost, c->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
  if (e != cudaSuccess) return remember(c, evie::fail(EVIE_ERR_CUDA, "evie_read_top_active: %s", cudaGetErrorString(e)));
  if (rows) *rows = c->cap_rows;
  return EVIE_OK;
}

// sampling.rs:27-29 (Sampler::new) per slot; NULL = SampleParams::default (greedy).
evie_status evie_set_sampler(evie_ctx* c, int slot, const evie_sample_params* p) {
  if (!c) return evie::fail(EVIE_ERR_ARG, "evie_set_sampler: null context");
  if (slot < 0 || slot >= c->slots) return remember(c, evie::fail(EVIE_ERR_ARG, "evie_set_sampler: bad slot %d", slot));
  const evie_sample_params d{0.0f, 1.0f, 0.0f, 1.0f, 0};
  const evie_sample_params& q = p ? *p : d;
  const evie::SamplerParams sp{q.temperature, q.top_p, q.min_p, q.repetition_penalty};
  const uint64_t rng = evie::sampler_seed_state(q.seed);
  if (cudaSetDevice(c->device) != cudaSuccess) return remember(c, evie::fail(EVIE_ERR_CUDA, "cudaSetDevice failed"));
  cudaError_t e = cudaStreamSynchronize(c->stream);
  if (e == cudaSuccess) e = cudaMemcpy(c->samp + slot, &sp, sizeof(sp), cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(c->samp_rng + slot, &rng, 8, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return remember(c, evie::fail(EVIE_ERR_CUDA, "evie_set_sampler: %s", cudaGetErrorString(e)));
  // plain greedy (temperature <= 0, no penalty) is the argmax kernel's token; anything else needs the sampler
  c->h_samp_on[slot] = !(q.temperature <= 0.0f) || q.repetition_penalty != 1.0f;
  bool any = false;
  for (char on : c->h_samp_on) any = any || on;
  if (any != c->samp_active) {  // the sampler launch is part of every captured graph
    drop_graphs(c);
    c->samp_active = any;
  }
  return EVIE_OK;
}

// gpu/mod.rs:567-575: zero the slot's recurrent and conv state; KV entries are overwritten by position.
evie_status evie_reset_slot(evie_ctx* c, int slot) {
  if (!c) return evie::fail(EVIE_ERR_ARG, "evie_reset_slot: null context");
  auto& s = c->s;
  if (slot < 0 || slot >= c->slots) return remember(c, evie::fail(EVIE_ERR_ARG, "evie_reset_slot: bad slot %d", slot));
  const size_t cs = (size_t)std::max(c->n_lin, 1) * (s.K - 1) * s.conv_dim;
  const size_t rs = (size_t)std::max(c->n_lin, 1) * s.hv * s.dk * s.dv;
  cudaSetDevice(c->device);
  cudaError_t e = cudaMemsetAsync(c->conv_state + (size_t)slot * cs, 0, cs * 4, c->stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(c->rec_state + (size_t)slot * rs, 0, rs * 4, c->stream);
  if (e == cudaSuccess)
    e = cudaMemsetAsync(c->seen + (size_t)slot * c->seen_words, 0, (size_t)c->seen_words * 4, c->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
  if (e != cudaSuccess) return remember(c, evie::fail(EVIE_ERR_CUDA, "evie_reset_slot: %s", cudaGetErrorString(e)));
  return EVIE_OK;
}

evie_status evie_set_scale(evie_ctx* c, const float* scale, size_t n) {
  if (!c) return evie::fail(EVIE_ERR_ARG, "evie_set_scale: null context");
  const size_t want = (size_t)c->s.L * c->s.n;
  if (!scale || n != want)  // gpu/mod.rs:550 ignores a wrong length; here it is an error the caller sees
    return remember(c, evie::fail(EVIE_ERR_ARG, "evie_set_scale: expected %zu scales, got %zu", want, n));
  cudaSetDevice(c->device);
  cudaError_t e = cudaStreamSynchronize(c->stream);
  if (e == cudaSuccess) e = cudaMemcpy(c->scale, scale, n * 4, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return remember(c, evie::fail(EVIE_ERR_CUDA, "evie_set_scale: %s", cudaGetErrorString(e)));
  return EVIE_OK;
}

evie_status evie_track_max(evie_ctx* c, int on) {
  if (!c) return evie::fail(EVIE_ERR_ARG, "evie_track_max: null context");
  c->track = on != 0;
  if (on) {  // gpu/mod.rs:583-587: turning tracking on clears the maxima
    cudaSetDevice(c->device);
    cudaError_t e = cudaMemsetAsync(c->maxbuf, 0, (size_t)c->s.L * c->s.n * 4, c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess) return remember(c, evie::fail(EVIE_ERR_CUDA, "evie_track_max: %s", cudaGetErrorString(e)));
  }
  return EVIE_OK;
}

evie_status evie_read_max(evie_ctx* c, float* out, size_t n) {
  if (!c) return evie::fail(EVIE_ERR_ARG, "evie_read_max: null context");
  const size_t want = (size_t)c->s.L * c->s.n;
  if (!out || n < want) return remember(c, evie::fail(EVIE_ERR_ARG, "evie_read_max: need room for %zu values", want));
  cudaSetDevice(c->device);
  cudaError_t e = cudaStreamSynchronize(c->stream);
  if (e == cudaSuccess) e = cudaMemcpy(out, c->maxbuf, want * 4, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return remember(c, evie::fail(EVIE_ERR_CUDA, "evie_read_max: %s", cudaGetErrorString(e)));
  return EVIE_OK;
}

}  // extern "C"
