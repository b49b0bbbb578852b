// CPU ORACLE — TEST INFRASTRUCTURE ONLY.
//
// A plain C++ restatement of casettek/raster-inference's deterministic
// integer-weight transformer path, used as the parity checker for the B200
// product in raster-inference_b200/ and as the timed CPU baseline.  Only
// tests/, __graft_entry__.smoke() and bench.py (cpu_baseline leg and the
// `--impl reference` arm) load it.  It is never part of the shipped path.
//
// What it restates (reference file:line):
//   - detwgt v2 reader, fail-closed: src/shared/model/gemma/io.rs:230-395
//   - detwgt v2 encoder: src/shared/numerics/det_num/artifact.rs:61-206
//   - Gemma config semantics: src/shared/model/gemma/io.rs:98-190, :1896-2045
//   - embedding: io.rs:2118-2132, :2446-2518
//   - PLE prepare (prefill): src/routines/prefill_prepare_aux/native/tiles.rs:111-243
//   - PLE input (decode): src/shared/numerics/det_kernels.rs:1142-1208
//   - layer prefill: det_kernels.rs:499-821 (+ det_tensor.rs:250-268 cache retention)
//   - layer decode: det_kernels.rs:866-1133 (+ det_tensor.rs:308-337 append/trim)
//   - logits: det_kernels.rs:1217-1267; select: det_num/ops.rs:463
//   - drivers: prefill_range/native/deterministic_tiles.rs:69-199,
//     decode_layer_range/native/tiles.rs:133-197,
//     decode_transition_finalize/native/tiles.rs:9-65,
//     prefill_finalize/native/tiles.rs:11-107
//   - commitments: src/shared/numerics/transformer_kernels.rs:1395-1482
//
// Parallelism is output-index splitting only (like the reference's rayon
// drivers, det_kernels.rs:156-178), so results are thread-count independent.
#include <algorithm>
#include <atomic>
#include <condition_variable>
#include <mutex>
#include <cmath>
#include <cstdio>
#include <functional>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "det_num.hpp"
#include "sha256.hpp"

using namespace dor;

// ---------------------------------------------------------------------------
// threading: a persistent pool (like the reference's global rayon pool);
// parallel_for splits [0, n) into contiguous chunks, one per worker.
// ---------------------------------------------------------------------------
static int g_threads = 1;

class Pool {
 public:
  void resize(int n) {
    stop();
    n_ = n;
    // resize() and run() are called from one host thread, so no job is
    // published while workers start; each worker begins at the current
    // generation and takes every job published afterwards.
    uint64_t g = gen_;
    for (int i = 1; i < n; ++i) workers_.emplace_back([this, i, g] { loop(i, g); });
  }
  void run(size_t n, const std::function<void(size_t, size_t)>& fn) {
    int t = n_ < 1 ? 1 : n_;
    if (t <= 1 || n < 2) { fn(0, n); return; }
    {
      std::unique_lock<std::mutex> lk(mu_);
      fn_ = &fn;
      n_items_ = n;
      pending_ = t - 1;
      ++gen_;
    }
    cv_.notify_all();
    chunk(0, t, n, fn);
    std::unique_lock<std::mutex> lk(mu_);
    done_.wait(lk, [this] { return pending_ == 0; });
  }
  ~Pool() { stop(); }

 private:
  static void chunk(int i, int t, size_t n, const std::function<void(size_t, size_t)>& fn) {
    size_t c = (n + t - 1) / t, lo = i * c, hi = std::min(n, lo + c);
    if (lo < hi) fn(lo, hi);
  }
  void loop(int i, uint64_t seen) {
    for (;;) {
      const std::function<void(size_t, size_t)>* fn;
      size_t n;
      {
        std::unique_lock<std::mutex> lk(mu_);
        cv_.wait(lk, [&] { return quit_ || gen_ != seen; });
        if (quit_) return;
        seen = gen_;
        fn = fn_;
        n = n_items_;
      }
      chunk(i, n_, n, *fn);
      std::unique_lock<std::mutex> lk(mu_);
      if (--pending_ == 0) done_.notify_one();
    }
  }
  void stop() {
    {
      std::unique_lock<std::mutex> lk(mu_);
      quit_ = true;
    }
    cv_.notify_all();
    for (auto& w : workers_) w.join();
    workers_.clear();
    quit_ = false;
  }
  std::vector<std::thread> workers_;
  std::mutex mu_;
  std::condition_variable cv_, done_;
  const std::function<void(size_t, size_t)>* fn_ = nullptr;
  size_t n_items_ = 0;
  int pending_ = 0, n_ = 1;
  uint64_t gen_ = 0;
  bool quit_ = false;
};
static Pool g_pool;

static void parallel_for(size_t n, const std::function<void(size_t, size_t)>& fn) { g_pool.run(n, fn); }

struct Fail : std::runtime_error {
  explicit Fail(const std::string& m) : std::runtime_error(m) {}
};

// ---------------------------------------------------------------------------
// detwgt v2 reader (io.rs:230-395) — fail closed
// ---------------------------------------------------------------------------
struct Tensor {
  std::vector<size_t> shape;
  int width = 32;               // 16 or 32
  std::vector<int16_t> w16;     // payload when width == 16
  std::vector<int32_t> w32;     // payload when width == 32
  size_t rows() const { return shape.size() == 2 ? shape[0] : 1; }
  size_t cols() const { return shape.empty() ? 0 : shape.back(); }
  int32_t at(size_t i) const { return width == 16 ? (int32_t)w16[i] : w32[i]; }
};

static const uint64_t ROW_MASS_LIMIT = (uint64_t)1 << 31;  // det_num/mod.rs:17

struct Reader {
  const uint8_t* b;
  size_t n, cur = 0;
  const uint8_t* take(size_t len) {
    if (len > n - cur) throw Fail("artifact ended unexpectedly");
    const uint8_t* p = b + cur;
    cur += len;
    return p;
  }
  uint32_t u32() { const uint8_t* p = take(4); uint32_t v; memcpy(&v, p, 4); return v; }
  uint64_t u64() { const uint8_t* p = take(8); uint64_t v; memcpy(&v, p, 8); return v; }
};

static std::map<std::string, Tensor> read_detwgt(const std::vector<uint8_t>& bytes) {
  Reader r{bytes.data(), bytes.size()};
  const uint8_t* magic = r.take(8);
  if (memcmp(magic, "DNWGTV0\0", 8) != 0) throw Fail("unsupported deterministic artifact magic");
  uint32_t ver = r.u32();
  if (ver != 2) throw Fail("unsupported deterministic artifact format version " + std::to_string(ver));
  uint32_t spec = r.u32();
  if (spec != 1) throw Fail("unsupported deterministic artifact det_num spec version " + std::to_string(spec));
  uint64_t count = r.u64();
  std::map<std::string, Tensor> out;
  for (uint64_t t = 0; t < count; ++t) {
    uint32_t name_len = r.u32();
    const uint8_t* np = r.take(name_len);
    std::string name((const char*)np, name_len);
    uint32_t rank = r.u32();
    Tensor tn;
    unsigned __int128 prod = 1;
    for (uint32_t i = 0; i < rank; ++i) {
      uint64_t d = r.u64();
      tn.shape.push_back((size_t)d);
      prod *= d;
      if (prod > (unsigned __int128)UINT64_MAX) throw Fail("tensor shape overflowed");
    }
    uint64_t ec = r.u64();
    if ((unsigned __int128)ec != prod) throw Fail("tensor `" + name + "` element count mismatch");
    uint32_t wt = r.u32();
    if (wt != 16 && wt != 32) throw Fail("tensor `" + name + "` has an invalid element width");
    tn.width = (int)wt;
    uint64_t pl = r.u64();
    if ((unsigned __int128)pl != (unsigned __int128)ec * (wt / 8)) throw Fail("tensor `" + name + "` payload length mismatch");
    uint64_t mass = r.u64();
    if (rank >= 2 && mass >= ROW_MASS_LIMIT) throw Fail("tensor `" + name + "` max row mass violates the overflow bound");
    size_t pad = (size_t)((64 - r.cur % 64) % 64);
    const uint8_t* pp = r.take(pad);
    for (size_t i = 0; i < pad; ++i)
      if (pp[i] != 0) throw Fail("tensor `" + name + "` has non-zero payload alignment padding");
    const uint8_t* payload = r.take((size_t)pl);
    if (wt == 16) { tn.w16.resize(ec); memcpy(tn.w16.data(), payload, pl); }
    else { tn.w32.resize(ec); memcpy(tn.w32.data(), payload, pl); }
    if (out.count(name)) throw Fail("deterministic artifact contains duplicate tensor `" + name + "`");
    out.emplace(name, std::move(tn));
  }
  if (r.cur != bytes.size()) throw Fail("deterministic artifact has trailing bytes after tensor payloads");
  return out;
}

// ---------------------------------------------------------------------------
// config (io.rs:61-190, :1896-1994)
// ---------------------------------------------------------------------------
extern "C" {
typedef struct {
  int32_t hidden_size, num_hidden_layers, num_attention_heads, num_key_value_heads, head_dim;
  int32_t global_head_dim;              // -1 absent
  int32_t num_global_key_value_heads;   // -1 absent
  int32_t hidden_size_per_layer_input;  // -1 absent
  int32_t vocab_size;
  int32_t vocab_size_per_layer_input;   // -1 absent
  int32_t sliding_window;
  int32_t num_kv_shared_layers;         // -1 absent
  int32_t attention_k_eq_v;             // -1 absent, else 0/1
  int32_t tie_word_embeddings;          // -1 absent, else 0/1
  int32_t bidirectional_all;            // use_bidirectional_attention == "all"
  int32_t enable_moe_block;
  int32_t hidden_activation_is_gelu_tanh;
  int32_t has_softcap;
  float final_logit_softcapping;
  float rms_norm_eps;
  int32_t has_full_partial, has_full_theta, has_sliding_theta, has_global_theta;
  float full_partial_rotary_factor, full_rope_theta, sliding_rope_theta, global_rope_theta;
  int32_t n_layer_types;
  int32_t layer_is_sliding[1024];
} dor_config;
}

struct LayerSpec {
  bool sliding;
  size_t head_dim, num_kv_heads, rotary_dim, window;  // window: effective sliding window (sliding only)
  bool cache_trim;                                     // cache_sliding_window is Some
  int donor;                                           // kv_shared_layer_index or -1
  bool k_eq_v;
  int64_t rope_base, rope_step;
  const Tensor *q, *k, *v, *o, *gate, *up, *down, *ple_gate, *ple_proj;
  const Tensor *q_norm, *k_norm, *in_ln, *post_attn_ln, *pre_ff_ln, *post_ff_ln, *ple_norm;
  bool has_scalar;
  int32_t scalar;
};

struct Model {
  std::map<std::string, Tensor> t;
  size_t H, L, Hq, V, P, ple_vocab;
  int64_t eps;
  bool has_softcap;
  int32_t softcap;
  int32_t emb_scale, ple_emb_scale, ple_proj_scale, ple_in_scale;
  const Tensor *emb, *lm_head, *final_norm, *ple_table, *ple_model_proj, *ple_proj_norm;
  std::vector<LayerSpec> layers;
};

static const Tensor& need(const Model& m, const std::string& name, int rank) {
  auto it = m.t.find(name);
  if (it == m.t.end()) throw Fail("failed to load tensor `" + name + "` from deterministic artifact");
  if (rank > 0 && (int)it->second.shape.size() != rank) throw Fail("tensor `" + name + "` has unexpected rank");
  return it->second;
}

static std::unique_ptr<Model> build_model(std::map<std::string, Tensor>&& tensors, const dor_config& c) {
  auto mp = std::make_unique<Model>();
  Model& m = *mp;
  m.t = std::move(tensors);
  if (c.enable_moe_block) throw Fail("only Gemma 4 dense layers are supported");
  if (!c.hidden_activation_is_gelu_tanh) throw Fail("only gelu_pytorch_tanh is supported");
  if (c.num_hidden_layers != c.n_layer_types) throw Fail("Gemma config layer count mismatch");
  m.H = c.hidden_size;
  m.L = c.num_hidden_layers;
  m.Hq = c.num_attention_heads;
  m.V = c.vocab_size;
  m.P = c.hidden_size_per_layer_input > 0 ? c.hidden_size_per_layer_input : 0;
  m.ple_vocab = c.vocab_size_per_layer_input >= 0 ? c.vocab_size_per_layer_input : c.vocab_size;
  m.eps = f32_to_acc(c.rms_norm_eps);
  m.has_softcap = c.has_softcap != 0;
  m.softcap = m.has_softcap ? f32_to_act(c.final_logit_softcapping) : 0;

  // embedding source (io.rs:44-48, :2118-2132): first available name, scale sqrt(cols)
  const char* emb_names[] = {"model.language_model.embed_tokens.weight", "language_model.embed_tokens.weight",
                             "embed_tokens.weight"};
  m.emb = nullptr;
  for (const char* n : emb_names) {
    auto it = m.t.find(n);
    if (it != m.t.end()) {
      if (it->second.shape.size() != 2) throw Fail("embedding tensor must be a matrix");
      m.emb = &it->second;
      break;
    }
  }
  if (!m.emb) throw Fail("failed to find any supported embedding tensor");
  m.emb_scale = f32_to_act(std::sqrt((float)m.emb->shape[1]));

  // kv sharing (io.rs:165-190)
  size_t nshared = c.num_kv_shared_layers > 0 ? (size_t)c.num_kv_shared_layers : 0;
  size_t first_shared = m.L >= nshared ? m.L - nshared : 0;
  std::vector<int> donor(m.L, -1);
  std::vector<bool> is_donor(m.L, false);
  if (nshared > 0) {
    for (size_t l = first_shared; l < m.L; ++l) {
      int d = -1;
      for (size_t j = 0; j < first_shared; ++j)
        if (c.layer_is_sliding[j] == c.layer_is_sliding[l]) d = (int)j;
      if (d < 0) throw Fail("Gemma layer is configured to share KV without a prior donor layer");
      donor[l] = d;
      is_donor[d] = true;
    }
  }
  bool k_eq_v_cfg = c.attention_k_eq_v == 1;
  float partial = c.has_full_partial ? c.full_partial_rotary_factor : 0.25f;
  float local_theta = c.has_sliding_theta ? c.sliding_rope_theta : 10000.0f;
  float full_theta = c.has_full_theta ? c.full_rope_theta : (c.has_global_theta ? c.global_rope_theta : 1000000.0f);
  size_t eff_window = c.bidirectional_all ? (size_t)(c.sliding_window / 2 + 1) : (size_t)c.sliding_window;
  size_t global_hd = c.global_head_dim > 0 ? (size_t)c.global_head_dim : (size_t)c.head_dim;
  std::map<std::pair<int64_t, size_t>, int64_t> step_cache;

  for (size_t l = 0; l < m.L; ++l) {
    LayerSpec ls{};
    std::string p = "model.language_model.layers." + std::to_string(l);
    ls.sliding = c.layer_is_sliding[l] != 0;
    ls.head_dim = ls.sliding ? (size_t)c.head_dim : global_hd;
    if (ls.sliding) ls.num_kv_heads = c.num_key_value_heads;
    else if (k_eq_v_cfg) ls.num_kv_heads = c.num_global_key_value_heads > 0 ? c.num_global_key_value_heads : c.num_key_value_heads;
    else ls.num_kv_heads = c.num_key_value_heads;
    ls.rotary_dim = ls.sliding ? ls.head_dim : (size_t)((float)ls.head_dim * partial);
    ls.donor = donor[l];
    ls.window = eff_window;
    ls.cache_trim = ls.sliding && !is_donor[l];
    ls.k_eq_v = !ls.sliding && k_eq_v_cfg;
    ls.rope_base = f32_to_acc(ls.sliding ? local_theta : full_theta);
    if (ls.rotary_dim > 0) {
      if (ls.rotary_dim % 2 != 0) throw Fail("rope_rotate_pairs requires an even rotary_dim");
      if (ls.rotary_dim > ls.head_dim) throw Fail("rotary_dim exceeds head_dim");
      if (ls.head_dim < 2 || ls.head_dim % 2) throw Fail("rope requires an even freq_base_dim");
      if (ls.rope_base <= 0) throw Fail("rope requires a positive base");
      auto key = std::make_pair(ls.rope_base, ls.head_dim);
      auto it = step_cache.find(key);
      if (it == step_cache.end()) it = step_cache.emplace(key, rope_frequency_step(ls.rope_base, ls.head_dim)).first;
      ls.rope_step = it->second;
    }
    ls.q = &need(m, p + ".self_attn.q_proj.weight", 2);
    ls.k = &need(m, p + ".self_attn.k_proj.weight", 2);
    ls.v = nullptr;
    if (ls.k_eq_v) {
      auto it = m.t.find(p + ".self_attn.v_proj.weight");
      if (it != m.t.end()) { if (it->second.shape.size() != 2) throw Fail("v_proj rank"); ls.v = &it->second; }
    } else {
      ls.v = &need(m, p + ".self_attn.v_proj.weight", 2);
    }
    ls.o = &need(m, p + ".self_attn.o_proj.weight", 2);
    ls.gate = &need(m, p + ".mlp.gate_proj.weight", 2);
    ls.up = &need(m, p + ".mlp.up_proj.weight", 2);
    ls.down = &need(m, p + ".mlp.down_proj.weight", 2);
    ls.q_norm = &need(m, p + ".self_attn.q_norm.weight", 1);
    ls.k_norm = &need(m, p + ".self_attn.k_norm.weight", 1);
    ls.in_ln = &need(m, p + ".input_layernorm.weight", 1);
    ls.post_attn_ln = &need(m, p + ".post_attention_layernorm.weight", 1);
    ls.pre_ff_ln = &need(m, p + ".pre_feedforward_layernorm.weight", 1);
    ls.post_ff_ln = &need(m, p + ".post_feedforward_layernorm.weight", 1);
    if (m.P > 0) {
      ls.ple_gate = &need(m, p + ".per_layer_input_gate.weight", 2);
      ls.ple_proj = &need(m, p + ".per_layer_projection.weight", 2);
      ls.ple_norm = &need(m, p + ".post_per_layer_input_norm.weight", 1);
    }
    auto sc = m.t.find(p + ".layer_scalar");
    ls.has_scalar = sc != m.t.end();
    if (ls.has_scalar) {
      if (sc->second.shape != std::vector<size_t>{1}) throw Fail("layer_scalar must have shape [1]");
      ls.scalar = sc->second.at(0);
    }
    if (ls.num_kv_heads == 0) throw Fail("invalid Gemma head configuration");
    if (m.Hq / ls.num_kv_heads == 0) throw Fail("Gemma layer must have at least one KV group");
    m.layers.push_back(ls);
  }
  m.final_norm = &need(m, "model.language_model.norm.weight", 1);
  bool tied = c.tie_word_embeddings != 0;  // default true (io.rs:119)
  m.lm_head = tied ? m.emb : &need(m, "model.language_model.lm_head.weight", 2);
  m.ple_table = m.ple_model_proj = m.ple_proj_norm = nullptr;
  if (m.P > 0) {
    m.ple_table = &need(m, "model.language_model.embed_tokens_per_layer.weight", 2);
    m.ple_model_proj = &need(m, "model.language_model.per_layer_model_projection.weight", 2);
    m.ple_proj_norm = &need(m, "model.language_model.per_layer_projection_norm.weight", 1);
    if (m.ple_table->shape[0] < m.ple_vocab || m.ple_table->shape[1] < m.L * m.P) throw Fail("PLE token embedding slice out of bounds");
    if (m.ple_model_proj->shape[0] < m.L * m.P || m.ple_model_proj->shape[1] < m.H) throw Fail("PLE model projection slice out of bounds");
    // io.rs:1226-1231: sqrt(P), H^-0.5, 2^-0.5 computed in f32, then f32_to_act
    m.ple_emb_scale = f32_to_act(std::sqrt((float)m.P));
    m.ple_proj_scale = f32_to_act(std::pow((float)m.H, -0.5f));
    m.ple_in_scale = f32_to_act(std::pow(2.0f, -0.5f));
  }
  return mp;
}

// ---------------------------------------------------------------------------
// GEMV / linear (det_kernels.rs:108-203): y[r] = requantize(sum_k x[k]*W[r,k])
// ---------------------------------------------------------------------------
static inline int64_t dot_row(const int32_t* x, const Tensor& w, size_t row_start, size_t col_off, size_t k) {
  uint64_t acc = 0;
  if (w.width == 16) {
    const int16_t* p = w.w16.data() + row_start + col_off;
    for (size_t i = 0; i < k; ++i) acc += (uint64_t)((int64_t)x[i] * (int64_t)p[i]);
  } else {
    const int32_t* p = w.w32.data() + row_start + col_off;
    for (size_t i = 0; i < k; ++i) acc += (uint64_t)((int64_t)x[i] * (int64_t)p[i]);
  }
  return (int64_t)acc;
}

// dot_row for four consecutive token rows of X (row stride xs) at once, one
// weight load per four products.
static inline void dot_row4(const int32_t* x, size_t xs, const Tensor& w, size_t row_start, size_t col_off, size_t k,
                            int64_t* out) {
  uint64_t a0 = 0, a1 = 0, a2 = 0, a3 = 0;
  const int32_t *x0 = x, *x1 = x + xs, *x2 = x + 2 * xs, *x3 = x + 3 * xs;
  if (w.width == 16) {
    const int16_t* p = w.w16.data() + row_start + col_off;
    for (size_t i = 0; i < k; ++i) {
      int64_t v = p[i];
      a0 += (uint64_t)((int64_t)x0[i] * v); a1 += (uint64_t)((int64_t)x1[i] * v);
      a2 += (uint64_t)((int64_t)x2[i] * v); a3 += (uint64_t)((int64_t)x3[i] * v);
    }
  } else {
    const int32_t* p = w.w32.data() + row_start + col_off;
    for (size_t i = 0; i < k; ++i) {
      int64_t v = p[i];
      a0 += (uint64_t)((int64_t)x0[i] * v); a1 += (uint64_t)((int64_t)x1[i] * v);
      a2 += (uint64_t)((int64_t)x2[i] * v); a3 += (uint64_t)((int64_t)x3[i] * v);
    }
  }
  out[0] = (int64_t)a0; out[1] = (int64_t)a1; out[2] = (int64_t)a2; out[3] = (int64_t)a3;
}

// rows [row_off, row_off+n) and cols [col_off, col_off+k) of w; X is [S,k].
// Every output is the reference's per-row dot product (det_kernels.rs:180-203
// runs one det_linear_rows_into per token row); the work is only visited in
// blocks of 64 weight rows x 16 token rows so that a block's weight rows stay
// in cache while the block's tokens use them.  Wrapping sums are
// order-independent, so the visiting order does not change any result.
static void linear(const int32_t* X, size_t S, const Tensor& w, size_t row_off, size_t n, size_t col_off, size_t k,
                   int32_t* Y) {
  size_t cols = w.cols();
  const size_t RB = 64, SB = 16;
  size_t nrb = (n + RB - 1) / RB, nsb = (S + SB - 1) / SB;
  parallel_for(nrb * nsb, [&](size_t lo, size_t hi) {
    for (size_t it = lo; it < hi; ++it) {
      size_t r0 = (it / nsb) * RB, r1 = std::min(n, r0 + RB);
      size_t s0 = (it % nsb) * SB, s1 = std::min(S, s0 + SB);
      for (size_t r = r0; r < r1; ++r) {
        size_t s = s0;
        for (; s + 4 <= s1; s += 4) {
          int64_t acc[4];
          dot_row4(X + s * k, k, w, (row_off + r) * cols, col_off, k, acc);
          for (int j = 0; j < 4; ++j) Y[(s + j) * n + r] = requantize(acc[j]);
        }
        for (; s < s1; ++s) Y[s * n + r] = requantize(dot_row(X + s * k, w, (row_off + r) * cols, col_off, k));
      }
    }
  });
}
static void linear_full(const int32_t* X, size_t S, const Tensor& w, int32_t* Y) {
  linear(X, S, w, 0, w.rows(), 0, w.cols(), Y);
}

static std::vector<int32_t> wvec(const Tensor& t) {
  std::vector<int32_t> v(t.w16.size() + t.w32.size());
  for (size_t i = 0; i < v.size(); ++i) v[i] = t.at(i);
  return v;
}

static void rms_rows(int32_t* X, size_t S, size_t n, const std::vector<int32_t>& g, int64_t eps) {
  if (g.size() != n) throw Fail("rms norm width mismatch");
  parallel_for(S, [&](size_t lo, size_t hi) {
    for (size_t s = lo; s < hi; ++s) rms_norm_in_place(X + s * n, g.data(), n, eps);
  });
}

// ---------------------------------------------------------------------------
// KV cache (det_tensor.rs:147-337): per KV head, logical rows with front trim
// ---------------------------------------------------------------------------
struct HeadBuf {
  std::vector<int32_t> data;
  size_t start = 0, len = 0;
  const int32_t* row(size_t i, size_t d) const { return data.data() + (start + i) * d; }
  void push(const int32_t* r, size_t d) { data.insert(data.end(), r, r + d); ++len; }
  void pop_front(size_t d) {
    ++start; --len;
    if (start > len) { data.erase(data.begin(), data.begin() + start * d); start = 0; }
  }
};
struct LayerCache {
  bool det = false;
  size_t heads = 0, d = 0;
  std::vector<HeadBuf> k, v;
  size_t len() const { return k.empty() ? 0 : k[0].len; }
};
struct Seq {
  std::vector<LayerCache> caches;
  size_t position = 0, token_count = 0;
  bool prefilled = false;
};

// attention_output_into (det_kernels.rs:340-367) for one query over rows
// [start, start+rows) of one KV head.
static void attend(const int32_t* q, const HeadBuf& kb, const HeadBuf& vb, size_t start, size_t rows, size_t d,
                   int32_t* out, std::vector<int32_t>& logits, std::vector<int64_t>& ex, std::vector<int32_t>& w) {
  logits.resize(rows); ex.resize(rows); w.resize(rows);
  for (size_t j = 0; j < rows; ++j) {
    const int32_t* kr = kb.row(start + j, d);
    uint64_t a = 0;
    for (size_t i = 0; i < d; ++i) a += (uint64_t)((int64_t)q[i] * (int64_t)kr[i]);
    logits[j] = requantize((int64_t)a);
  }
  attention_softmax(logits.data(), rows, ex.data(), w.data());
  for (size_t i = 0; i < d; ++i) {
    uint64_t a = 0;
    for (size_t j = 0; j < rows; ++j) a += (uint64_t)((int64_t)vb.row(start + j, d)[i] * (int64_t)w[j]);
    out[i] = requantize((int64_t)a);
  }
}

// ---------------------------------------------------------------------------
// embedding (io.rs:2446-2518)
// ---------------------------------------------------------------------------
static void embed(const Model& m, const uint32_t* ids, size_t n, int32_t* out) {
  if (n == 0) throw Fail("transformer embedding requires at least one token id");
  size_t H = m.emb->shape[1];
  for (size_t i = 0; i < n; ++i) {
    if (ids[i] >= m.emb->shape[0]) throw Fail("token id " + std::to_string(ids[i]) + " is out of bounds for embedding tensor");
    for (size_t j = 0; j < H; ++j) out[i * H + j] = scale_act(m.emb->at((size_t)ids[i] * H + j), m.emb_scale);
  }
}

// PLE input for one token row (prefill_prepare_aux/native/tiles.rs:189-235 and
// det_kernels.rs:1142-1208 — the same arithmetic): x0 = embedded input row.
static void ple_input_rows(const Model& m, size_t l, const uint32_t* ids, const int32_t* x0, size_t S, int32_t* out) {
  size_t P = m.P, H = m.H;
  linear(x0, S, *m.ple_model_proj, l * P, P, 0, H, out);
  std::vector<int32_t> g = wvec(*m.ple_proj_norm);
  size_t tcols = m.ple_table->shape[1];
  for (size_t s = 0; s < S; ++s) {
    if (ids[s] >= m.ple_vocab) throw Fail("PLE token id out of bounds");
    int32_t* row = out + s * P;
    for (size_t i = 0; i < P; ++i) row[i] = scale_act(row[i], m.ple_proj_scale);
    rms_norm_in_place(row, g.data(), P, m.eps);
    for (size_t i = 0; i < P; ++i) {
      int32_t e = scale_act(m.ple_table->at((size_t)ids[s] * tcols + l * P + i), m.ple_emb_scale);
      row[i] = scale_act(add_sat(e, row[i]), m.ple_in_scale);
    }
  }
}

// ---------------------------------------------------------------------------
// layer prefill (det_kernels.rs:499-821)
// ---------------------------------------------------------------------------
static void layer_prefill(const Model& m, size_t l, std::vector<int32_t>& xs, size_t S, const int32_t* ple_in,
                          std::vector<LayerCache>& caches) {
  const LayerSpec& L = m.layers[l];
  size_t H = m.H, Hq = m.Hq, d = L.head_dim, Hkv = L.num_kv_heads, groups = Hq / Hkv;
  if (groups == 0) throw Fail("Gemma layer must have at least one KV group");
  std::vector<int32_t> normed = xs;
  rms_rows(normed.data(), S, H, wvec(*L.in_ln), m.eps);

  std::vector<int32_t> q(S * Hq * d);
  if (L.q->rows() != Hq * d || L.q->cols() != H) throw Fail("q_proj shape mismatch");
  linear_full(normed.data(), S, *L.q, q.data());
  std::vector<int32_t> qn = wvec(*L.q_norm), kn = wvec(*L.k_norm);
  for (size_t r = 0; r < S * Hq; ++r) rms_norm_in_place(q.data() + r * d, qn.data(), d, m.eps);

  LayerCache own;
  const LayerCache* kvsrc;
  if (L.donor >= 0) {
    // Donor-sharing layers attend over the donor's cache; their own K/V
    // projections do not affect any output and are skipped.
    kvsrc = &caches[L.donor];
    if (!kvsrc->det) throw Fail("deterministic attention requires canonical key cache rows");
  } else {
    std::vector<int32_t> k(S * Hkv * d), v(S * Hkv * d);
    if (L.k->rows() != Hkv * d) throw Fail("k_proj shape mismatch");
    linear_full(normed.data(), S, *L.k, k.data());
    if (L.v) linear_full(normed.data(), S, *L.v, v.data());
    else if (L.k_eq_v) v = k;  // raw K before norms (det_kernels.rs:517-518)
    else throw Fail("Gemma layer is missing v_proj without attention_k_eq_v enabled");
    for (size_t r = 0; r < S * Hkv; ++r) {
      rms_norm_in_place(k.data() + r * d, kn.data(), d, m.eps);
      value_rms_norm_in_place(v.data() + r * d, d, m.eps);
    }
    for (size_t s = 0; s < S; ++s)
      for (size_t h = 0; h < Hkv; ++h) rope_rotate_with_step(k.data() + (s * Hkv + h) * d, L.rotary_dim, L.rope_step, s);
    size_t retained = L.cache_trim ? (S > L.window ? S - L.window : 0) : 0;
    own.det = true; own.heads = Hkv; own.d = d;
    own.k.resize(Hkv); own.v.resize(Hkv);
    // Attention reads the full S rows; the cache keeps the tail only.
    LayerCache full = own;
    for (size_t h = 0; h < Hkv; ++h)
      for (size_t s = 0; s < S; ++s) {
        full.k[h].push(k.data() + (s * Hkv + h) * d, d);
        full.v[h].push(v.data() + (s * Hkv + h) * d, d);
        if (s >= retained) { own.k[h].push(k.data() + (s * Hkv + h) * d, d); own.v[h].push(v.data() + (s * Hkv + h) * d, d); }
      }
    caches[l] = std::move(full);
    kvsrc = &caches[l];
  }
  for (size_t s = 0; s < S; ++s)
    for (size_t h = 0; h < Hq; ++h) rope_rotate_with_step(q.data() + (s * Hq + h) * d, L.rotary_dim, L.rope_step, s);

  std::vector<int32_t> comb(S * Hq * d);
  bool windowed = L.sliding;
  parallel_for(Hq * S, [&](size_t lo, size_t hi) {
    std::vector<int32_t> lg, w;
    std::vector<int64_t> ex;
    for (size_t it = lo; it < hi; ++it) {
      size_t h = it / S, i = it % S, kv = h / groups;
      size_t start = windowed ? ((i + 1) > L.window ? i + 1 - L.window : 0) : 0;
      size_t cnt = i + 1 - start;
      size_t avail = kvsrc->len();
      size_t st = std::min(start, avail);
      size_t rows = std::min(cnt, avail - st);
      attend(q.data() + (i * Hq + h) * d, kvsrc->k[kv], kvsrc->v[kv], st, rows, d, comb.data() + (i * Hq + h) * d, lg, ex, w);
    }
  });
  if (L.donor < 0) caches[l] = std::move(own);
  else { caches[l] = LayerCache(); caches[l].heads = Hkv; }

  std::vector<int32_t> attn(S * H);
  linear_full(comb.data(), S, *L.o, attn.data());
  rms_rows(attn.data(), S, H, wvec(*L.post_attn_ln), m.eps);
  for (size_t i = 0; i < S * H; ++i) attn[i] = add_sat(attn[i], xs[i]);
  xs.swap(attn);

  std::vector<int32_t> nrm = xs;
  rms_rows(nrm.data(), S, H, wvec(*L.pre_ff_ln), m.eps);
  size_t F = L.gate->rows();
  std::vector<int32_t> gate(S * F), up(S * F);
  linear_full(nrm.data(), S, *L.gate, gate.data());
  linear_full(nrm.data(), S, *L.up, up.data());
  for (size_t i = 0; i < S * F; ++i) gate[i] = mul_sat(gelu_act(gate[i]), up[i]);
  std::vector<int32_t> ff(S * H);
  linear_full(gate.data(), S, *L.down, ff.data());
  rms_rows(ff.data(), S, H, wvec(*L.post_ff_ln), m.eps);
  for (size_t i = 0; i < S * H; ++i) ff[i] = add_sat(ff[i], xs[i]);
  xs.swap(ff);

  if (m.P > 0 && ple_in) {
    size_t P = m.P;
    std::vector<int32_t> g(S * P);
    linear_full(xs.data(), S, *L.ple_gate, g.data());
    for (size_t i = 0; i < S * P; ++i) g[i] = mul_sat(gelu_act(g[i]), ple_in[i]);
    std::vector<int32_t> pr(S * H);
    linear_full(g.data(), S, *L.ple_proj, pr.data());
    rms_rows(pr.data(), S, H, wvec(*L.ple_norm), m.eps);
    for (size_t i = 0; i < S * H; ++i) pr[i] = add_sat(pr[i], xs[i]);
    xs.swap(pr);
  }
  if (L.has_scalar)
    for (auto& x : xs) x = scale_act(x, L.scalar);
}

// ---------------------------------------------------------------------------
// layer decode (det_kernels.rs:866-1133)
// ---------------------------------------------------------------------------
static void layer_decode(const Model& m, size_t l, std::vector<int32_t>& x, const int32_t* ple_in, Seq& sq) {
  const LayerSpec& L = m.layers[l];
  size_t H = m.H, Hq = m.Hq, d = L.head_dim, Hkv = L.num_kv_heads, groups = Hq / Hkv;
  if (groups == 0) throw Fail("Gemma layer must have at least one KV group");
  std::vector<int32_t> normed = x;
  rms_norm_in_place(normed.data(), wvec(*L.in_ln).data(), H, m.eps);
  std::vector<int32_t> q(Hq * d);
  linear_full(normed.data(), 1, *L.q, q.data());
  std::vector<int32_t> qn = wvec(*L.q_norm), kn = wvec(*L.k_norm);
  for (size_t h = 0; h < Hq; ++h) rms_norm_in_place(q.data() + h * d, qn.data(), d, m.eps);
  for (size_t h = 0; h < Hq; ++h) rope_rotate_with_step(q.data() + h * d, L.rotary_dim, L.rope_step, sq.position);

  LayerCache& own = sq.caches[l];
  if (L.donor < 0) {
    std::vector<int32_t> k(Hkv * d), v(Hkv * d);
    linear_full(normed.data(), 1, *L.k, k.data());
    if (L.v) linear_full(normed.data(), 1, *L.v, v.data());
    else if (L.k_eq_v) v = k;
    else throw Fail("Gemma layer is missing v_proj without attention_k_eq_v enabled");
    for (size_t h = 0; h < Hkv; ++h) {
      rms_norm_in_place(k.data() + h * d, kn.data(), d, m.eps);
      value_rms_norm_in_place(v.data() + h * d, d, m.eps);
      rope_rotate_with_step(k.data() + h * d, L.rotary_dim, L.rope_step, sq.position);
    }
    if (!own.det) { own.det = true; own.heads = Hkv; own.d = d; own.k.assign(Hkv, HeadBuf()); own.v.assign(Hkv, HeadBuf()); }
    for (size_t h = 0; h < Hkv; ++h) {
      own.k[h].push(k.data() + h * d, d);
      own.v[h].push(v.data() + h * d, d);
      if (L.cache_trim)
        while (own.k[h].len > L.window) { own.k[h].pop_front(d); own.v[h].pop_front(d); }
    }
  }
  const LayerCache& ac = L.donor >= 0 ? sq.caches[L.donor] : own;
  if (!ac.det) throw Fail("deterministic attention requires canonical key cache rows");
  size_t len = ac.len();
  size_t key_start = L.sliding ? (len > L.window ? len - L.window : 0) : 0;
  size_t wl = len - key_start;
  std::vector<int32_t> comb(Hq * d);
  parallel_for(Hq, [&](size_t lo, size_t hi) {
    std::vector<int32_t> lg, w;
    std::vector<int64_t> ex;
    for (size_t h = lo; h < hi; ++h) {
      size_t kv = h / groups;
      attend(q.data() + h * d, ac.k[kv], ac.v[kv], key_start, wl, d, comb.data() + h * d, lg, ex, w);
    }
  });
  std::vector<int32_t> attn(H);
  linear_full(comb.data(), 1, *L.o, attn.data());
  rms_norm_in_place(attn.data(), wvec(*L.post_attn_ln).data(), H, m.eps);
  std::vector<int32_t> xs(H);
  for (size_t i = 0; i < H; ++i) xs[i] = add_sat(x[i], attn[i]);

  std::vector<int32_t> nrm = xs;
  rms_norm_in_place(nrm.data(), wvec(*L.pre_ff_ln).data(), H, m.eps);
  size_t F = L.gate->rows();
  std::vector<int32_t> gate(F), up(F);
  linear_full(nrm.data(), 1, *L.gate, gate.data());
  linear_full(nrm.data(), 1, *L.up, up.data());
  for (size_t i = 0; i < F; ++i) gate[i] = mul_sat(gelu_act(gate[i]), up[i]);
  std::vector<int32_t> ff(H);
  linear_full(gate.data(), 1, *L.down, ff.data());
  rms_norm_in_place(ff.data(), wvec(*L.post_ff_ln).data(), H, m.eps);
  for (size_t i = 0; i < H; ++i) xs[i] = add_sat(xs[i], ff[i]);

  if (m.P > 0 && ple_in) {
    size_t P = m.P;
    std::vector<int32_t> g(P);
    linear_full(xs.data(), 1, *L.ple_gate, g.data());
    for (size_t i = 0; i < P; ++i) g[i] = mul_sat(gelu_act(g[i]), ple_in[i]);
    std::vector<int32_t> pr(H);
    linear_full(g.data(), 1, *L.ple_proj, pr.data());
    rms_norm_in_place(pr.data(), wvec(*L.ple_norm).data(), H, m.eps);
    for (size_t i = 0; i < H; ++i) xs[i] = add_sat(xs[i], pr[i]);
  }
  if (L.has_scalar)
    for (auto& v : xs) v = scale_act(v, L.scalar);
  x.swap(xs);
}

// det_hidden_to_logits (det_kernels.rs:1217-1267)
static void hidden_to_logits(const Model& m, const int32_t* hidden, int32_t* logits) {
  std::vector<int32_t> n(hidden, hidden + m.H);
  rms_norm_in_place(n.data(), wvec(*m.final_norm).data(), m.H, m.eps);
  if (m.lm_head->cols() != m.H) throw Fail("logits projection input width mismatch");
  linear_full(n.data(), 1, *m.lm_head, logits);
  if (m.has_softcap)
    for (size_t i = 0; i < m.lm_head->rows(); ++i) logits[i] = softcap_act(logits[i], m.softcap);
}

// ---------------------------------------------------------------------------
// commitments (transformer_kernels.rs:1395-1482)
// ---------------------------------------------------------------------------
static std::string act_commitment(const int32_t* x, size_t rows, size_t cols) {
  Sha256 h;
  h.update("raster-det-num-act-v1", 21);
  h.update_u64(rows);
  for (size_t r = 0; r < rows; ++r) { h.update_u64(cols); h.update_i32s(x + r * cols, cols); }
  return h.hex();
}
static std::string vec_commitment(const int32_t* x, size_t n) {
  Sha256 h;
  h.update("raster-det-num-act-vector-v1", 28);
  h.update_u64(n);
  h.update_i32s(x, n);
  return h.hex();
}
// build_det_kv_cache_commitment (transformer_kernels.rs:1460-1482) over the
// caches of the first nl layers (all layers when nl is 0)
static bool kv_commitment(const Seq& sq, std::string* out, size_t nl = 0) {
  if (nl == 0 || nl > sq.caches.size()) nl = sq.caches.size();
  Sha256 h;
  h.update("raster-det-num-kv-cache-v1", 26);
  h.update_u64(nl);
  for (size_t l = 0; l < nl; ++l) {
    const LayerCache& c = sq.caches[l];
    if (!c.det) return false;
    h.update_u64(c.heads);
    for (int kind = 0; kind < 2; ++kind) {
      const std::vector<HeadBuf>& hb = kind == 0 ? c.k : c.v;
      h.update(kind == 0 ? "k" : "v", 1);
      h.update_u64(hb.size());
      for (const HeadBuf& b : hb) {
        h.update_u64(b.len);
        for (size_t r = 0; r < b.len; ++r) { h.update_u64(c.d); h.update_i32s(b.row(r, c.d), c.d); }
      }
    }
  }
  *out = h.hex();
  return true;
}

// ---------------------------------------------------------------------------
// C API
// ---------------------------------------------------------------------------
static void set_err(char* err, size_t len, const std::string& m) {
  if (err && len) { snprintf(err, len, "%s", m.c_str()); }
}
static void put_hash(char* dst, const std::string& h) { memcpy(dst, h.c_str(), 65); }

extern "C" {

struct dor_model { std::unique_ptr<Model> m; };
struct dor_seq { Seq s; };

void dor_set_threads(int n) {
  int t = n < 1 ? 1 : n;
  if (t != g_threads) { g_threads = t; g_pool.resize(t); }
}
int dor_get_threads(void) { return g_threads; }

dor_model* dor_model_open(const char* path, const dor_config* cfg, char* err, size_t errlen) {
  try {
    FILE* f = fopen(path, "rb");
    if (!f) throw Fail(std::string("failed to open deterministic artifact ") + path);
    std::vector<uint8_t> bytes;
    fseek(f, 0, SEEK_END);
    long sz = ftell(f);
    fseek(f, 0, SEEK_SET);
    bytes.resize((size_t)sz);
    size_t got = sz > 0 ? fread(bytes.data(), 1, (size_t)sz, f) : 0;
    fclose(f);
    if (got != (size_t)sz) throw Fail("short read");
    auto t = read_detwgt(bytes);
    auto* h = new dor_model;
    h->m = build_model(std::move(t), *cfg);
    return h;
  } catch (const std::exception& e) {
    set_err(err, errlen, e.what());
    return nullptr;
  }
}
// Fail-closed parse of an in-memory artifact; returns tensor count or -1.
long dor_detwgt_validate(const uint8_t* bytes, size_t n, char* err, size_t errlen) {
  try {
    std::vector<uint8_t> b(bytes, bytes + n);
    return (long)read_detwgt(b).size();
  } catch (const std::exception& e) {
    set_err(err, errlen, e.what());
    return -1;
  }
}
// Seeded synthetic model: the counter-based generator of
// raster-inference_b200/detwgt.py (the same tensor names, shapes and values as
// detwgt.write_synthetic_model), filled on all oracle threads.
static uint64_t fnv1a64(const std::string& s) {
  uint64_t h = 0xCBF29CE484222325ull;
  for (unsigned char c : s) { h ^= c; h *= 0x100000001B3ull; }
  return h;
}
static uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
static Tensor synth_tensor(const std::string& name, std::vector<size_t> shape, uint64_t seed, int width) {
  Tensor t;
  t.shape = shape;
  size_t n = 1;
  for (size_t d : shape) n *= d;
  t.width = shape.size() == 1 ? 32 : width;
  if (t.width == 16) t.w16.resize(n); else t.w32.resize(n);
  uint64_t key = fnv1a64(name) ^ seed;
  int64_t bound = (int64_t)(0x7fffffffLL / (int64_t)shape.back());
  bool rank1 = shape.size() == 1;
  parallel_for((n + 4095) / 4096, [&](size_t lo, size_t hi) {
    for (size_t b = lo; b < hi; ++b)
      for (size_t i = b * 4096; i < std::min(n, (b + 1) * 4096); ++i) {
        uint64_t z = mix64(key + (uint64_t)(i + 1) * 0x9E3779B97F4A7C15ull);
        int32_t v;
        if (rank1) v = 32768 + (int32_t)(z >> 48);
        else if (width == 16) v = (int32_t)(z >> 48) - 32768;
        else v = (int32_t)((int64_t)(z % (uint64_t)(2 * bound + 1)) - bound);
        if (t.width == 16) t.w16[i] = (int16_t)v; else t.w32[i] = v;
      }
  });
  return t;
}

dor_model* dor_model_open_synthetic(const dor_config* c, uint64_t seed, int width, int intermediate_size,
                                    int with_scalar, char* err, size_t errlen) {
  try {
    std::map<std::string, Tensor> t;
    size_t H = c->hidden_size, V = c->vocab_size, L = c->num_hidden_layers, Hq = c->num_attention_heads;
    size_t F = intermediate_size, P = c->hidden_size_per_layer_input > 0 ? c->hidden_size_per_layer_input : 0;
    size_t dg = c->global_head_dim > 0 ? c->global_head_dim : c->head_dim;
    bool keqv = c->attention_k_eq_v == 1;
    size_t gkv = c->num_global_key_value_heads > 0 ? c->num_global_key_value_heads : c->num_key_value_heads;
    size_t pv = c->vocab_size_per_layer_input >= 0 ? c->vocab_size_per_layer_input : V;
    auto add = [&](const std::string& n, std::vector<size_t> sh) { t.emplace(n, synth_tensor(n, sh, seed, width)); };
    add("model.language_model.embed_tokens.weight", {V, H});
    for (size_t l = 0; l < L; ++l) {
      bool sl = c->layer_is_sliding[l] != 0;
      size_t hd = sl ? (size_t)c->head_dim : dg;
      size_t nkv = sl ? (size_t)c->num_key_value_heads : (keqv ? gkv : (size_t)c->num_key_value_heads);
      std::string p = "model.language_model.layers." + std::to_string(l);
      add(p + ".self_attn.q_proj.weight", {Hq * hd, H});
      add(p + ".self_attn.k_proj.weight", {nkv * hd, H});
      if (sl || !keqv) add(p + ".self_attn.v_proj.weight", {nkv * hd, H});
      add(p + ".self_attn.o_proj.weight", {H, Hq * hd});
      add(p + ".self_attn.q_norm.weight", {hd});
      add(p + ".self_attn.k_norm.weight", {hd});
      for (const char* nn : {"input_layernorm", "post_attention_layernorm", "pre_feedforward_layernorm",
                             "post_feedforward_layernorm"})
        add(p + "." + nn + ".weight", {H});
      add(p + ".mlp.gate_proj.weight", {F, H});
      add(p + ".mlp.up_proj.weight", {F, H});
      add(p + ".mlp.down_proj.weight", {H, F});
      if (P > 0) {
        add(p + ".per_layer_input_gate.weight", {P, H});
        add(p + ".per_layer_projection.weight", {H, P});
        add(p + ".post_per_layer_input_norm.weight", {H});
      }
      if (with_scalar) add(p + ".layer_scalar", {1});
    }
    if (P > 0) {
      add("model.language_model.embed_tokens_per_layer.weight", {pv, L * P});
      add("model.language_model.per_layer_model_projection.weight", {L * P, H});
      add("model.language_model.per_layer_projection_norm.weight", {P});
    }
    add("model.language_model.norm.weight", {H});
    if (c->tie_word_embeddings == 0) add("model.language_model.lm_head.weight", {V, H});
    auto* h = new dor_model;
    h->m = build_model(std::move(t), *c);
    return h;
  } catch (const std::exception& e) {
    set_err(err, errlen, e.what());
    return nullptr;
  }
}

void dor_model_close(dor_model* h) { delete h; }
// info: H, V, L, Hq, P, then per layer: head_dim, kv_heads, rotary, sliding, window, cache_trim, donor, k_eq_v
int dor_model_info(const dor_model* h, int64_t* out, size_t cap) {
  const Model& m = *h->m;
  std::vector<int64_t> v = {(int64_t)m.H, (int64_t)m.lm_head->rows(), (int64_t)m.L, (int64_t)m.Hq, (int64_t)m.P};
  for (auto& l : m.layers) {
    v.insert(v.end(), {(int64_t)l.head_dim, (int64_t)l.num_kv_heads, (int64_t)l.rotary_dim, (int64_t)l.sliding,
                       (int64_t)l.window, (int64_t)l.cache_trim, (int64_t)l.donor, (int64_t)l.k_eq_v});
  }
  for (size_t i = 0; i < v.size() && i < cap; ++i) out[i] = v[i];
  return (int)v.size();
}

dor_seq* dor_seq_new(const dor_model* h) {
  auto* s = new dor_seq;
  s->s.caches.resize(h->m->L);
  return s;
}
void dor_seq_free(dor_seq* s) { delete s; }
int64_t dor_seq_position(const dor_seq* s) { return (int64_t)s->s.position; }

int dor_embed(const dor_model* h, const uint32_t* ids, size_t n, int32_t* out, char* err, size_t errlen) {
  try { embed(*h->m, ids, n, out); return 0; }
  catch (const std::exception& e) { set_err(err, errlen, e.what()); return -1; }
}

// Full prefill (input.embedding -> prefill_prepare_aux -> prefill.range over
// all layers -> prefill.finalize).  Outputs are optional (NULL to skip):
// hidden [n*H] final hidden states, logits [V], layer_hashes [L*65] per-layer
// slab commitments, final_hash[65] slab commitment of the final hidden states.
int dor_prefill(const dor_model* h, dor_seq* sq, const uint32_t* ids, size_t n, int32_t* hidden, int32_t* logits,
                char* layer_hashes, char* err, size_t errlen) {
  try {
    const Model& m = *h->m;
    Seq& s = sq->s;
    if (n == 0) throw Fail("transformer prefill requires at least one token");
    std::vector<int32_t> x0(n * m.H);
    embed(m, ids, n, x0.data());
    std::vector<std::vector<int32_t>> ple(m.L);
    if (m.P > 0)
      for (size_t l = 0; l < m.L; ++l) { ple[l].resize(n * m.P); ple_input_rows(m, l, ids, x0.data(), n, ple[l].data()); }
    std::vector<int32_t> xs = x0;
    s.caches.assign(m.L, LayerCache());
    for (size_t l = 0; l < m.L; ++l) {
      layer_prefill(m, l, xs, n, m.P > 0 ? ple[l].data() : nullptr, s.caches);
      if (layer_hashes) put_hash(layer_hashes + 65 * l, act_commitment(xs.data(), n, m.H));
    }
    if (hidden) memcpy(hidden, xs.data(), xs.size() * 4);
    if (logits) hidden_to_logits(m, xs.data() + (n - 1) * m.H, logits);
    s.position = n;
    s.token_count = n;
    s.prefilled = true;
    return 0;
  } catch (const std::exception& e) { set_err(err, errlen, e.what()); return -1; }
}

// One decode transition (decode_layer_range over all layers +
// decode_transition_finalize): hidden [H] layer-stack output, logits [V],
// layer_hashes [L*65] per-layer row commitments.
int dor_decode(const dor_model* h, dor_seq* sq, uint32_t token, int32_t* hidden, int32_t* logits, char* layer_hashes,
               char* err, size_t errlen) {
  try {
    const Model& m = *h->m;
    Seq& s = sq->s;
    if (!s.prefilled) throw Fail("decode requires a prefilled sequence");
    std::vector<int32_t> x0(m.H);
    embed(m, &token, 1, x0.data());
    std::vector<int32_t> x = x0, ple(m.P);
    for (size_t l = 0; l < m.L; ++l) {
      if (m.P > 0) ple_input_rows(m, l, &token, x0.data(), 1, ple.data());
      layer_decode(m, l, x, m.P > 0 ? ple.data() : nullptr, s);
      if (layer_hashes) put_hash(layer_hashes + 65 * l, act_commitment(x.data(), 1, m.H));
    }
    if (hidden) memcpy(hidden, x.data(), m.H * 4);
    if (logits) hidden_to_logits(m, x.data(), logits);
    s.position += 1;
    s.token_count += 1;
    return 0;
  } catch (const std::exception& e) { set_err(err, errlen, e.what()); return -1; }
}

// Fills a prefilled-looking KV cache of `ctx` rows per layer with seeded
// values (for timing decode at long context without a full CPU prefill).
int dor_seq_fill_synthetic(const dor_model* h, dor_seq* sq, size_t ctx, uint64_t seed) {
  const Model& m = *h->m;
  Seq& s = sq->s;
  s.caches.assign(m.L, LayerCache());
  uint64_t st = seed | 1;
  for (size_t l = 0; l < m.L; ++l) {
    const LayerSpec& L = m.layers[l];
    if (L.donor >= 0) { s.caches[l].heads = L.num_kv_heads; continue; }
    LayerCache& c = s.caches[l];
    c.det = true; c.heads = L.num_kv_heads; c.d = L.head_dim;
    c.k.resize(c.heads); c.v.resize(c.heads);
    size_t rows = L.cache_trim ? std::min(ctx, L.window) : ctx;
    std::vector<int32_t> r(L.head_dim);
    for (size_t hh = 0; hh < c.heads; ++hh)
      for (size_t i = 0; i < rows; ++i) {
        for (auto& v : r) { st ^= st << 13; st ^= st >> 7; st ^= st << 17; v = (int32_t)(st >> 48) - 32768; }
        c.k[hh].push(r.data(), L.head_dim);
        c.v[hh].push(r.data(), L.head_dim);
      }
  }
  s.position = ctx;
  s.token_count = ctx;
  s.prefilled = true;
  return 0;
}

int dor_kv_commitment(const dor_seq* sq, char* out) {
  std::string hx;
  if (!kv_commitment(sq->s, &hx)) return 1;
  put_hash(out, hx);
  return 0;
}
// the commitment over the caches of layers [0, layers)
int dor_kv_commitment_prefix(const dor_seq* sq, size_t layers, char* out) {
  std::string hx;
  if (!kv_commitment(sq->s, &hx, layers)) return 1;
  put_hash(out, hx);
  return 0;
}
// rows of one (layer, kv head, kind 0=k 1=v): copies up to cap values, returns rows or -1
long dor_kv_read(const dor_seq* sq, int layer, int head, int kind, int32_t* out, size_t cap) {
  const Seq& s = sq->s;
  if (layer < 0 || (size_t)layer >= s.caches.size()) return -1;
  const LayerCache& c = s.caches[layer];
  if (!c.det || head < 0 || (size_t)head >= c.heads) return -1;
  const HeadBuf& b = kind == 0 ? c.k[head] : c.v[head];
  for (size_t r = 0; r < b.len && (r + 1) * c.d <= cap; ++r) memcpy(out + r * c.d, b.row(r, c.d), c.d * 4);
  return (long)b.len;
}

// attention_output_into (det_kernels.rs:340-367) for one query over `rows`
// key/value rows of width d.
void dor_attention_one(const int32_t* q, const int32_t* keys, const int32_t* values, size_t rows, size_t d,
                       int32_t* out) {
  HeadBuf kb, vb;
  for (size_t j = 0; j < rows; ++j) { kb.push(keys + j * d, d); vb.push(values + j * d, d); }
  std::vector<int32_t> lg, w;
  std::vector<int64_t> ex;
  attend(q, kb, vb, 0, rows, d, out, lg, ex, w);
}

uint32_t dor_argmax_first(const int32_t* x, size_t n) { return (uint32_t)argmax_first(x, n); }
void dor_act_commitment(const int32_t* x, size_t rows, size_t cols, char* out) { put_hash(out, act_commitment(x, rows, cols)); }
void dor_vec_commitment(const int32_t* x, size_t n, char* out) { put_hash(out, vec_commitment(x, n)); }
void dor_sha256_hex(const uint8_t* b, size_t n, char* out) { Sha256 h; h.update(b, n); put_hash(out, h.hex()); }

// GEMV over a raw weight array (width 16 or 32), rows N x cols K.
void dor_gemv(const int32_t* x, const void* w, int width, size_t N, size_t K, int32_t* y) {
  Tensor t;
  t.shape = {N, K};
  t.width = width;
  if (width == 16) t.w16.assign((const int16_t*)w, (const int16_t*)w + N * K);
  else t.w32.assign((const int32_t*)w, (const int32_t*)w + N * K);
  linear_full(x, 1, t, y);
}
// batched linear: X [S,K] -> Y [S,N]
void dor_linear(const int32_t* X, size_t S, const void* w, int width, size_t N, size_t K, int32_t* Y) {
  Tensor t;
  t.shape = {N, K};
  t.width = width;
  if (width == 16) t.w16.assign((const int16_t*)w, (const int16_t*)w + N * K);
  else t.w32.assign((const int32_t*)w, (const int32_t*)w + N * K);
  linear_full(X, S, t, Y);
}

// scalar / row ops for the known-answer tests
int32_t dor_requantize(int64_t a) { return requantize(a); }
int64_t dor_rshift_rte(int64_t a, uint32_t s) { return rshift_rte(a, s); }
int64_t dor_mac_bits(int64_t acc, int32_t a, int32_t b) { return mac_bits(acc, a, b); }
int64_t dor_acc_combine(int64_t a, int64_t b) { return acc_combine(a, b); }
int32_t dor_add_sat(int32_t a, int32_t b) { return add_sat(a, b); }
int32_t dor_sub_sat(int32_t a, int32_t b) { return sub_sat(a, b); }
int64_t dor_acc_add_sat(int64_t a, int64_t b) { return acc_add_sat(a, b); }
int32_t dor_mul_sat(int32_t a, int32_t b) { return mul_sat(a, b); }
int32_t dor_div_act(int32_t a, int32_t b) { return div_act(a, b); }
int64_t dor_div_acc_by_u32(int64_t a, uint32_t d) { return div_acc_by_u32(a, d); }
int32_t dor_tanh(int32_t x) { return tanh_act(x); }
int32_t dor_softcap(int32_t x, int32_t c) { return softcap_act(x, c); }
int32_t dor_gelu(int32_t x) { return gelu_act(x); }
int32_t dor_f32_to_act(float x) { return f32_to_act(x); }
int64_t dor_f32_to_acc(float x) { return f32_to_acc(x); }
int32_t dor_rms_norm_scale(const int32_t* x, size_t n, int64_t eps) { return rms_norm_scale(x, n, eps); }
void dor_rms_norm(int32_t* x, const int32_t* w, size_t n, int64_t eps) { rms_norm_in_place(x, w, n, eps); }
void dor_value_rms_norm(int32_t* x, size_t n, int64_t eps) { value_rms_norm_in_place(x, n, eps); }
void dor_softmax(const int32_t* logits, size_t n, int32_t* w) {
  std::vector<int64_t> ex(n);
  attention_softmax(logits, n, ex.data(), w);
}
int64_t dor_softmax_exp_term(int32_t logit, int32_t max_logit) { return attention_softmax_exp_term(logit, max_logit); }
int64_t dor_rope_step(int64_t base, size_t freq_base_dim) { return rope_frequency_step(base, freq_base_dim); }
void dor_rope(int32_t* v, size_t rotary_dim, size_t freq_base_dim, int64_t base, size_t position) {
  if (rotary_dim == 0 || position == 0) return;
  rope_rotate_with_step(v, rotary_dim, rope_frequency_step(base, freq_base_dim), position);
}
void dor_sin_cos(int64_t angle, int32_t* c, int32_t* s) { sin_cos_acc(angle, c, s); }
int32_t dor_attention_score(const int32_t* q, const int32_t* k, size_t n) {
  uint64_t a = 0;
  for (size_t i = 0; i < n; ++i) a += (uint64_t)((int64_t)q[i] * (int64_t)k[i]);
  return requantize((int64_t)a);
}
// weighted sum: out[i] = requantize(sum_j v[j*width+i]*w[j])
void dor_weighted_sum(const int32_t* w, size_t rows, const int32_t* v, size_t width, int32_t* out) {
  for (size_t i = 0; i < width; ++i) {
    uint64_t a = 0;
    for (size_t j = 0; j < rows; ++j) a += (uint64_t)((int64_t)v[j * width + i] * (int64_t)w[j]);
    out[i] = requantize((int64_t)a);
  }
}

}  // extern "C"
