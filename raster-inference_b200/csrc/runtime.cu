// rdet runtime: model loading into HBM, per-sequence KV caches, and the
// prefill / decode / select routines of the reference det path, composed
// from the sm_100a kernels in kernels.cu.  Implements include/rdet.h.
#include <dlfcn.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <condition_variable>
#include <cstdio>
#include <cstring>
#include <deque>
#include <functional>
#include <map>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include <nccl.h>  // types only: libnccl is loaded at run time

#include "det_dev.cuh"
#include "json.h"
#include "kernels.h"
#include "rdet.h"
#include "sha256.h"

namespace rdet {

// ---------------------------------------------------------------------------
// errors
// ---------------------------------------------------------------------------
struct Fail {
  int code;
  std::string msg;
};
static thread_local std::string g_last_error;

#define CK(x)                                                                                     \
  do {                                                                                            \
    cudaError_t e_ = (x);                                                                         \
    if (e_ != cudaSuccess) throw Fail{RDET_E_CUDA, std::string(#x) + ": " + cudaGetErrorString(e_)}; \
  } while (0)
#define REQUIRE(cond, code, msg) \
  do {                           \
    if (!(cond)) throw Fail{code, msg}; \
  } while (0)

// ---------------------------------------------------------------------------
// host-side det conversions for load-time constants
// (reference det_num/convert.rs:82-189, ops.rs:555-611)
// ---------------------------------------------------------------------------
typedef __int128 i128;
typedef unsigned __int128 u128;

static i128 f32_fixed(float x, int frac, u128 maxpos, u128 maxneg) {
  uint32_t bits;
  memcpy(&bits, &x, 4);
  REQUIRE(((bits >> 23) & 0xff) != 0xff, RDET_E_FORMAT, "det conversion requires a finite f32");
  bool neg = bits >> 31;
  int e8 = (bits >> 23) & 0xff;
  uint32_t frac_bits = bits & 0x7fffff;
  if (e8 == 0 && frac_bits == 0) return 0;
  u128 sig = e8 ? ((1u << 23) | frac_bits) : frac_bits;
  int exp2 = (e8 ? e8 - 150 : -149) + frac;
  u128 lim = neg ? maxneg : maxpos;
  u128 mag;
  if (exp2 >= 0) {
    mag = (exp2 >= 128 || sig > (lim >> exp2)) ? lim : (sig << exp2);
  } else {
    int sh = -exp2;
    if (sh >= 128) mag = 0;
    else {
      u128 q = sig >> sh, rem = sig & (((u128)1 << sh) - 1), half = (u128)1 << (sh - 1);
      mag = (rem > half || (rem == half && (q & 1))) ? q + 1 : q;
      if (mag > lim) mag = lim;
    }
  }
  if (neg) return mag >= maxneg ? -(i128)maxneg : -(i128)mag;
  return (i128)mag;
}
static int32_t host_f32_to_act(float x) {
  i128 v = f32_fixed(x, 16, (u128)INT32_MAX, (u128)1 << 31);
  return v < (i128)INT32_MIN ? INT32_MIN : (v > (i128)INT32_MAX ? INT32_MAX : (int32_t)v);
}
static int64_t host_f32_to_acc(float x) {
  i128 v = f32_fixed(x, 32, (u128)INT64_MAX, (u128)1 << 63);
  return v < (i128)INT64_MIN ? INT64_MIN : (v > (i128)INT64_MAX ? INT64_MAX : (int64_t)v);
}
static i128 rte_div128(i128 n, i128 d) {
  i128 q = n / d, r = n % d;
  if (r == 0) return q;
  i128 ar = r < 0 ? -r : r, ad = d < 0 ? -d : d;
  i128 step = ((n < 0) != (d < 0)) ? -1 : 1;
  if (2 * ar < ad) return q;
  if (2 * ar > ad) return q + step;
  return (q & 1) ? q + step : q;
}
static int64_t clamp64(i128 v) {
  return v > (i128)INT64_MAX ? INT64_MAX : (v < (i128)INT64_MIN ? INT64_MIN : (int64_t)v);
}
static int64_t host_pow_acc(int64_t b, uint32_t e) {
  int64_t r = kOneAcc;
  for (uint32_t i = 0; i < e; ++i) r = acc_mul(r, b);
  return r;
}
// ops.rs:561 nth_root_acc — bisection with ties-to-even rounding
static int64_t host_nth_root(int64_t v, uint32_t deg) {
  if (deg == 1 || v == kOneAcc) return v;
  int64_t lo = 0, hi = v > kOneAcc ? v : kOneAcc;
  while (lo < hi) {
    int64_t mid = lo + (hi - lo + 1) / 2;
    if (host_pow_acc(mid, deg) <= v) lo = mid; else hi = mid - 1;
  }
  int64_t up = lo == INT64_MAX ? lo : lo + 1;
  i128 le = (i128)v - host_pow_acc(lo, deg), ue = (i128)host_pow_acc(up, deg) - v;
  if (le < 0) le = -le;
  if (ue < 0) ue = -ue;
  if (ue < le) return up;
  if (le < ue) return lo;
  return (lo & 1) ? up : lo;
}
// inverse-frequency recurrence of rope_rotate_pairs_in_place (ops.rs:184-195):
// inv[0] = 1.0, inv[i+1] = acc_mul(inv[i], step), step = div_acc(1, base^(1/(dim/2)))
static std::vector<int64_t> rope_inv_freq(int64_t base, int freq_dim, int rotary) {
  int64_t root = host_nth_root(base, (uint32_t)(freq_dim / 2));
  REQUIRE(root != 0, RDET_E_FORMAT, "rope base root is zero");
  int64_t step = clamp64(rte_div128((i128)kOneAcc << 32, (i128)root));
  std::vector<int64_t> t(rotary / 2);
  int64_t f = kOneAcc;
  for (int i = 0; i < rotary / 2; ++i) { t[i] = f; f = acc_mul(f, step); }
  return t;
}

// ---------------------------------------------------------------------------
// config (reference GemmaTextConfigFile, io.rs:61-190 and :1896-2045)
// ---------------------------------------------------------------------------
struct LayerCfg {
  bool sliding = false;
  int head_dim = 0, kv_heads = 0, rotary = 0, window = 0;
  bool trim = false;  // cache_sliding_window is Some
  int donor = -1;     // kv_shared_layer_index
  bool k_eq_v = false;
  float rope_theta = 0;
};
struct ModelCfg {
  int H = 0, L = 0, Hq = 0, kv = 0, d = 0, dg = 0, V = 0, P = 0, ple_vocab = 0, sliding_window = 0;
  bool tied = true, has_softcap = false;
  float softcap = 0, eps = 0;
  std::vector<LayerCfg> layers;
};

static const json::Value& text_cfg(const json::Value& root) {
  const json::Value* t = root.get("text_config");
  return t ? *t : root;
}
static const json::Value* opt_field(const json::Value& t, const char* k) {
  const json::Value* v = t.get(k);
  return (v && !v->is_null()) ? v : nullptr;
}
static long req_int(const json::Value& t, const char* k) {
  const json::Value* v = opt_field(t, k);
  REQUIRE(v && v->kind == json::Value::Num, RDET_E_FORMAT, std::string("config.json: missing field ") + k);
  return (long)v->num;
}
static float num_f32(const json::Value& v) { return strtof(v.str.c_str(), nullptr); }

static ModelCfg parse_config(const std::string& text) {
  json::Value root;
  try {
    root = json::parse(text);
  } catch (const std::exception& e) {
    throw Fail{RDET_E_FORMAT, e.what()};
  }
  const json::Value& t = text_cfg(root);
  ModelCfg c;
  const json::Value* moe = opt_field(t, "enable_moe_block");
  REQUIRE(moe && moe->kind == json::Value::Bool, RDET_E_FORMAT, "config.json: missing field enable_moe_block");
  REQUIRE(!moe->b, RDET_E_FORMAT, "only Gemma 4 dense layers are supported, not MoE checkpoints");
  const json::Value* act = opt_field(t, "hidden_activation");
  REQUIRE(act && act->kind == json::Value::Str, RDET_E_FORMAT, "config.json: missing field hidden_activation");
  REQUIRE(act->str == "gelu_pytorch_tanh", RDET_E_FORMAT, "only gelu_pytorch_tanh is supported, got " + act->str);
  c.H = (int)req_int(t, "hidden_size");
  c.L = (int)req_int(t, "num_hidden_layers");
  c.Hq = (int)req_int(t, "num_attention_heads");
  c.kv = (int)req_int(t, "num_key_value_heads");
  c.d = (int)req_int(t, "head_dim");
  c.V = (int)req_int(t, "vocab_size");
  c.sliding_window = (int)req_int(t, "sliding_window");
  const json::Value* v;
  c.dg = (v = opt_field(t, "global_head_dim")) ? (int)v->num : c.d;
  c.P = (v = opt_field(t, "hidden_size_per_layer_input")) ? (int)v->num : 0;
  c.ple_vocab = (v = opt_field(t, "vocab_size_per_layer_input")) ? (int)v->num : c.V;
  int gkv = (v = opt_field(t, "num_global_key_value_heads")) ? (int)v->num : c.kv;
  bool keqv = (v = opt_field(t, "attention_k_eq_v")) ? v->b : false;
  c.tied = (v = opt_field(t, "tie_word_embeddings")) ? v->b : true;
  int nshared = (v = opt_field(t, "num_kv_shared_layers")) ? (int)v->num : 0;
  bool bidir = (v = opt_field(t, "use_bidirectional_attention")) && v->kind == json::Value::Str && v->str == "all";
  if ((v = opt_field(t, "final_logit_softcapping"))) { c.has_softcap = true; c.softcap = num_f32(*v); }
  const json::Value* epsv = opt_field(t, "rms_norm_eps");
  REQUIRE(epsv, RDET_E_FORMAT, "config.json: missing field rms_norm_eps");
  c.eps = num_f32(*epsv);
  // rope parameters (io.rs:123-150)
  float partial = 0.25f, local_theta = 10000.0f, full_theta = 1000000.0f;
  const json::Value* rp = opt_field(t, "rope_parameters");
  if (rp) {
    const json::Value* fa = opt_field(*rp, "full_attention");
    const json::Value* sa = opt_field(*rp, "sliding_attention");
    const json::Value* g = opt_field(*rp, "rope_theta");
    if (fa && (v = opt_field(*fa, "partial_rotary_factor"))) partial = num_f32(*v);
    if (sa && (v = opt_field(*sa, "rope_theta"))) local_theta = num_f32(*v);
    if (fa && (v = opt_field(*fa, "rope_theta"))) full_theta = num_f32(*v);
    else if (g) full_theta = num_f32(*g);
  }
  const json::Value* lt = opt_field(t, "layer_types");
  REQUIRE(lt && lt->kind == json::Value::Arr, RDET_E_FORMAT, "config.json: missing field layer_types");
  REQUIRE((int)lt->arr.size() == c.L, RDET_E_FORMAT, "Gemma config layer count mismatch: num_hidden_layers vs layer_types");
  std::vector<bool> sl(c.L);
  for (int l = 0; l < c.L; ++l) sl[l] = lt->arr[l].str == "sliding_attention";
  // KV sharing (io.rs:165-190): the last num_kv_shared_layers layers reuse the
  // cache of the last earlier layer of the same attention type.
  int first_shared = nshared > c.L ? 0 : c.L - nshared;
  std::vector<int> donor(c.L, -1);
  std::vector<bool> is_donor(c.L, false);
  if (nshared > 0)
    for (int l = first_shared; l < c.L; ++l) {
      int dnr = -1;
      for (int j = first_shared - 1; j >= 0; --j)
        if (sl[j] == sl[l]) { dnr = j; break; }
      REQUIRE(dnr >= 0, RDET_E_FORMAT, "Gemma layer " + std::to_string(l) + " is configured to share KV without a prior donor layer");
      donor[l] = dnr;
      is_donor[dnr] = true;
    }
  int window = bidir ? c.sliding_window / 2 + 1 : c.sliding_window;
  for (int l = 0; l < c.L; ++l) {
    LayerCfg lc;
    lc.sliding = sl[l];
    lc.head_dim = lc.sliding ? c.d : c.dg;
    lc.kv_heads = lc.sliding ? c.kv : (keqv ? gkv : c.kv);
    lc.rotary = lc.sliding ? lc.head_dim : (int)((float)lc.head_dim * partial);
    lc.window = lc.sliding ? window : 0;
    lc.trim = lc.sliding && !is_donor[l];
    lc.donor = donor[l];
    lc.k_eq_v = !lc.sliding && keqv;
    lc.rope_theta = lc.sliding ? local_theta : full_theta;
    REQUIRE(lc.kv_heads > 0 && c.Hq / lc.kv_heads > 0, RDET_E_FORMAT, "invalid Gemma head configuration");
    REQUIRE(c.Hq / lc.kv_heads <= 8, RDET_E_FORMAT, "more than 8 query heads per KV head is not supported");
    REQUIRE(lc.rotary % 2 == 0 && lc.rotary <= lc.head_dim, RDET_E_FORMAT, "rope_rotate_pairs requires an even rotary_dim within head_dim");
    if (lc.rotary > 0) REQUIRE(lc.head_dim >= 2 && lc.head_dim % 2 == 0, RDET_E_FORMAT, "rope requires an even freq_base_dim");
    c.layers.push_back(lc);
  }
  return c;
}

// ---------------------------------------------------------------------------
// tensor sources: a detwgt v2 artifact (fail-closed) or the seeded generator
// ---------------------------------------------------------------------------
struct TensorInfo {
  std::vector<uint64_t> shape;
  int width = 32;
  const uint8_t* payload = nullptr;  // host pointer into the mapped artifact
  uint64_t bytes = 0;
};

struct MappedFile {
  void* base = nullptr;
  size_t size = 0;
  ~MappedFile() { if (base && base != MAP_FAILED) munmap(base, size); }
};

// detwgt v2 reader (io.rs:230-395): every check the reference makes, in the
// same order, failing closed.
static std::map<std::string, TensorInfo> parse_detwgt(const uint8_t* b, size_t n) {
  size_t cur = 0;
  auto take = [&](size_t len) -> const uint8_t* {
    REQUIRE(len <= n - cur, RDET_E_FORMAT, "artifact ended unexpectedly");
    const uint8_t* p = b + cur;
    cur += len;
    return p;
  };
  auto u32 = [&]() { uint32_t v; memcpy(&v, take(4), 4); return v; };
  auto u64 = [&]() { uint64_t v; memcpy(&v, take(8), 8); return v; };
  REQUIRE(memcmp(take(8), "DNWGTV0\0", 8) == 0, RDET_E_FORMAT, "unsupported deterministic artifact magic");
  uint32_t ver = u32();
  REQUIRE(ver == 2, RDET_E_FORMAT, "unsupported deterministic artifact format version " + std::to_string(ver) + "; expected 2");
  uint32_t spec = u32();
  REQUIRE(spec == 1, RDET_E_FORMAT, "unsupported deterministic artifact det_num spec version " + std::to_string(spec));
  uint64_t count = u64();
  std::map<std::string, TensorInfo> out;
  for (uint64_t t = 0; t < count; ++t) {
    uint32_t nl = u32();
    std::string name((const char*)take(nl), nl);
    uint32_t rank = u32();
    TensorInfo ti;
    u128 prod = 1;
    for (uint32_t i = 0; i < rank; ++i) {
      uint64_t dim = u64();
      ti.shape.push_back(dim);
      prod *= dim;
      REQUIRE(prod <= (u128)UINT64_MAX, RDET_E_FORMAT, "tensor shape overflowed");
    }
    uint64_t ec = u64();
    REQUIRE((u128)ec == prod, RDET_E_FORMAT, "tensor `" + name + "` element count mismatch");
    uint32_t w = u32();
    REQUIRE(w == 16 || w == 32, RDET_E_FORMAT, "tensor `" + name + "` has an invalid element width");
    ti.width = (int)w;
    uint64_t pl = u64();
    REQUIRE((u128)pl == (u128)ec * (w / 8), RDET_E_FORMAT, "tensor `" + name + "` payload length mismatch");
    uint64_t mass = u64();
    REQUIRE(!(rank >= 2 && mass >= ((uint64_t)1 << 31)), RDET_E_FORMAT,
            "tensor `" + name + "` max row mass violates the conversion-time overflow bound");
    size_t pad = (64 - cur % 64) % 64;
    const uint8_t* pp = take(pad);
    for (size_t i = 0; i < pad; ++i) REQUIRE(pp[i] == 0, RDET_E_FORMAT, "tensor `" + name + "` has non-zero payload alignment padding");
    ti.payload = take((size_t)pl);
    ti.bytes = pl;
    REQUIRE(out.find(name) == out.end(), RDET_E_FORMAT, "deterministic artifact contains duplicate tensor `" + name + "`");
    out.emplace(name, ti);
  }
  REQUIRE(cur == n, RDET_E_FORMAT, "deterministic artifact has trailing bytes after tensor payloads");
  return out;
}

static uint64_t fnv1a64(const std::string& s) {
  uint64_t h = 0xCBF29CE484222325ull;
  for (unsigned char ch : s) { h ^= ch; h *= 0x100000001B3ull; }
  return h;
}

// Synthetic tensor table: the same names and shapes as detwgt.layer_shapes().
static std::map<std::string, TensorInfo> synthetic_table(const ModelCfg& c, const json::Value& t, int width, int F) {
  std::map<std::string, TensorInfo> m;
  auto add = [&](const std::string& n, std::vector<uint64_t> shape) {
    TensorInfo ti;
    ti.shape = shape;
    ti.width = shape.size() == 1 ? 32 : width;
    uint64_t cnt = 1;
    for (auto d : shape) cnt *= d;
    ti.bytes = cnt * (ti.width / 8);
    m[n] = ti;
  };
  add("model.language_model.embed_tokens.weight", {(uint64_t)c.V, (uint64_t)c.H});
  const json::Value* lsv = opt_field(t, "_synthetic_layer_scalar");
  bool with_scalar = lsv ? lsv->b : true;
  for (int l = 0; l < c.L; ++l) {
    const LayerCfg& lc = c.layers[l];
    std::string p = "model.language_model.layers." + std::to_string(l);
    uint64_t hd = lc.head_dim, nkv = lc.kv_heads;
    add(p + ".self_attn.q_proj.weight", {(uint64_t)c.Hq * hd, (uint64_t)c.H});
    add(p + ".self_attn.k_proj.weight", {nkv * hd, (uint64_t)c.H});
    if (!lc.k_eq_v) add(p + ".self_attn.v_proj.weight", {nkv * hd, (uint64_t)c.H});
    add(p + ".self_attn.o_proj.weight", {(uint64_t)c.H, (uint64_t)c.Hq * hd});
    add(p + ".self_attn.q_norm.weight", {hd});
    add(p + ".self_attn.k_norm.weight", {hd});
    for (const char* nn : {"input_layernorm", "post_attention_layernorm", "pre_feedforward_layernorm", "post_feedforward_layernorm"})
      add(p + "." + nn + ".weight", {(uint64_t)c.H});
    add(p + ".mlp.gate_proj.weight", {(uint64_t)F, (uint64_t)c.H});
    add(p + ".mlp.up_proj.weight", {(uint64_t)F, (uint64_t)c.H});
    add(p + ".mlp.down_proj.weight", {(uint64_t)c.H, (uint64_t)F});
    if (c.P > 0) {
      add(p + ".per_layer_input_gate.weight", {(uint64_t)c.P, (uint64_t)c.H});
      add(p + ".per_layer_projection.weight", {(uint64_t)c.H, (uint64_t)c.P});
      add(p + ".post_per_layer_input_norm.weight", {(uint64_t)c.H});
    }
    if (with_scalar) add(p + ".layer_scalar", {1});
  }
  if (c.P > 0) {
    add("model.language_model.embed_tokens_per_layer.weight", {(uint64_t)c.ple_vocab, (uint64_t)c.L * c.P});
    add("model.language_model.per_layer_model_projection.weight", {(uint64_t)c.L * c.P, (uint64_t)c.H});
    add("model.language_model.per_layer_projection_norm.weight", {(uint64_t)c.P});
  }
  add("model.language_model.norm.weight", {(uint64_t)c.H});
  const json::Value* tie = opt_field(t, "tie_word_embeddings");
  if (tie && !tie->b) add("model.language_model.lm_head.weight", {(uint64_t)c.V, (uint64_t)c.H});
  return m;
}

// ---------------------------------------------------------------------------
// device model
// ---------------------------------------------------------------------------
struct LayerDev {
  LayerCfg cfg;
  int F = 0;
  DevMat q, k, v, o, gate, up, down, ple_gate, ple_proj;
  const int32_t *q_norm = nullptr, *k_norm = nullptr, *in_ln = nullptr, *post_attn_ln = nullptr,
                *pre_ff_ln = nullptr, *post_ff_ln = nullptr, *ple_norm = nullptr;
  bool has_scalar = false;
  int32_t scalar = 0;
  const int64_t* inv_freq = nullptr;
  // tensor-core prefill operands (byte planes), built when eligible
  TcWeight tq, tk, tv, to, tgu, tdown, tpg, tpp, tqkv;
};

struct PrefillWs {
  int S = 0;
  int32_t *x0 = nullptr, *xa = nullptr, *xb = nullptr, *nrm = nullptr, *q = nullptr, *kraw = nullptr,
          *vraw = nullptr, *qo = nullptr, *comb = nullptr, *attn = nullptr, *hbuf = nullptr, *ple_proj = nullptr,
          *ple_all = nullptr, *g = nullptr, *pr = nullptr, *scores = nullptr;
  int64_t* exps = nullptr;
  int64_t scratch_elems = 0;
  uint32_t* ids = nullptr;
};
struct DecodeWs {
  int32_t *x0 = nullptr, *t1 = nullptr, *t2 = nullptr, *q = nullptr, *kraw = nullptr, *vraw = nullptr,
          *qo = nullptr, *comb = nullptr, *attn = nullptr, *hbuf = nullptr, *ple_proj = nullptr, *ple_all = nullptr,
          *g = nullptr, *pr = nullptr, *argpart = nullptr;
};

// ---------------------------------------------------------------------------
// NCCL, loaded when tensor-parallel decode is first set up (the library has no
// link-time dependency on it; a process that already loaded libnccl.so.2, as
// torch does, shares that copy)
// ---------------------------------------------------------------------------
struct NcclApi {
  bool ok = false;
  decltype(&ncclGetUniqueId) getUniqueId = nullptr;
  decltype(&ncclCommInitRank) commInitRank = nullptr;
  decltype(&ncclAllReduce) allReduce = nullptr;
  decltype(&ncclAllGather) allGather = nullptr;
  decltype(&ncclCommDestroy) commDestroy = nullptr;
  decltype(&ncclGetErrorString) errorString = nullptr;
};
static NcclApi& nccl_api() {
  static NcclApi n;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    n.getUniqueId = reinterpret_cast<decltype(&ncclGetUniqueId)>(dlsym(h, "ncclGetUniqueId"));
    n.commInitRank = reinterpret_cast<decltype(&ncclCommInitRank)>(dlsym(h, "ncclCommInitRank"));
    n.allReduce = reinterpret_cast<decltype(&ncclAllReduce)>(dlsym(h, "ncclAllReduce"));
    n.allGather = reinterpret_cast<decltype(&ncclAllGather)>(dlsym(h, "ncclAllGather"));
    n.commDestroy = reinterpret_cast<decltype(&ncclCommDestroy)>(dlsym(h, "ncclCommDestroy"));
    n.errorString = reinterpret_cast<decltype(&ncclGetErrorString)>(dlsym(h, "ncclGetErrorString"));
    n.ok = n.getUniqueId && n.commInitRank && n.allReduce && n.allGather && n.commDestroy && n.errorString;
  });
  return n;
}
#define NCK(x)                                                                                    \
  do {                                                                                            \
    ncclResult_t r_ = (x);                                                                        \
    if (r_ != ncclSuccess) throw Fail{RDET_E_CUDA, std::string(#x) + ": " + nccl_api().errorString(r_)}; \
  } while (0)

// Tensor-parallel shard of the batched decode (every rank holds the whole
// model; these are the byte planes of this rank's slices)
struct TpLayer {
  TcWeight q, o, gu, down, pg, pp;
};
struct TpState {
  int rank = 0, world = 1;
  ncclComm_t comm = nullptr;
  int Hql = 0, head0 = 0, Fl = 0, Pl = 0, Vl = 0;
  std::vector<TpLayer> layers;
  TcWeight lm;
  int rows = 0;                // rows of the buffers below
  int64_t* part = nullptr;     // [rows, H] partial sums before requantize
  int32_t* lgl = nullptr;      // [rows, Vl] this rank's logits
  int32_t* lga = nullptr;      // [world, rows, Vl] gathered logits
  // NVLink reduction (rdet_tp_ipc_export / _connect): recv [world][2][p2p_rows][H]
  // holds every rank's column-slice sums of a reduction (two alternating
  // slots); each rank's split-K finish stores its sums into its own slot of
  // every rank's recv (peer stores over NVLink), then publishes the
  // reduction's number in the peers' flags (one word per source rank); the
  // next row kernel adds the world slots from local memory.  recv and flags
  // are mapped into the other ranks through CUDA IPC.
  bool p2p = false;
  int p2p_rows = 0;
  int64_t* recv = nullptr;
  uint32_t* flags = nullptr;
  int64_t* peer_recv[8] = {};
  TpPeerFlags peer_flags;
  std::vector<void*> ipc_opened;
  uint32_t seq = 0;            // reductions issued so far
  const int64_t* last = nullptr;  // the buffer holding the last reduction's local sums
  // Vocab-sharded selection (rdet_tp_shard_logits): a batched decode ends
  // with each row's first max over this rank's vocab rows as (value, global
  // index) pairs, all-gathered [world][rows][chunks][2] and reduced to the
  // tokens; the full logit rows are never assembled.
  bool shard_logits = false;
  int sel_rows = 0, sel_chunks = 0;
  int32_t* lpairs = nullptr;   // [sel_rows][chunks][2] this rank's pairs
  int32_t* gpairs = nullptr;   // [world][sel_rows][chunks][2]
  uint32_t* tokens = nullptr;  // [sel_rows] the selected tokens of the last batch
  uint64_t epoch = 0;          // sharded batched decodes so far
};

struct Seq;

// Per-layer prefill commitments off the critical path.  Each layer's output
// is copied into a device slab on the compute stream (device to device, so
// the next layers may overwrite their buffers at once), downloaded into a
// pinned host slab on a copy stream, and hashed by a host worker while the
// GPU runs the following layers.  A slab is reused only after its hash is
// done, which also means its download has finished.
struct CommitPipe {
  int nslots = 0;
  size_t slot_elems = 0;
  int32_t* dslab = nullptr;  // [nslots, slot_elems] (Ctx::dalloc)
  int32_t* hslab = nullptr;  // pinned, same shape
  cudaStream_t copy = nullptr;
  std::vector<cudaEvent_t> staged, copied;
  std::vector<char> busy;    // slot's hash not finished
  int next = 0;
  std::mutex mu;
  std::condition_variable cv;
  std::deque<std::function<void()>> jobs;
  int pending = 0;           // submitted and not finished
  std::string error;
  bool stop = false;
  std::vector<std::thread> workers;
};

// Reusable pinned staging for the KV-cache commitment (two halves: one being
// downloaded while the other is hashed).
struct KvStage {
  int32_t* host = nullptr;
  size_t half_elems = 0;
  cudaEvent_t ev[2] = {nullptr, nullptr};
};

struct Ctx {
  int device = 0;
  cudaStream_t stream = nullptr;
  ModelCfg cfg;
  int F = 0, dmax = 0, kvmax = 0;
  int64_t eps = 0;
  int32_t softcap = 0, emb_scale = 0, ple_emb_scale = 0, ple_proj_scale = 0, ple_in_scale = 0;
  DevMat emb, lm_head, ple_table, ple_model_proj;
  const int32_t *final_norm = nullptr, *ple_proj_norm = nullptr;
  std::vector<LayerDev> layers;
  std::vector<void*> allocs;
  uint64_t weight_bytes = 0;
  uint32_t max_prefill = 4096, flags = 0;
  PrefillWs pw;
  DecodeWs dw;
  int32_t* d_err = nullptr;
  int argblocks = 0;
  // rdet_select_batch: row pointer table, chunk pairs and tokens for up to sel_rows rows
  int sel_rows = 0;
  int32_t** sel_tab = nullptr;
  int32_t* sel_part = nullptr;
  uint32_t* sel_tok = nullptr;
  Seq* prefill_owner = nullptr;  // sequence whose routine-granular prefill is in flight
  Seq* decode_owner = nullptr;
  std::vector<void*> live_seqs;  // rdet_seq handles still open on this context
  bool tc = false;               // prefill linears run on the tensor cores
  TcWeight t_ple_model, t_lm_head;
  void* tc_act = nullptr;        // activation byte planes of the current linear
  int tc_act_k = 0;              // largest K the activation planes hold
  void* tc_split = nullptr;      // split-K partial sums of the tensor-core linear
  size_t tc_split_bytes = 0;
  void* ta_ws = nullptr;         // workspace of the tensor-core prefill attention
  size_t ta_ws_bytes = 0;
  // distinct RoPE inverse-frequency tables (device pointer, rotary / 2) and,
  // for a prefill, each one's (cos, sin) factors per prompt position
  std::vector<std::pair<const int64_t*, int>> rope_list;
  int32_t* rope_cs = nullptr;    // [rope_list.size()][max_prefill][max half][2]
  int rope_half_max = 0;
  // batched decode: per-row tables (device) and the batch logits
  struct {
    int rows = 0;                  // rows the tables hold
    void* mem = nullptr;           // one allocation for every table below
    uint32_t* ids = nullptr;
    int32_t** pos = nullptr;       // [rows] each sequence's device position
    int32_t* caps = nullptr;       // [rows]
    int32_t* order = nullptr;      // [rows] attention launch order, longest context first
    int32_t** kc = nullptr;        // [L][rows] (a KV-sharing layer lists its donor's cache)
    int32_t** vc = nullptr;
    int32_t** dec_out = nullptr;   // [rows] each sequence's per-layer outputs
    int32_t** logits_dst = nullptr;
    const unsigned char** maps = nullptr;  // [rows] each sequence's cache tensor maps (Seq::d_maps)
    bool maps_ok = false;          // every row of the current batch has them
    int32_t* logits = nullptr;     // [rows, V]
  } bw;
  TpState tp;
  CommitPipe cp;
  KvStage kvs;

  void* dalloc(size_t bytes) {
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes ? bytes : 16);
    if (e != cudaSuccess) throw Fail{RDET_E_OOM, std::string("cudaMalloc failed: ") + cudaGetErrorString(e)};
    allocs.push_back(p);
    return p;
  }
  template <typename T>
  T* dalloc_n(size_t n) { return static_cast<T*>(dalloc(n * sizeof(T))); }
  ~Ctx() {
    cudaSetDevice(device);
    if (stream) cudaStreamSynchronize(stream);
    {
      std::unique_lock<std::mutex> lk(cp.mu);
      cp.cv.wait(lk, [&] { return cp.pending == 0; });
      cp.stop = true;
    }
    cp.cv.notify_all();
    for (auto& t : cp.workers) t.join();
    for (cudaEvent_t e : cp.staged) cudaEventDestroy(e);
    for (cudaEvent_t e : cp.copied) cudaEventDestroy(e);
    if (cp.copy) cudaStreamDestroy(cp.copy);
    if (cp.hslab) cudaFreeHost(cp.hslab);
    for (cudaEvent_t e : kvs.ev)
      if (e) cudaEventDestroy(e);
    if (kvs.host) cudaFreeHost(kvs.host);
    for (void* p : tp.ipc_opened) cudaIpcCloseMemHandle(p);
    if (tp.comm) nccl_api().commDestroy(tp.comm);
    for (void* p : allocs) cudaFree(p);
    if (stream) cudaStreamDestroy(stream);
  }
};

struct Seq {
  Ctx* ctx = nullptr;
  int cap = 0;
  std::vector<int32_t*> kc, vc;  // per layer [Hkv, cap, d]; nullptr for KV-sharing layers
  int32_t* d_pos = nullptr;      // device copy of `pos`
  int pos = 0;                   // tokens in the cache (position of the next token)
  bool prefilled = false;
  int32_t* logits = nullptr;     // [V]
  // the last batched decode left this sequence's logits vocab-sharded over
  // the tensor-parallel ranks: only its selected token is known, in row
  // sel_row of that decode's tokens (valid while sel_epoch is current)
  bool logits_sharded = false;
  int sel_row = -1;
  uint64_t sel_epoch = 0;
  // tensor maps of the caches for the batched tensor-core attention:
  // [layer][K, V], 128 bytes each (zero for layers without own caches or
  // with head dims it does not take); maps_ok: every eligible one encoded
  unsigned char* d_maps = nullptr;
  bool maps_ok = false;
  uint32_t* d_token = nullptr;
  uint32_t* d_hist = nullptr;    // generated tokens (graph path)
  int32_t* d_step = nullptr;
  int hist_cap = 0;
  AttnScratch asc;
  int32_t* dec_out = nullptr;    // [L, H] per-layer outputs of the last decode
  int32_t* hid = nullptr;        // [S, H] final hidden of the last prefill
  int32_t* embd = nullptr;       // [S, H] embedding of the last prefill
  int hid_rows = 0, last_S = 0;
  bool last_was_prefill = true;
  std::vector<std::string> layer_hashes;  // per-layer prefill commitments (flag)
  // routine state
  int prefill_next = -1, prefill_S = 0;
  int32_t* prefill_cur = nullptr;
  int decode_next = -1;
  int32_t* decode_cur = nullptr;
  cudaGraphExec_t graph = nullptr;  // one decode_transition for the token in d_token
  int graph_kernels = 0;
  std::vector<void*> allocs;
  void* dalloc(size_t bytes) {
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes ? bytes : 16);
    if (e != cudaSuccess) throw Fail{RDET_E_OOM, std::string("cudaMalloc failed: ") + cudaGetErrorString(e)};
    allocs.push_back(p);
    return p;
  }
  int device = 0;
  ~Seq() {
    cudaSetDevice(device);
    cudaDeviceSynchronize();
    if (graph) cudaGraphExecDestroy(graph);
    for (void* p : allocs) cudaFree(p);
  }
};

// ---------------------------------------------------------------------------
// loading
// ---------------------------------------------------------------------------
struct Loader {
  Ctx& c;
  std::map<std::string, TensorInfo>& tab;
  bool synthetic;
  uint64_t seed;
  bool dry;  // validate names and shapes only (no device work)
  const TensorInfo* find(const std::string& n) {
    auto it = tab.find(n);
    return it == tab.end() ? nullptr : &it->second;
  }
  const TensorInfo& need(const std::string& n, size_t rank) {
    const TensorInfo* t = find(n);
    REQUIRE(t, RDET_E_FORMAT, "failed to load tensor `" + n + "` from deterministic artifact");
    REQUIRE(t->shape.size() == rank, RDET_E_FORMAT,
            "tensor `" + n + "` has rank " + std::to_string(t->shape.size()) + ", expected " + std::to_string(rank));
    return *t;
  }
  void* upload_raw(const std::string& n, const TensorInfo& t) {
    if (dry) return nullptr;
    void* p = c.dalloc(t.bytes);
    c.weight_bytes += t.bytes;
    if (synthetic) {
      uint64_t cnt = 1;
      for (auto d : t.shape) cnt *= d;
      launch_synth(p, t.width, (int)t.shape.size(), (int64_t)cnt, (int64_t)t.shape.back(), fnv1a64(n) ^ seed, c.stream);
      CK(cudaGetLastError());
    } else {
      CK(cudaMemcpyAsync(p, t.payload, t.bytes, cudaMemcpyHostToDevice, c.stream));
      CK(cudaStreamSynchronize(c.stream));
    }
    return p;
  }
  DevMat mat(const std::string& n, int rows = -1, int cols = -1) {
    const TensorInfo& t = need(n, 2);
    if (rows >= 0) REQUIRE((int)t.shape[0] == rows, RDET_E_FORMAT, "tensor `" + n + "` has unexpected row count");
    if (cols >= 0) REQUIRE((int)t.shape[1] == cols, RDET_E_FORMAT, "tensor `" + n + "` has unexpected column count");
    DevMat m;
    m.p = upload_raw(n, t);
    m.width = t.width;
    m.rows = (int)t.shape[0];
    m.cols = (int)t.shape[1];
    return m;
  }
  // rank-1 gains widened to i32 on the device
  const int32_t* vec(const std::string& n, int len) {
    const TensorInfo& t = need(n, 1);
    REQUIRE((int)t.shape[0] == len, RDET_E_FORMAT, "rms norm width mismatch for `" + n + "`");
    if (dry) return nullptr;
    if (t.width == 32 || synthetic) return static_cast<const int32_t*>(upload_raw(n, t));
    std::vector<int32_t> w(len);
    const int16_t* src = reinterpret_cast<const int16_t*>(t.payload);
    for (int i = 0; i < len; ++i) { int16_t v; memcpy(&v, src + i, 2); w[i] = v; }
    int32_t* p = c.dalloc_n<int32_t>(len);
    c.weight_bytes += (uint64_t)len * 4;
    CK(cudaMemcpy(p, w.data(), (size_t)len * 4, cudaMemcpyHostToDevice));
    return p;
  }
  bool scalar(const std::string& n, int32_t* out) {
    const TensorInfo* t = find(n);
    if (!t) return false;
    REQUIRE(t->shape.size() == 1 && t->shape[0] == 1, RDET_E_FORMAT, "tensor `" + n + "` expected shape [1] for a scalar");
    if (dry) {
      *out = 0;
    } else if (synthetic) {
      void* p = upload_raw(n, *t);  // generated on the device, read back once
      c.weight_bytes -= t->bytes;   // held on the host like an artifact scalar
      CK(cudaMemcpy(out, p, 4, cudaMemcpyDeviceToHost));
    } else if (t->width == 16) {
      int16_t v;
      memcpy(&v, t->payload, 2);
      *out = v;
    } else {
      memcpy(out, t->payload, 4);
    }
    return true;
  }
};

static void build_model(Ctx& c, std::map<std::string, TensorInfo>& tab, bool synthetic, uint64_t seed,
                        bool dry = false) {
  ModelCfg& m = c.cfg;
  Loader ld{c, tab, synthetic, seed, dry};
  const char* emb_names[] = {"model.language_model.embed_tokens.weight", "language_model.embed_tokens.weight", "embed_tokens.weight"};
  std::string emb_name;
  for (const char* n : emb_names)
    if (ld.find(n)) { emb_name = n; break; }
  REQUIRE(!emb_name.empty(), RDET_E_FORMAT, "failed to find any supported embedding tensor");
  c.emb = ld.mat(emb_name);
  REQUIRE(c.emb.cols == m.H, RDET_E_FORMAT, "embedding tensor width mismatch");
  c.emb_scale = host_f32_to_act(std::sqrt((float)c.emb.cols));  // io.rs:2123
  c.eps = host_f32_to_acc(m.eps);
  c.softcap = m.has_softcap ? host_f32_to_act(m.softcap) : 0;
  if (m.has_softcap) REQUIRE(c.softcap > 0, RDET_E_FORMAT, "softcap_act requires a strictly positive softcap");
  std::map<std::pair<int64_t, int>, const int64_t*> rope_tabs;
  for (int l = 0; l < m.L; ++l) {
    const LayerCfg& lc = m.layers[l];
    LayerDev L;
    L.cfg = lc;
    std::string p = "model.language_model.layers." + std::to_string(l);
    int hd = lc.head_dim;
    L.q = ld.mat(p + ".self_attn.q_proj.weight", m.Hq * hd, m.H);
    L.k = ld.mat(p + ".self_attn.k_proj.weight", lc.kv_heads * hd, m.H);
    if (lc.k_eq_v) {
      if (ld.find(p + ".self_attn.v_proj.weight")) L.v = ld.mat(p + ".self_attn.v_proj.weight", lc.kv_heads * hd, m.H);
    } else {
      L.v = ld.mat(p + ".self_attn.v_proj.weight", lc.kv_heads * hd, m.H);
    }
    L.o = ld.mat(p + ".self_attn.o_proj.weight", m.H, m.Hq * hd);
    L.gate = ld.mat(p + ".mlp.gate_proj.weight", -1, m.H);
    L.F = L.gate.rows;
    L.up = ld.mat(p + ".mlp.up_proj.weight", L.F, m.H);
    L.down = ld.mat(p + ".mlp.down_proj.weight", m.H, L.F);
    L.q_norm = ld.vec(p + ".self_attn.q_norm.weight", hd);
    L.k_norm = ld.vec(p + ".self_attn.k_norm.weight", hd);
    L.in_ln = ld.vec(p + ".input_layernorm.weight", m.H);
    L.post_attn_ln = ld.vec(p + ".post_attention_layernorm.weight", m.H);
    L.pre_ff_ln = ld.vec(p + ".pre_feedforward_layernorm.weight", m.H);
    L.post_ff_ln = ld.vec(p + ".post_feedforward_layernorm.weight", m.H);
    if (m.P > 0) {
      L.ple_gate = ld.mat(p + ".per_layer_input_gate.weight", m.P, m.H);
      L.ple_proj = ld.mat(p + ".per_layer_projection.weight", m.H, m.P);
      L.ple_norm = ld.vec(p + ".post_per_layer_input_norm.weight", m.H);
    }
    L.has_scalar = ld.scalar(p + ".layer_scalar", &L.scalar);
    if (lc.rotary > 0 && !dry) {
      int64_t base = host_f32_to_acc(lc.rope_theta);
      REQUIRE(base > 0, RDET_E_FORMAT, "rope_rotate_pairs requires a positive base");
      auto key = std::make_pair(base, hd * 65536 + lc.rotary);
      auto it = rope_tabs.find(key);
      if (it == rope_tabs.end()) {
        std::vector<int64_t> t = rope_inv_freq(base, hd, lc.rotary);
        int64_t* dp = c.dalloc_n<int64_t>(t.size());
        CK(cudaMemcpy(dp, t.data(), t.size() * 8, cudaMemcpyHostToDevice));
        it = rope_tabs.emplace(key, dp).first;
        c.rope_list.emplace_back(dp, lc.rotary / 2);
      }
      L.inv_freq = it->second;
    }
    c.F = std::max(c.F, L.F);
    c.dmax = std::max(c.dmax, hd);
    c.kvmax = std::max(c.kvmax, lc.kv_heads);
    c.layers.push_back(L);
  }
  c.final_norm = ld.vec("model.language_model.norm.weight", m.H);
  c.lm_head = m.tied ? c.emb : ld.mat("model.language_model.lm_head.weight", -1, m.H);
  if (m.P > 0) {
    c.ple_table = ld.mat("model.language_model.embed_tokens_per_layer.weight");
    REQUIRE(c.ple_table.rows >= m.ple_vocab && c.ple_table.cols >= m.L * m.P, RDET_E_FORMAT, "PLE token embedding slice is out of bounds");
    c.ple_table.rows = m.ple_vocab;  // rows beyond vocab_size_per_layer_input are not addressable
    c.ple_model_proj = ld.mat("model.language_model.per_layer_model_projection.weight");
    REQUIRE(c.ple_model_proj.rows >= m.L * m.P && c.ple_model_proj.cols == m.H, RDET_E_FORMAT, "PLE model projection slice is out of bounds");
    c.ple_model_proj.rows = m.L * m.P;
    c.ple_proj_norm = ld.vec("model.language_model.per_layer_projection_norm.weight", m.P);
    c.ple_emb_scale = host_f32_to_act(std::sqrt((float)m.P));              // io.rs:1226-1227
    c.ple_proj_scale = host_f32_to_act(std::pow((float)m.H, -0.5f));      // io.rs:1228-1229
    c.ple_in_scale = host_f32_to_act(std::pow(2.0f, -0.5f));              // io.rs:1230-1231
  }
  if (!dry) CK(cudaStreamSynchronize(c.stream));
}

static void alloc_workspaces(Ctx& c) {
  const ModelCfg& m = c.cfg;
  size_t S = c.max_prefill;
  PrefillWs& w = c.pw;
  w.S = (int)S;
  size_t HqD = (size_t)m.Hq * c.dmax, KvD = (size_t)c.kvmax * c.dmax, LP = (size_t)m.L * std::max(m.P, 1);
  w.x0 = c.dalloc_n<int32_t>(S * m.H);
  w.xa = c.dalloc_n<int32_t>(S * m.H);
  w.xb = c.dalloc_n<int32_t>(S * m.H);
  w.nrm = c.dalloc_n<int32_t>(S * m.H);
  w.q = c.dalloc_n<int32_t>(S * HqD);
  w.kraw = c.dalloc_n<int32_t>(S * KvD);
  w.vraw = c.dalloc_n<int32_t>(S * KvD);
  w.qo = c.dalloc_n<int32_t>(S * HqD);
  w.comb = c.dalloc_n<int32_t>(S * HqD);
  w.attn = c.dalloc_n<int32_t>(S * m.H);
  w.hbuf = c.dalloc_n<int32_t>(S * c.F);
  w.ple_proj = c.dalloc_n<int32_t>(S * LP);
  w.ple_all = c.dalloc_n<int32_t>(S * LP);
  w.g = c.dalloc_n<int32_t>(S * std::max(m.P, 1));
  w.pr = c.dalloc_n<int32_t>(S * m.H);
  w.ids = c.dalloc_n<uint32_t>(S);
  for (auto& r : c.rope_list) c.rope_half_max = std::max(c.rope_half_max, r.second);
  if (!c.rope_list.empty())
    c.rope_cs = c.dalloc_n<int32_t>(c.rope_list.size() * S * (size_t)c.rope_half_max * 2);
  w.scratch_elems = (int64_t)m.Hq * S * S;
  w.scores = c.dalloc_n<int32_t>(w.scratch_elems);
  w.exps = c.dalloc_n<int64_t>(w.scratch_elems);
  DecodeWs& d = c.dw;
  d.x0 = c.dalloc_n<int32_t>(m.H);
  d.t1 = c.dalloc_n<int32_t>(m.H);
  d.t2 = c.dalloc_n<int32_t>(m.H);
  d.q = c.dalloc_n<int32_t>(HqD);
  d.kraw = c.dalloc_n<int32_t>(KvD);
  d.vraw = c.dalloc_n<int32_t>(KvD);
  d.qo = c.dalloc_n<int32_t>(HqD);
  d.comb = c.dalloc_n<int32_t>(HqD);
  d.attn = c.dalloc_n<int32_t>(m.H);
  d.hbuf = c.dalloc_n<int32_t>(c.F);
  d.ple_proj = c.dalloc_n<int32_t>(LP);
  d.ple_all = c.dalloc_n<int32_t>(LP);
  d.g = c.dalloc_n<int32_t>(std::max(m.P, 1));
  d.pr = c.dalloc_n<int32_t>(m.H);
  c.argblocks = std::min(sm_count() * 2, (m.V + 255) / 256);
  if (c.argblocks < 1) c.argblocks = 1;
  d.argpart = c.dalloc_n<int32_t>(2 * c.argblocks);
  c.d_err = c.dalloc_n<int32_t>(1);
  CK(cudaMemset(c.d_err, 0, 4));
}

constexpr size_t kTcSplitScratch = 64ull << 20;  // split-K partials for short row counts

// Byte planes of every prefill weight the tensor-core linear can take (i16,
// K a multiple of 16): one more copy of those weights in HBM.
static void prepare_tensor_cores(Ctx& c) {
  if ((c.flags & RDET_FLAG_NO_TENSOR_CORES) || !tc_supported()) return;
  const ModelCfg& m = c.cfg;
  // prefill attention on the tensor cores: one workspace sized for the
  // largest eligible layer shape at max_prefill tokens
  for (const LayerDev& L : c.layers)
    c.ta_ws_bytes = std::max(c.ta_ws_bytes, tc_attn_ws_bytes((int)c.max_prefill, m.Hq, L.cfg.kv_heads, L.cfg.head_dim));
  if (c.ta_ws_bytes) c.ta_ws = c.dalloc(c.ta_ws_bytes);
  int kmax = 0;
  auto prep = [&](TcWeight& t, const DevMat& w, const DevMat* u = nullptr) {
    if (!w.p || !tc_weight_eligible(w) || (u && (!u->p || !tc_weight_eligible(*u) || u->rows != w.rows ||
                                                 u->cols != w.cols)))
      return;
    void* mem = c.dalloc(tc_weight_bytes(w.rows, w.cols, u != nullptr));
    REQUIRE(tc_prepare_weight(t, w, u, mem, c.stream), RDET_E_CUDA, "tensor map encoding failed");
    kmax = std::max(kmax, w.cols);
  };
  for (LayerDev& L : c.layers) {
    // a layer's own q, k (and v) share one plane buffer: separate views for the
    // prefill GEMMs, the whole for one batched-decode GEMM
    bool grouped = false;
    if (L.cfg.donor < 0) {
      DevMat mats[3] = {L.q, L.k, L.v};
      const int n = L.v.p ? 3 : 2;
      bool ok = true;
      for (int i = 0; i < n; ++i) ok = ok && mats[i].p && tc_weight_eligible(mats[i]) && mats[i].cols == L.q.cols;
      if (ok) {
        TcWeight views[3];
        void* mem = c.dalloc(tc_weight_group_bytes(mats, n));
        REQUIRE(tc_prepare_weight_group(views, mats, n, L.tqkv, mem, c.stream), RDET_E_CUDA,
                "tensor map encoding failed");
        L.tq = views[0];
        L.tk = views[1];
        if (n == 3) L.tv = views[2];
        kmax = std::max(kmax, L.q.cols);
        grouped = true;
      }
    }
    if (!grouped) {
      prep(L.tq, L.q);
      if (L.cfg.donor < 0) {
        prep(L.tk, L.k);
        if (L.v.p) prep(L.tv, L.v);
      }
    }
    prep(L.to, L.o);
    prep(L.tgu, L.gate, &L.up);
    prep(L.tdown, L.down);
    if (m.P > 0) {
      prep(L.tpg, L.ple_gate);
      prep(L.tpp, L.ple_proj);
    }
  }
  if (m.P > 0) prep(c.t_ple_model, c.ple_model_proj);
  prep(c.t_lm_head, c.lm_head);  // logits of batched decode
  if (kmax > 0) {
    c.tc_act = c.dalloc(tc_act_bytes((int)c.max_prefill, kmax));
    c.tc_act_k = kmax;
    c.tc_split_bytes = kTcSplitScratch;
    c.tc_split = c.dalloc(c.tc_split_bytes);
  }
  CK(cudaStreamSynchronize(c.stream));
  CK(cudaGetLastError());
  c.tc = kmax > 0;
}

// Prefill linear: tensor cores when the weight has byte planes and the
// prompt is long enough to fill them, else the CUDA-core kernel.  Both are
// bit-exact.  `act` carries the activation planes of X between calls that
// share X (pass the same TcAct with prepared = true).
constexpr int kTcMinRows = 32;
struct ActPlanes {
  TcAct a;
  bool ready = false;   // a holds the planes of the normalized rows
  bool normed = false;  // the normalized rows are already in the workspace (w.nrm)
};
// True when a prefill linear of weight planes `t` over S rows of `cols`
// columns runs on the tensor cores.
static bool prefill_tc(const Ctx& c, const TcWeight& t, int S, int cols) {
  return c.tc && t.planes && S >= kTcMinRows && cols <= c.tc_act_k;
}
static void prefill_linear(Ctx& c, const int32_t* X, int S, const DevMat& w, const TcWeight& t, int32_t* Y,
                           int32_t epi, const int32_t* vec, ActPlanes* shared = nullptr) {
  cudaStream_t s = c.stream;
  if (prefill_tc(c, t, S, w.cols)) {
    ActPlanes local;
    ActPlanes& ap = shared ? *shared : local;
    if (!ap.ready) {
      REQUIRE(tc_prepare_act(ap.a, X, S, w.cols, c.tc_act, s), RDET_E_CUDA, "tensor map encoding failed");
      ap.ready = true;
    }
    TcOut o;
    o.y = Y;
    o.epi = epi;
    o.vec = vec;
    o.scratch = c.tc_split;
    o.scratch_bytes = c.tc_split_bytes;
    launch_tc_linear(ap.a, t, o, s);
    return;
  }
  launch_linear(X, S, w, Y, epi, vec, s);
}
// MLP gate/up pair: Y = mul_sat(gelu(X Wg^T), X Wu^T)
static void prefill_geglu(Ctx& c, const int32_t* X, int S, const LayerDev& L, int32_t* Y,
                          ActPlanes* shared = nullptr) {
  cudaStream_t s = c.stream;
  if (prefill_tc(c, L.tgu, S, L.gate.cols)) {
    ActPlanes local;
    ActPlanes& ap = shared ? *shared : local;
    if (!ap.ready) {
      REQUIRE(tc_prepare_act(ap.a, X, S, L.gate.cols, c.tc_act, s), RDET_E_CUDA, "tensor map encoding failed");
      ap.ready = true;
    }
    const TcAct& a = ap.a;
    TcOut o;
    o.y = Y;
    o.scratch = c.tc_split;
    o.scratch_bytes = c.tc_split_bytes;
    launch_tc_linear(a, L.tgu, o, s);
    return;
  }
  launch_linear_geglu(X, S, L.gate, L.up, Y, s);
}

// Fused per-row norm of the batched decode (row_norm_kernel).  With `ap`,
// the kernel also writes the activation byte planes of y for the next
// tensor-core GEMM and attaches them.  Returns false (nothing launched) when
// a row pointer or gain is not 16-byte aligned or n % 4 != 0.
static bool row_norm(Ctx& c, RowNormArgs ra, int B, ActPlanes* ap) {
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (ra.n % 4 != 0 || !al(ra.a) || !al(ra.a64) || !al(ra.res) || !al(ra.g1) || !al(ra.g2) || !al(ra.t_out) ||
      !al(ra.y_out))
    return false;
  if (ra.scatter && (ra.scatter_off * 4) % 16 != 0) return false;
  const bool planes = ap && c.tc && B >= kTcMinRows && ra.n <= c.tc_act_k;
  // tile flags only where the linear reads them (past the short-row kernel)
  const bool flags = planes && B > kTcShortRows;
  if (planes) {
    ra.planes = static_cast<uint8_t*>(c.tc_act);
    ra.rowsum = reinterpret_cast<uint64_t*>(ra.planes + 4 * (size_t)B * ra.n);
  }
  if (flags) {
    ra.tile4 = tc_act_tile4(c.tc_act, B, ra.n);
    CK(cudaMemsetAsync(ra.tile4, 0, (size_t)(B + kTcFlagRows - 1) / kTcFlagRows * 4, c.stream));
  }
  launch_row_norm(ra, B, c.stream);
  if (planes) {
    REQUIRE(tc_attach_act(ap->a, B, ra.n, c.tc_act, flags), RDET_E_CUDA, "tensor map encoding failed");
    ap->ready = true;
  }
  return true;
}

static void check_err_flag(Ctx& c, const char* what) {
  int32_t e = 0;
  CK(cudaMemcpyAsync(&e, c.d_err, 4, cudaMemcpyDeviceToHost, c.stream));
  CK(cudaStreamSynchronize(c.stream));
  if (e) {
    CK(cudaMemset(c.d_err, 0, 4));
    throw Fail{RDET_E_RANGE, std::string(what) + ": token id is out of bounds for the embedding tensor"};
  }
  if (stream_error_flag(true))
    throw Fail{RDET_E_CUDA, std::string(what) + ": a weight-streaming pipeline wait timed out"};
}

// ---------------------------------------------------------------------------
// prefill (deterministic_tiles.rs:69-199; det_kernels.rs:678-821)
// ---------------------------------------------------------------------------
static void prefill_begin(Ctx& c, Seq& q, const uint32_t* ids, size_t n) {
  const ModelCfg& m = c.cfg;
  REQUIRE(n > 0, RDET_E_INVALID, "transformer embedding requires at least one token id");
  REQUIRE(n <= c.max_prefill, RDET_E_RANGE, "prompt longer than the context's max_prefill");
  REQUIRE((int)n <= q.cap, RDET_E_RANGE, "prompt longer than the sequence capacity");
  for (size_t i = 0; i < n; ++i)
    REQUIRE(ids[i] < (uint32_t)c.emb.rows, RDET_E_RANGE, "token id " + std::to_string(ids[i]) + " is out of bounds for embedding tensor");
  if (m.P > 0)
    for (size_t i = 0; i < n; ++i) REQUIRE(ids[i] < (uint32_t)m.ple_vocab, RDET_E_RANGE, "token id is out of bounds for the PLE table");
  PrefillWs& w = c.pw;
  int S = (int)n;
  cudaStream_t s = c.stream;
  CK(cudaMemcpyAsync(w.ids, ids, n * 4, cudaMemcpyHostToDevice, s));
  CK(cudaMemsetAsync(q.d_pos, 0, 4, s));
  q.pos = 0;
  q.prefilled = false;
  launch_embed(w.ids, S, c.emb, c.emb_scale, w.x0, c.d_err, s);
  // RoPE factors of positions [0, S), once per distinct frequency table
  for (size_t t = 0; t < c.rope_list.size(); ++t)
    launch_rope_table(c.rope_list[t].first, c.rope_list[t].second, S,
                      c.rope_cs + t * (size_t)c.max_prefill * c.rope_half_max * 2, s);
  if (m.P > 0) {
    prefill_linear(c, w.x0, S, c.ple_model_proj, c.t_ple_model, w.ple_proj, kEpiPlain, nullptr);
    PleArgs pa;
    pa.S = S; pa.L = m.L; pa.P = m.P; pa.ids = w.ids; pa.proj = w.ple_proj; pa.table = c.ple_table;
    pa.norm = c.ple_proj_norm; pa.eps = c.eps; pa.emb_scale = c.ple_emb_scale; pa.proj_scale = c.ple_proj_scale;
    pa.in_scale = c.ple_in_scale; pa.out = w.ple_all; pa.err = c.d_err;
    launch_ple(pa, s);
  }
  CK(cudaGetLastError());
  if (q.hid_rows < S) {
    q.hid = static_cast<int32_t*>(q.dalloc((size_t)S * m.H * 4));
    q.embd = static_cast<int32_t*>(q.dalloc((size_t)S * m.H * 4));
    q.hid_rows = S;
  }
  CK(cudaMemcpyAsync(q.embd, w.x0, (size_t)S * m.H * 4, cudaMemcpyDeviceToDevice, s));
  CK(cudaMemcpyAsync(w.xa, w.x0, (size_t)S * m.H * 4, cudaMemcpyDeviceToDevice, s));
  q.prefill_S = S;
  q.prefill_cur = w.xa;
  q.prefill_next = 0;
  q.layer_hashes.assign(m.L, std::string());
  c.prefill_owner = &q;
  check_err_flag(c, "prefill");
}

static std::string act_hash_rows(const int32_t* host, size_t rows, size_t cols) {
  Sha256 h;
  h.put("raster-det-num-act-v1", 21);
  h.put_u64(rows);
  for (size_t r = 0; r < rows; ++r) { h.put_u64(cols); h.put(host + r * cols, cols * 4); }
  return h.hex();
}

static void commit_pipe_start(Ctx& c) {
  CommitPipe& p = c.cp;
  if (p.nslots) return;
  const unsigned hw = std::thread::hardware_concurrency();
  const int workers = std::max(1, std::min(6, (int)(hw > 2 ? hw - 2 : 1)));
  const int nslots = workers + 2;
  p.slot_elems = (size_t)c.max_prefill * c.cfg.H;
  p.dslab = c.dalloc_n<int32_t>(p.slot_elems * nslots);
  void* h = nullptr;
  if (cudaHostAlloc(&h, p.slot_elems * nslots * 4, cudaHostAllocDefault) != cudaSuccess)
    throw Fail{RDET_E_OOM, "pinned staging for the layer commitments could not be allocated"};
  p.hslab = static_cast<int32_t*>(h);
  CK(cudaStreamCreateWithFlags(&p.copy, cudaStreamNonBlocking));
  p.staged.assign(nslots, nullptr);
  p.copied.assign(nslots, nullptr);
  for (int k = 0; k < nslots; ++k) {
    CK(cudaEventCreateWithFlags(&p.staged[k], cudaEventDisableTiming));
    CK(cudaEventCreateWithFlags(&p.copied[k], cudaEventDisableTiming));
  }
  p.busy.assign(nslots, 0);
  p.nslots = nslots;
  const int dev = c.device;
  for (int i = 0; i < workers; ++i)
    p.workers.emplace_back([&p, dev] {
      cudaSetDevice(dev);
      for (;;) {
        std::function<void()> job;
        {
          std::unique_lock<std::mutex> lk(p.mu);
          p.cv.wait(lk, [&] { return p.stop || !p.jobs.empty(); });
          if (p.jobs.empty()) return;
          job = std::move(p.jobs.front());
          p.jobs.pop_front();
        }
        job();
      }
    });
}

// Stages layer output `src` ([rows, H]) and queues its hash into *dst.
static void commit_layer_async(Ctx& c, const int32_t* src, int rows, std::string* dst) {
  commit_pipe_start(c);
  CommitPipe& p = c.cp;
  const int k = p.next;
  p.next = (k + 1) % p.nslots;
  {
    std::unique_lock<std::mutex> lk(p.mu);
    p.cv.wait(lk, [&] { return !p.busy[k]; });
    p.busy[k] = 1;
    ++p.pending;
  }
  const size_t cols = c.cfg.H, n = (size_t)rows * cols;
  int32_t* ds = p.dslab + k * p.slot_elems;
  int32_t* hs = p.hslab + k * p.slot_elems;
  try {
    CK(cudaMemcpyAsync(ds, src, n * 4, cudaMemcpyDeviceToDevice, c.stream));
    CK(cudaEventRecord(p.staged[k], c.stream));
    CK(cudaStreamWaitEvent(p.copy, p.staged[k], 0));
    CK(cudaMemcpyAsync(hs, ds, n * 4, cudaMemcpyDeviceToHost, p.copy));
    CK(cudaEventRecord(p.copied[k], p.copy));
  } catch (...) {
    {
      std::lock_guard<std::mutex> lk(p.mu);
      p.busy[k] = 0;
      --p.pending;
    }
    p.cv.notify_all();
    throw;
  }
  cudaEvent_t ev = p.copied[k];
  {
    std::lock_guard<std::mutex> lk(p.mu);
    p.jobs.emplace_back([&p, k, ev, hs, rows, cols, dst] {
      cudaError_t e = cudaEventSynchronize(ev);
      std::string hx;
      if (e == cudaSuccess) hx = act_hash_rows(hs, rows, cols);
      {
        std::lock_guard<std::mutex> lk2(p.mu);
        if (e == cudaSuccess) *dst = hx;
        else if (p.error.empty()) p.error = std::string("layer commitment download: ") + cudaGetErrorString(e);
        p.busy[k] = 0;
        --p.pending;
      }
      p.cv.notify_all();
    });
  }
  p.cv.notify_all();
}

// Waits for every queued layer hash; reports the first failure when `report`.
static void commit_join(Ctx& c, bool report) {
  CommitPipe& p = c.cp;
  std::string err;
  {
    std::unique_lock<std::mutex> lk(p.mu);
    p.cv.wait(lk, [&] { return p.pending == 0; });
    err.swap(p.error);
  }
  if (report && !err.empty()) throw Fail{RDET_E_CUDA, err};
}

static void prefill_layer(Ctx& c, Seq& q, int l) {
  const ModelCfg& m = c.cfg;
  const LayerDev& L = c.layers[l];
  const LayerCfg& lc = L.cfg;
  PrefillWs& w = c.pw;
  cudaStream_t s = c.stream;
  const int S = q.prefill_S, H = m.H, d = lc.head_dim;
  int32_t* cur = q.prefill_cur;
  int32_t* other = cur == w.xa ? w.xb : w.xa;
  // The row norms run as row_norm_kernel, which also writes the byte planes
  // of the next linear's input (the plain norm kernels when a row pointer is
  // not 16-byte aligned).  A normed row goes to w.nrm only when a linear
  // reading it runs on the CUDA cores.
  ActPlanes nrm_planes;  // q, k and v read the same normed input
  {
    const bool own_kv = lc.donor < 0;
    const bool all_tc = prefill_tc(c, L.tq, S, H) && (!own_kv || prefill_tc(c, L.tk, S, H)) &&
                        (!own_kv || !L.v.p || prefill_tc(c, L.tv, S, H));
    RowNormArgs ra;
    ra.a = cur; ra.g1 = L.in_ln; ra.n = H; ra.eps = c.eps; ra.y_out = all_tc ? nullptr : w.nrm;
    if (!row_norm(c, ra, S, &nrm_planes)) launch_rmsnorm_rows(cur, S, H, L.in_ln, c.eps, w.nrm, s);
  }
  prefill_linear(c, w.nrm, S, L.q, L.tq, w.q, kEpiPlain, nullptr, &nrm_planes);
  QkvPostArgs qa;
  qa.S = S; qa.pos = q.d_pos; qa.Hq = m.Hq; qa.Hkv = lc.kv_heads; qa.d = d; qa.rotary = lc.rotary;
  qa.inv_freq = L.inv_freq; qa.q_in = w.q; qa.q_norm = L.q_norm; qa.k_norm = L.k_norm; qa.eps = c.eps;
  qa.q_out = w.qo; qa.cap = q.cap;
  for (size_t t = 0; t < c.rope_list.size(); ++t)
    if (c.rope_list[t].first == L.inv_freq)
      qa.rope_cs = c.rope_cs + t * (size_t)c.max_prefill * c.rope_half_max * 2;
  const int32_t *kcache, *vcache;
  if (lc.donor < 0) {
    prefill_linear(c, w.nrm, S, L.k, L.tk, w.kraw, kEpiPlain, nullptr, &nrm_planes);
    const int32_t* vsrc = w.kraw;  // k_eq_v: V is the raw K projection (det_kernels.rs:517-518)
    if (L.v.p) { prefill_linear(c, w.nrm, S, L.v, L.tv, w.vraw, kEpiPlain, nullptr, &nrm_planes); vsrc = w.vraw; }
    qa.k_in = w.kraw; qa.v_in = vsrc; qa.k_cache = q.kc[l]; qa.v_cache = q.vc[l];
    kcache = q.kc[l];
    vcache = q.vc[l];
  } else {
    // KV-sharing layers attend over the donor's cache; their own K/V
    // projections cannot affect any output and are not computed.
    kcache = q.kc[lc.donor];
    vcache = q.vc[lc.donor];
  }
  launch_qkv_post(qa, s);
  AttnPrefillArgs aa;
  aa.S = S; aa.Hq = m.Hq; aa.Hkv = lc.kv_heads; aa.d = d; aa.window = lc.window; aa.q = w.qo;
  aa.k_cache = kcache; aa.v_cache = vcache; aa.cap = q.cap; aa.out = w.comb; aa.scores = w.scores; aa.exps = w.exps;
  aa.scratch_elems = w.scratch_elems;
  if (!(c.ta_ws && launch_attn_prefill_tc(aa, c.ta_ws, c.ta_ws_bytes, s))) launch_attn_prefill(aa, s);
  prefill_linear(c, w.comb, S, L.o, L.to, w.attn, kEpiPlain, nullptr);
  bool ple = m.P > 0;
  // t1 = xs + norm(attn) -> other, and the MLP input norm(t1) with its planes
  ActPlanes ff_planes;
  {
    RowNormArgs ra;
    ra.a = w.attn; ra.res = cur; ra.g1 = L.post_attn_ln; ra.g2 = L.pre_ff_ln; ra.n = H; ra.eps = c.eps;
    ra.t_out = other; ra.y_out = prefill_tc(c, L.tgu, S, H) ? nullptr : w.nrm;
    if (!row_norm(c, ra, S, &ff_planes)) {
      launch_norm_residual_rows(w.attn, cur, S, H, L.post_attn_ln, c.eps, false, 0, other, s);
      launch_rmsnorm_rows(other, S, H, L.pre_ff_ln, c.eps, w.nrm, s);
    }
  }
  prefill_geglu(c, w.nrm, S, L, w.hbuf, &ff_planes);
  prefill_linear(c, w.hbuf, S, L.down, L.tdown, w.attn, kEpiPlain, nullptr);
  // t2 = t1 + norm(ff) -> cur, with the planes of t2 for the per-layer-input gate
  ActPlanes t2_planes;
  {
    RowNormArgs ra;
    ra.a = w.attn; ra.res = other; ra.g1 = L.post_ff_ln; ra.n = H; ra.eps = c.eps;
    ra.has_scalar = !ple && L.has_scalar; ra.scalar = L.scalar; ra.t_out = cur;
    if (!row_norm(c, ra, S, ple ? &t2_planes : nullptr))
      launch_norm_residual_rows(w.attn, other, S, H, L.post_ff_ln, c.eps, !ple && L.has_scalar, L.scalar, cur, s);
  }
  int32_t* result = cur;
  if (ple) {
    prefill_linear(c, cur, S, L.ple_gate, L.tpg, w.g, kEpiGeluMul, w.ple_all + (size_t)l * S * m.P, &t2_planes);
    prefill_linear(c, w.g, S, L.ple_proj, L.tpp, w.pr, kEpiPlain, nullptr);
    launch_norm_residual_rows(w.pr, cur, S, H, L.ple_norm, c.eps, L.has_scalar, L.scalar, other, s);
    result = other;
  }
  CK(cudaGetLastError());
  q.prefill_cur = result;
  if (c.flags & RDET_FLAG_LAYER_COMMITMENTS) commit_layer_async(c, result, S, &q.layer_hashes[l]);
}

static void gemv_logits(Ctx& c, const int32_t* hidden_row, int32_t* logits, cudaStream_t s) {
  GemvArgs g;
  g.K = c.cfg.H;
  g.nseg = 1;
  g.seg[0].w = c.lm_head;
  g.seg[0].y = logits;
  g.seg[0].epi = c.cfg.has_softcap ? kEpiSoftcap : kEpiPlain;
  g.softcap = c.softcap;
  g.pro = kProNorm;
  g.a = hidden_row;
  g.g1 = c.final_norm;
  g.eps = c.eps;
  launch_gemv(g, s);
}

static void prefill_finalize(Ctx& c, Seq& q) {
  const ModelCfg& m = c.cfg;
  REQUIRE(q.prefill_next == m.L, RDET_E_STATE, "prefill.finalize requires every layer to have run");
  cudaStream_t s = c.stream;
  int S = q.prefill_S;
  CK(cudaMemcpyAsync(q.hid, q.prefill_cur, (size_t)S * m.H * 4, cudaMemcpyDeviceToDevice, s));
  gemv_logits(c, q.prefill_cur + (size_t)(S - 1) * m.H, q.logits, s);
  int32_t pos = S;
  CK(cudaMemcpyAsync(q.d_pos, &pos, 4, cudaMemcpyHostToDevice, s));
  CK(cudaStreamSynchronize(s));
  CK(cudaGetLastError());
  q.pos = S;
  q.last_S = S;
  q.prefilled = true;
  q.logits_sharded = false;
  q.last_was_prefill = true;
  q.prefill_next = -1;
  c.prefill_owner = nullptr;
}

// ---------------------------------------------------------------------------
// decode (decode_layer_range/native/tiles.rs:133-197; det_kernels.rs:866-1208)
// ---------------------------------------------------------------------------
static void decode_embed(Ctx& c, Seq& q, const uint32_t* d_token) {
  const ModelCfg& m = c.cfg;
  DecodeWs& w = c.dw;
  cudaStream_t s = c.stream;
  launch_embed(d_token, 1, c.emb, c.emb_scale, w.x0, c.d_err, s);
  if (m.P > 0) {
    GemvArgs g;
    g.K = m.H;
    g.seg[0].w = c.ple_model_proj;
    g.seg[0].y = w.ple_proj;
    g.a = w.x0;
    launch_gemv(g, s);
    PleArgs pa;
    pa.S = 1; pa.L = m.L; pa.P = m.P; pa.ids = d_token; pa.proj = w.ple_proj; pa.table = c.ple_table;
    pa.norm = c.ple_proj_norm; pa.eps = c.eps; pa.emb_scale = c.ple_emb_scale; pa.proj_scale = c.ple_proj_scale;
    pa.in_scale = c.ple_in_scale; pa.out = w.ple_all; pa.err = c.d_err;
    launch_ple(pa, s);
  }
}

// The tail of a decode layer (final RMSNorm + residual + layer scalar) left
// for the next kernel's prologue when the decode step is fused.
struct PendingTail {
  bool set = false;
  const int32_t* a = nullptr;    // branch output to normalize
  const int32_t* res = nullptr;  // residual input
  const int32_t* g = nullptr;    // norm gain
  bool has_scalar = false;
  int32_t scalar = 0;
  int32_t* out = nullptr;        // where the layer output row is stored
};

// Fills the prologue of a GEMV over the layer input: plain RMSNorm of `cur`,
// or (fused step) the previous layer's pending tail followed by the norm.
static void input_prologue(Ctx& c, GemvArgs& g, const int32_t* cur, const int32_t* gain, const PendingTail* pend) {
  g.eps = c.eps;
  if (pend && pend->set) {
    g.pro = kProResScaleNorm;
    g.a = pend->a;
    g.res = pend->res;
    g.g1 = pend->g;
    g.has_scalar = pend->has_scalar;
    g.scalar = pend->scalar;
    g.g2 = gain;
    g.t_out = pend->out;
  } else {
    g.pro = kProNorm;
    g.a = cur;
    g.g1 = gain;
  }
}

static const int32_t* decode_layer(Ctx& c, Seq& q, int l, const int32_t* cur, PendingTail* pend = nullptr) {
  const ModelCfg& m = c.cfg;
  const LayerDev& L = c.layers[l];
  const LayerCfg& lc = L.cfg;
  DecodeWs& w = c.dw;
  cudaStream_t s = c.stream;
  const int H = m.H, d = lc.head_dim;
  // q/k/v projections of rmsnorm(x)
  GemvArgs g;
  g.K = H;
  input_prologue(c, g, cur, L.in_ln, pend);
  g.nseg = 1;
  g.seg[0].w = L.q;
  g.seg[0].y = w.q;
  const int32_t *kcache, *vcache;
  QkvPostArgs qa;
  qa.S = 1; qa.pos = q.d_pos; qa.Hq = m.Hq; qa.Hkv = lc.kv_heads; qa.d = d; qa.rotary = lc.rotary;
  qa.inv_freq = L.inv_freq; qa.q_in = w.q; qa.q_norm = L.q_norm; qa.k_norm = L.k_norm; qa.eps = c.eps;
  qa.q_out = w.qo; qa.cap = q.cap;
  if (lc.donor < 0) {
    g.seg[1].w = L.k;
    g.seg[1].y = w.kraw;
    g.nseg = 2;
    const int32_t* vsrc = w.kraw;
    if (L.v.p) { g.seg[2].w = L.v; g.seg[2].y = w.vraw; g.nseg = 3; vsrc = w.vraw; }
    qa.k_in = w.kraw; qa.v_in = vsrc; qa.k_cache = q.kc[l]; qa.v_cache = q.vc[l];
    kcache = q.kc[l];
    vcache = q.vc[l];
  } else {
    kcache = q.kc[lc.donor];
    vcache = q.vc[lc.donor];
  }
  launch_gemv(g, s);
  AttnDecodeArgs aa;
  aa.pos = q.d_pos; aa.Hq = m.Hq; aa.Hkv = lc.kv_heads; aa.d = d; aa.window = lc.window; aa.q = w.qo;
  aa.k_cache = kcache; aa.v_cache = vcache; aa.cap = q.cap; aa.out = w.comb; aa.sc = q.asc;
  aa.rows_per_split = 64;
  // The fused step normalizes, rotates and appends inside the attention
  // kernel; the routine-granular path keeps the separate qkv_post kernel.
  const bool fuse_qkv =
      pend != nullptr && attn_decode_cluster_fits(m.Hq, lc.kv_heads, d, lc.window, q.cap, lc.rotary);
  if (fuse_qkv) {
    aa.fuse.q_in = w.q;
    aa.fuse.k_in = qa.k_in;
    aa.fuse.v_in = qa.v_in;
    aa.fuse.q_norm = L.q_norm;
    aa.fuse.k_norm = L.k_norm;
    aa.fuse.eps = c.eps;
    aa.fuse.rotary = lc.rotary;
    aa.fuse.inv_freq = L.inv_freq;
    aa.fuse.k_out = qa.k_cache;
    aa.fuse.v_out = qa.v_cache;
  } else {
    launch_qkv_post(qa, s);
  }
  launch_attn_decode_cluster(aa, s);
  GemvArgs go;
  go.K = m.Hq * d;
  go.seg[0].w = L.o;
  go.seg[0].y = w.attn;
  go.a = w.comb;

  launch_gemv(go, s);
  // t1 = x + norm(attn); MLP input = norm(t1)
  GemvArgs gg;
  gg.K = H;
  gg.pro = kProResNorm;
  gg.a = w.attn; gg.res = cur; gg.g1 = L.post_attn_ln; gg.g2 = L.pre_ff_ln; gg.eps = c.eps; gg.t_out = w.t1;
  gg.pair_geglu = true;
  gg.nseg = 2;
  gg.seg[0].w = L.gate; gg.seg[0].y = w.hbuf;
  gg.seg[1].w = L.up;
  launch_gemv(gg, s);
  GemvArgs gd;
  gd.K = L.F;
  gd.seg[0].w = L.down;
  gd.seg[0].y = w.attn;
  gd.a = w.hbuf;
  launch_gemv(gd, s);
  int32_t* out = q.dec_out + (size_t)l * H;
  if (m.P > 0) {
    // t2 = t1 + norm(ff) (stored by block 0); gate = gelu(Wg t2) * ple_in
    GemvArgs gp;
    gp.K = H;
    gp.pro = kProResScale;
    gp.a = w.attn; gp.res = w.t1; gp.g1 = L.post_ff_ln; gp.eps = c.eps; gp.t_out = w.t2;
    gp.seg[0].w = L.ple_gate; gp.seg[0].y = w.g; gp.seg[0].epi = kEpiGeluMul;
    gp.seg[0].vec = w.ple_all + (size_t)l * m.P;

    launch_gemv(gp, s);
    GemvArgs gq;
    gq.K = m.P;
    gq.seg[0].w = L.ple_proj; gq.seg[0].y = w.pr;
    gq.a = w.g;
    launch_gemv(gq, s);
  }
  const int32_t* ta = m.P > 0 ? w.pr : w.attn;
  const int32_t* tres = m.P > 0 ? w.t2 : w.t1;
  const int32_t* tg = m.P > 0 ? L.ple_norm : L.post_ff_ln;
  if (pend) {
    pend->set = true;
    pend->a = ta;
    pend->res = tres;
    pend->g = tg;
    pend->has_scalar = L.has_scalar;
    pend->scalar = L.scalar;
    pend->out = out;
  } else {
    launch_norm_residual_rows(ta, tres, 1, H, tg, c.eps, L.has_scalar, L.scalar, out, s);
  }
  return out;
}

static void decode_finalize_launch(Ctx& c, Seq& q, const int32_t* cur, const PendingTail* pend = nullptr) {
  if (pend && pend->set) {
    GemvArgs g;
    g.K = c.cfg.H;
    g.nseg = 1;
    g.seg[0].w = c.lm_head;
    g.seg[0].y = q.logits;
    g.seg[0].epi = c.cfg.has_softcap ? kEpiSoftcap : kEpiPlain;
    g.softcap = c.softcap;
    input_prologue(c, g, cur, c.final_norm, pend);
    launch_gemv(g, c.stream);
  } else {
    gemv_logits(c, cur, q.logits, c.stream);
  }
  launch_add_i32(q.d_pos, 1, c.stream);
}

// Full decode step for the token already in q.d_token (graph-capturable).
// Each layer's final norm + residual runs as the prologue of the next GEMV.
static void decode_step_launch(Ctx& c, Seq& q) {
  decode_embed(c, q, q.d_token);
  const int32_t* cur = c.dw.x0;
  PendingTail pend;
  for (int l = 0; l < c.cfg.L; ++l) cur = decode_layer(c, q, l, cur, &pend);
  decode_finalize_launch(c, q, cur, &pend);
}

static void select_launch(Ctx& c, Seq& q) {
  launch_argmax(q.logits, c.cfg.V, c.dw.argpart, c.argblocks, q.d_token, c.stream);
}

// The sequence's full logit row exists on this device.
static void require_logits(const Seq& q) {
  REQUIRE(q.prefilled, RDET_E_STATE, "no logits available (run prefill first)");
  REQUIRE(!q.logits_sharded, RDET_E_STATE,
          "the logits of this sequence are vocab-sharded over the tensor-parallel ranks "
          "(rdet_tp_shard_logits): select its token with rdet_select_batch");
}

// RoPE factors of every batch row at its own position, once per distinct
// frequency table, into the prefill's table buffer (rows <= max_prefill);
// qkv_post then reads them instead of evaluating sin/cos in every head.
static void batch_rope_tables(Ctx& c, int B) {
  for (size_t t = 0; t < c.rope_list.size(); ++t)
    launch_rope_rows(c.rope_list[t].first, c.rope_list[t].second, B, c.bw.pos,
                     c.rope_cs + t * (size_t)c.max_prefill * c.rope_half_max * 2, c.stream);
}
static const int32_t* rope_table_of(const Ctx& c, const int64_t* inv_freq) {
  for (size_t t = 0; t < c.rope_list.size(); ++t)
    if (c.rope_list[t].first == inv_freq) return c.rope_cs + t * (size_t)c.max_prefill * c.rope_half_max * 2;
  return nullptr;
}

static void check_decode_ready(Ctx& c, Seq& q) {
  REQUIRE(q.prefilled, RDET_E_STATE, "decode requires a prefilled sequence");
  REQUIRE(q.pos < q.cap, RDET_E_RANGE, "sequence KV cache is full");
  REQUIRE(c.prefill_owner == nullptr, RDET_E_STATE, "a routine-granular prefill is in flight on this context");
}

static void seq_alloc(Ctx& c, Seq& q, int cap) {
  const ModelCfg& m = c.cfg;
  q.ctx = &c;
  q.device = c.device;
  q.cap = cap;
  q.kc.assign(m.L, nullptr);
  q.vc.assign(m.L, nullptr);
  for (int l = 0; l < m.L; ++l) {
    const LayerCfg& lc = m.layers[l];
    if (lc.donor >= 0) continue;
    size_t n = (size_t)lc.kv_heads * cap * lc.head_dim;
    q.kc[l] = static_cast<int32_t*>(q.dalloc(n * 4));
    q.vc[l] = static_cast<int32_t*>(q.dalloc(n * 4));
  }
  {
    std::vector<unsigned char> maps((size_t)m.L * 256, 0);
    bool ok = true;
    for (int l = 0; l < m.L; ++l) {
      const LayerCfg& lc = m.layers[l];
      if (lc.donor >= 0 || lc.head_dim % 128 != 0) continue;
      const int rows = lc.kv_heads * cap;
      ok = ok && td_encode_cache_map(maps.data() + (size_t)l * 256, q.kc[l], rows, lc.head_dim) &&
           td_encode_cache_map(maps.data() + (size_t)l * 256 + 128, q.vc[l], rows, lc.head_dim);
    }
    q.d_maps = static_cast<unsigned char*>(q.dalloc(maps.size()));
    CK(cudaMemcpy(q.d_maps, maps.data(), maps.size(), cudaMemcpyHostToDevice));
    q.maps_ok = ok;
  }
  q.d_pos = static_cast<int32_t*>(q.dalloc(16));
  CK(cudaMemset(q.d_pos, 0, 16));
  q.logits = static_cast<int32_t*>(q.dalloc((size_t)m.V * 4));
  q.d_token = static_cast<uint32_t*>(q.dalloc(16));
  q.d_step = static_cast<int32_t*>(q.dalloc(16));
  q.dec_out = static_cast<int32_t*>(q.dalloc((size_t)m.L * m.H * 4));
  const int rps = 64;
  int splits = (cap + rps - 1) / rps;
  q.asc.max_splits = splits;
  q.asc.stride = cap;
  q.asc.scores = static_cast<int32_t*>(q.dalloc((size_t)m.Hq * cap * 4));
  q.asc.exps = static_cast<int64_t*>(q.dalloc((size_t)m.Hq * cap * 8));
  q.asc.pmax = static_cast<int32_t*>(q.dalloc((size_t)m.Hq * splits * 4));
  q.asc.pidx = static_cast<int32_t*>(q.dalloc((size_t)m.Hq * splits * 4));
  q.asc.psum = static_cast<int64_t*>(q.dalloc((size_t)m.Hq * splits * 8));
  q.asc.pwsum = static_cast<int64_t*>(q.dalloc((size_t)m.Hq * splits * 8));
  q.asc.pacc = static_cast<int64_t*>(q.dalloc((size_t)m.Hq * splits * c.dmax * 8));
}

// ---------------------------------------------------------------------------
// commitments / reads
// ---------------------------------------------------------------------------
static std::vector<int32_t> d2h(Ctx& c, const int32_t* p, size_t n) {
  std::vector<int32_t> h(n);
  if (n) CK(cudaMemcpyAsync(h.data(), p, n * 4, cudaMemcpyDeviceToHost, c.stream));
  CK(cudaStreamSynchronize(c.stream));
  return h;
}
// rows of the logical cache of (layer, head): trimmed sliding layers keep
// the last `window` rows (det_tensor.rs:308-337).
static void kv_rows(Ctx& c, Seq& q, int l, int* start, int* rows) {
  const LayerCfg& lc = c.cfg.layers[l];
  int len = q.pos;
  int keep = (lc.trim && len > lc.window) ? lc.window : len;
  *start = len - keep;
  *rows = keep;
}
static std::vector<int32_t> kv_read(Ctx& c, Seq& q, int l, int head, bool key) {
  const LayerCfg& lc = c.cfg.layers[l];
  int st, rows;
  kv_rows(c, q, l, &st, &rows);
  const int32_t* base = (key ? q.kc[l] : q.vc[l]) + ((size_t)head * q.cap + st) * lc.head_dim;
  return d2h(c, base, (size_t)rows * lc.head_dim);
}
// Over the caches of layers [0, nl) (the reference commits the caches built
// so far: after each prefill layer, and the whole list after prefill/decode).
// Hashes layer l's K then V cache in the commitment's byte order from host
// memory holding, per kind, every head's live rows back to back ([Hkv, rows,
// d], what kv_download writes).
static void kv_hash_layer(Sha256& h, const LayerCfg& lc, int rows, const int32_t* k, const int32_t* v) {
  h.put_u64((uint64_t)lc.kv_heads);
  for (int kind = 0; kind < 2; ++kind) {
    h.put(kind == 0 ? "k" : "v", 1);
    h.put_u64((uint64_t)lc.kv_heads);
    const int32_t* base = kind == 0 ? k : v;
    for (int hd = 0; hd < lc.kv_heads; ++hd) {
      h.put_u64((uint64_t)rows);
      const int32_t* hr = base + (size_t)hd * rows * lc.head_dim;
      for (int r = 0; r < rows; ++r) { h.put_u64((uint64_t)lc.head_dim); h.put(hr + (size_t)r * lc.head_dim, (size_t)lc.head_dim * 4); }
    }
  }
}

// Queues on c.stream one strided download of every head's live rows of
// layer l's K (kind 0) or V cache into dst.
static void kv_download(Ctx& c, Seq& q, int l, int kind, int32_t* dst) {
  const LayerCfg& lc = c.cfg.layers[l];
  int st, rows;
  kv_rows(c, q, l, &st, &rows);
  const size_t width = (size_t)rows * lc.head_dim * 4;
  const int32_t* src = (kind == 0 ? q.kc[l] : q.vc[l]) + (size_t)st * lc.head_dim;
  if (width)
    CK(cudaMemcpy2DAsync(dst, width, src, (size_t)q.cap * lc.head_dim * 4, width, lc.kv_heads,
                         cudaMemcpyDeviceToHost, c.stream));
}

static int32_t* pinned_alloc(size_t bytes, const char* what) {
  void* h = nullptr;
  if (cudaHostAlloc(&h, bytes ? bytes : 16, cudaHostAllocDefault) != cudaSuccess)
    throw Fail{RDET_E_OOM, std::string("pinned staging for the ") + what + " could not be allocated"};
  return static_cast<int32_t*>(h);
}

// Over the caches of layers [0, nl) (the reference commits the caches built
// so far: after each prefill layer, and the whole list after prefill/decode).
static bool kv_commitment(Ctx& c, Seq& q, std::string* out, int nl) {
  const ModelCfg& m = c.cfg;
  for (int l = 0; l < nl; ++l)
    if (!q.kc[l]) return false;  // a KV-sharing layer has no det cache of its own
  // both kinds of layer l+1 download into one half of the pinned stage while
  // layer l is hashed from the other
  size_t most = 0;
  for (int l = 0; l < nl; ++l) {
    int st, rows;
    kv_rows(c, q, l, &st, &rows);
    most = std::max(most, (size_t)2 * m.layers[l].kv_heads * rows * m.layers[l].head_dim);
  }
  KvStage& ks = c.kvs;
  if (!ks.ev[0]) {
    CK(cudaEventCreateWithFlags(&ks.ev[0], cudaEventDisableTiming));
    CK(cudaEventCreateWithFlags(&ks.ev[1], cudaEventDisableTiming));
  }
  if (ks.half_elems < most) {
    if (ks.host) CK(cudaFreeHost(ks.host));
    ks.host = nullptr;
    ks.half_elems = 0;
    ks.host = pinned_alloc(2 * most * 4, "KV commitment");
    ks.half_elems = most;
  }
  auto half = [&](int l) { return ks.host + (l & 1) * ks.half_elems; };
  auto enqueue = [&](int l) {
    const LayerCfg& lc = m.layers[l];
    int st, rows;
    kv_rows(c, q, l, &st, &rows);
    kv_download(c, q, l, 0, half(l));
    kv_download(c, q, l, 1, half(l) + (size_t)lc.kv_heads * rows * lc.head_dim);
    CK(cudaEventRecord(ks.ev[l & 1], c.stream));
  };
  Sha256 h;
  h.put("raster-det-num-kv-cache-v1", 26);
  h.put_u64((uint64_t)nl);
  if (nl) enqueue(0);
  for (int l = 0; l < nl; ++l) {
    if (l + 1 < nl) enqueue(l + 1);
    CK(cudaEventSynchronize(ks.ev[l & 1]));
    const LayerCfg& lc = m.layers[l];
    int st, rows;
    kv_rows(c, q, l, &st, &rows);
    kv_hash_layer(h, lc, rows, half(l), half(l) + (size_t)lc.kv_heads * rows * lc.head_dim);
  }
  *out = h.hex();
  return true;
}

// The commitments of the prefixes [0, p) for p = 1..n together: one download
// of the caches the longest prefix covers, then the prefixes' independent
// SHA-256 streams spread over host threads (longest first).  out[p-1] is
// empty where that prefix includes a KV-sharing layer.
static void kv_prefix_commitments(Ctx& c, Seq& q, int n, std::vector<std::string>* out) {
  const ModelCfg& m = c.cfg;
  out->assign(n, std::string());
  int own = 0;
  while (own < n && q.kc[own]) ++own;
  if (!own) return;
  std::vector<size_t> off(own + 1, 0);
  std::vector<int> rows(own);
  for (int l = 0; l < own; ++l) {
    int st;
    kv_rows(c, q, l, &st, &rows[l]);
    off[l + 1] = off[l] + (size_t)2 * m.layers[l].kv_heads * rows[l] * m.layers[l].head_dim;
  }
  std::unique_ptr<int32_t, cudaError_t (*)(void*)> host(pinned_alloc(off[own] * 4, "KV prefix commitments"),
                                                         cudaFreeHost);
  try {
    for (int l = 0; l < own; ++l) {
      const size_t kv = (size_t)m.layers[l].kv_heads * rows[l] * m.layers[l].head_dim;
      kv_download(c, q, l, 0, host.get() + off[l]);
      kv_download(c, q, l, 1, host.get() + off[l] + kv);
    }
    CK(cudaStreamSynchronize(c.stream));
  } catch (...) {
    cudaStreamSynchronize(c.stream);  // no download may still target the staging when it is freed
    throw;
  }
  std::atomic<int> next{0};
  auto work = [&] {
    for (int i; (i = next.fetch_add(1)) < own;) {
      const int p = own - i;  // longest prefix first
      Sha256 h;
      h.put("raster-det-num-kv-cache-v1", 26);
      h.put_u64((uint64_t)p);
      for (int l = 0; l < p; ++l) {
        const int32_t* k = host.get() + off[l];
        kv_hash_layer(h, m.layers[l], rows[l], k, k + (size_t)m.layers[l].kv_heads * rows[l] * m.layers[l].head_dim);
      }
      (*out)[p - 1] = h.hex();
    }
  };
  const unsigned hw = std::thread::hardware_concurrency();
  const int nt = std::max(1, std::min(own, std::min(8, (int)(hw > 1 ? hw - 1 : 1))));
  std::vector<std::thread> ts;
  for (int t = 1; t < nt; ++t) ts.emplace_back(work);
  work();
  for (auto& t : ts) t.join();
}

// Captures (once per sequence) the whole decode_transition of the token in
// d_token as one CUDA graph.
// ---------------------------------------------------------------------------
// Batched decode: every sequence of the batch advances by one token in one
// pass.  The projections run once over the batch rows (row GEMMs: tensor
// cores from 32 rows); q/k norm, RoPE, the KV append and the attention use
// each row's own position, caches and window.  Each row computes exactly
// what decode_layer computes for that sequence alone.
// ---------------------------------------------------------------------------
static void batch_tables(Ctx& c, Seq* const* seqs, int B) {
  const ModelCfg& m = c.cfg;
  auto& bw = c.bw;
  if (bw.rows < B) {
    const int rows = std::max(B, 8);
    const size_t ptrs = (size_t)rows * (4 + 2 * (size_t)m.L);
    const size_t bytes = ptrs * 8 + (size_t)rows * 12 + (size_t)rows * m.V * 4 + 256;
    bw.mem = c.dalloc(bytes);
    auto* base = static_cast<unsigned char*>(bw.mem);
    bw.pos = reinterpret_cast<int32_t**>(base);
    bw.dec_out = bw.pos + rows;
    bw.logits_dst = bw.dec_out + rows;
    bw.kc = bw.logits_dst + rows;
    bw.vc = bw.kc + (size_t)m.L * rows;
    bw.maps = reinterpret_cast<const unsigned char**>(reinterpret_cast<uintptr_t>(bw.vc + (size_t)m.L * rows));
    bw.ids = reinterpret_cast<uint32_t*>(reinterpret_cast<uintptr_t>(bw.maps + rows));
    bw.caps = reinterpret_cast<int32_t*>(bw.ids + rows);
    bw.order = bw.caps + rows;
    bw.logits = reinterpret_cast<int32_t*>((reinterpret_cast<uintptr_t>(bw.order + rows) + 255) & ~(uintptr_t)255);
    bw.rows = rows;
  }
  const int rows = bw.rows;
  std::vector<int32_t*> host((size_t)rows * (4 + 2 * (size_t)m.L), nullptr);
  bw.maps_ok = true;
  std::vector<int32_t> caps(2 * (size_t)rows, 0);  // [caps | row order]
  for (int b = 0; b < B; ++b) {
    Seq& q = *seqs[b];
    host[b] = q.d_pos;
    host[rows + b] = q.dec_out;
    host[2 * (size_t)rows + b] = q.logits;
    for (int l = 0; l < m.L; ++l) {
      const int own = m.layers[l].donor < 0 ? l : m.layers[l].donor;
      host[(3 + (size_t)l) * rows + b] = q.kc[own];
      host[(3 + (size_t)m.L + l) * rows + b] = q.vc[own];
    }
    host[(3 + 2 * (size_t)m.L) * rows + b] = reinterpret_cast<int32_t*>(q.d_maps);  // bw.maps[b]
    bw.maps_ok = bw.maps_ok && q.maps_ok;
    caps[b] = q.cap;
  }
  // attention launch order: longest context first (ties by row)
  int32_t* order = caps.data() + rows;
  for (int b = 0; b < rows; ++b) order[b] = b;
  std::stable_sort(order, order + B, [&](int32_t x, int32_t y) { return seqs[x]->pos > seqs[y]->pos; });
  CK(cudaMemcpyAsync(bw.pos, host.data(), host.size() * 8, cudaMemcpyHostToDevice, c.stream));
  CK(cudaMemcpyAsync(bw.caps, caps.data(), caps.size() * 4, cudaMemcpyHostToDevice, c.stream));
}

// in_planes: the layer input's norm already applied into w.nrm (and its
// tensor-core planes) by the previous layer's last row kernel when ready.
// next_gain / next_planes: this layer's last row kernel also writes
// norm(output) * next_gain into w.nrm and its planes (the next layer's input
// norm, or the final norm before lm_head), setting next_planes->ready.
static const int32_t* decode_batch_layer(Ctx& c, int B, int maxcap, int l, int32_t* cur, ActPlanes* in_planes,
                                         const int32_t* next_gain, ActPlanes* next_planes) {
  const ModelCfg& m = c.cfg;
  const LayerDev& L = c.layers[l];
  const LayerCfg& lc = L.cfg;
  PrefillWs& w = c.pw;
  auto& bw = c.bw;
  cudaStream_t s = c.stream;
  const int H = m.H, d = lc.head_dim;
  int32_t* other = cur == w.xa ? w.xb : w.xa;
  ActPlanes nrm_planes;
  if (in_planes && in_planes->ready) {
    nrm_planes = *in_planes;
  } else if (!in_planes || !in_planes->normed) {
    RowNormArgs ra;
    ra.a = cur; ra.g1 = L.in_ln; ra.n = H; ra.eps = c.eps; ra.y_out = w.nrm;
    if (!row_norm(c, ra, B, &nrm_planes)) launch_rmsnorm_rows(cur, B, H, L.in_ln, c.eps, w.nrm, s);
  }
  QkvPostArgs qa;
  qa.S = B; qa.Hq = m.Hq; qa.Hkv = lc.kv_heads; qa.d = d; qa.rotary = lc.rotary; qa.inv_freq = L.inv_freq;
  qa.q_norm = L.q_norm; qa.k_norm = L.k_norm; qa.eps = c.eps; qa.q_out = w.qo;
  qa.pos_rows = bw.pos; qa.cap_rows = bw.caps;
  qa.rope_cs = rope_table_of(c, L.inv_freq);
  // one tensor-core GEMM for q, k and v when their planes share a buffer
  // (rows [q | k | v] of w.hbuf, which the MLP overwrites later)
  const int nqkv = L.tqkv.nrows;
  if (lc.donor < 0 && nqkv > 0 && nrm_planes.ready && (size_t)nqkv <= (size_t)L.F) {
    TcOut o;
    o.y = w.hbuf;
    o.epi = kEpiPlain;
    o.scratch = c.tc_split;
    o.scratch_bytes = c.tc_split_bytes;
    launch_tc_linear(nrm_planes.a, L.tqkv, o, s);
    qa.ld = nqkv;
    qa.q_in = w.hbuf;
    qa.k_in = w.hbuf + L.q.rows;
    qa.v_in = L.v.p ? w.hbuf + L.q.rows + L.k.rows : qa.k_in;  // k_eq_v: V is the raw K projection
    qa.kc_rows = bw.kc + (size_t)l * bw.rows;
    qa.vc_rows = bw.vc + (size_t)l * bw.rows;
  } else {
    prefill_linear(c, w.nrm, B, L.q, L.tq, w.q, kEpiPlain, nullptr, &nrm_planes);
    qa.q_in = w.q;
    if (lc.donor < 0) {
      prefill_linear(c, w.nrm, B, L.k, L.tk, w.kraw, kEpiPlain, nullptr, &nrm_planes);
      const int32_t* vsrc = w.kraw;  // k_eq_v: V is the raw K projection
      if (L.v.p) { prefill_linear(c, w.nrm, B, L.v, L.tv, w.vraw, kEpiPlain, nullptr, &nrm_planes); vsrc = w.vraw; }
      qa.k_in = w.kraw; qa.v_in = vsrc;
      qa.kc_rows = bw.kc + (size_t)l * bw.rows;
      qa.vc_rows = bw.vc + (size_t)l * bw.rows;
    }
  }
  launch_qkv_post(qa, s);
  AttnDecodeArgs aa;
  aa.Hq = m.Hq; aa.Hkv = lc.kv_heads; aa.d = d; aa.window = lc.window; aa.q = w.qo; aa.out = w.comb;
  aa.cap = maxcap; aa.batch = B; aa.pos_rows = bw.pos; aa.cap_rows = bw.caps;
  aa.kc_rows = bw.kc + (size_t)l * bw.rows;
  aa.vc_rows = bw.vc + (size_t)l * bw.rows;
  aa.row_order = bw.order;
  aa.map_rows = bw.maps_ok ? bw.maps : nullptr;
  aa.map_layer = lc.donor < 0 ? l : lc.donor;
  launch_attn_decode_cluster(aa, s);
  prefill_linear(c, w.comb, B, L.o, L.to, w.attn, kEpiPlain, nullptr);
  const bool ple = m.P > 0;
  // post-attention norm + residual, then the MLP input norm (and its planes)
  ActPlanes ff_planes;
  {
    RowNormArgs ra;
    ra.a = w.attn; ra.res = cur; ra.g1 = L.post_attn_ln; ra.g2 = L.pre_ff_ln; ra.n = H; ra.eps = c.eps;
    ra.t_out = other; ra.y_out = w.nrm;
    if (!row_norm(c, ra, B, &ff_planes)) {
      launch_norm_residual_rows(w.attn, cur, B, H, L.post_attn_ln, c.eps, false, 0, other, s);
      launch_rmsnorm_rows(other, B, H, L.pre_ff_ln, c.eps, w.nrm, s);
    }
  }
  prefill_geglu(c, w.nrm, B, L, w.hbuf, &ff_planes);
  prefill_linear(c, w.hbuf, B, L.down, L.tdown, w.attn, kEpiPlain, nullptr);
  // post-MLP norm + residual: the layer output (no PLE; copied to each
  // sequence's layer-output row) or the per-layer-input GEMM's input
  ActPlanes pg_planes;
  bool scattered = false;
  {
    RowNormArgs ra;
    ra.a = w.attn; ra.res = other; ra.g1 = L.post_ff_ln; ra.n = H; ra.eps = c.eps;
    ra.has_scalar = !ple && L.has_scalar; ra.scalar = L.scalar; ra.t_out = cur;
    if (!ple) {
      ra.scatter = bw.dec_out; ra.scatter_off = (size_t)l * H;
      if (next_gain) { ra.g2 = next_gain; ra.y_out = w.nrm; }
    }
    if (row_norm(c, ra, B, ple ? &pg_planes : (next_gain ? next_planes : nullptr))) {
      scattered = !ple;
      if (!ple && next_gain) next_planes->normed = true;
    } else {
      launch_norm_residual_rows(w.attn, other, B, H, L.post_ff_ln, c.eps, !ple && L.has_scalar, L.scalar, cur, s);
    }
  }
  int32_t* result = cur;
  if (ple) {
    prefill_linear(c, cur, B, L.ple_gate, L.tpg, w.g, kEpiGeluMul, w.ple_all + (size_t)l * B * m.P, &pg_planes);
    prefill_linear(c, w.g, B, L.ple_proj, L.tpp, w.pr, kEpiPlain, nullptr);
    RowNormArgs ra;
    ra.a = w.pr; ra.res = cur; ra.g1 = L.ple_norm; ra.n = H; ra.eps = c.eps;
    ra.has_scalar = L.has_scalar; ra.scalar = L.scalar; ra.t_out = other;
    ra.scatter = bw.dec_out; ra.scatter_off = (size_t)l * H;
    if (next_gain) { ra.g2 = next_gain; ra.y_out = w.nrm; }
    if (row_norm(c, ra, B, next_gain ? next_planes : nullptr)) {
      scattered = true;
      if (next_gain) next_planes->normed = true;
    } else {
      launch_norm_residual_rows(w.pr, cur, B, H, L.ple_norm, c.eps, L.has_scalar, L.scalar, other, s);
    }
    result = other;
  }
  if (!scattered) launch_scatter_rows(result, B, H, bw.dec_out, (size_t)l * H, s);
  return result;
}

// ---------------------------------------------------------------------------
// Tensor-parallel batched decode.  Rank r of `world` computes query heads
// [head0, head0 + Hql) (q projection rows, attention), the gate/up rows
// [r*Fl, (r+1)*Fl), per-layer-input gate rows [r*Pl, (r+1)*Pl) and vocab
// rows [r*Vl, (r+1)*Vl).  The o, down and per-layer-input projections take
// the matching column slices and produce exact i64 partial sums that one
// NCCL all-reduce (int64 sum: wrapping addition is order-free) completes
// before requantize; logits are all-gathered.  K/V projections and appends
// run in full on every rank, so every rank's caches stay complete and every
// other path of the context stays valid.
// ---------------------------------------------------------------------------
static void tp_linear(Ctx& c, const int32_t* X, int S, int K, const TcWeight& w, const TcOut& o,
                      ActPlanes* shared = nullptr) {
  ActPlanes local;
  ActPlanes& ap = shared ? *shared : local;
  if (!ap.ready) {
    REQUIRE(tc_prepare_act(ap.a, X, S, K, c.tc_act, c.stream), RDET_E_CUDA, "tensor map encoding failed");
    ap.ready = true;
  }
  TcOut oo = o;
  oo.scratch = c.tc_split;
  oo.scratch_bytes = c.tc_split_bytes;
  REQUIRE(launch_tc_linear(ap.a, w, oo, c.stream), RDET_E_RANGE, "batch too large for the split-K scratch");
}

// Sums [S, N] of a column slice, completed over the ranks: with the NVLink
// reduction, left in this rank's alternating buffer and published to the
// peers (the next row kernel adds the peers' buffers as it loads); else an
// NCCL all-reduce in c.tp.part.  Either way the next row kernel requantizes.
static void tp_linear_sum(Ctx& c, const int32_t* X, int S, int K, const TcWeight& w) {
  TpState& t = c.tp;
  TcOut o;
  if (t.p2p) {
    REQUIRE(S <= t.p2p_rows, RDET_E_RANGE, "batch larger than the NVLink reduction buffers (rdet_tp_ipc_export)");
    const size_t slot = ((size_t)t.rank * 2 + (t.seq & 1)) * (size_t)t.p2p_rows * c.cfg.H;
    o.y64 = t.recv + slot;
    for (int r = 0; r < t.world; ++r)
      if (r != t.rank) o.y64_mirror.p[o.y64_mirror.n++] = t.peer_recv[r] + slot;
    tp_linear(c, X, S, K, w, o);
    t.last = o.y64;
    t.seq += 1;
    launch_tp_signal(t.peer_flags, t.world, t.rank, t.seq, c.stream);
    return;
  }
  o.y64 = t.part;
  tp_linear(c, X, S, K, w, o);
  NCK(nccl_api().allReduce(t.part, t.part, (size_t)S * w.N, ncclInt64, ncclSum, t.comm, c.stream));
  t.last = t.part;
}

// The row kernel's input after tp_linear_sum: the local sums plus, with the
// NVLink reduction, the peers' buffers of the same reduction and its flag.
static void tp_sum_input(const Ctx& c, RowNormArgs& ra) {
  const TpState& t = c.tp;
  ra.a64 = t.last;
  if (!t.p2p) return;
  const size_t slot = (t.seq - 1) & 1;
  for (int r = 0; r < t.world; ++r) {
    if (r == t.rank) continue;
    ra.a64_peer[ra.npeer++] = t.recv + ((size_t)r * 2 + slot) * (size_t)t.p2p_rows * c.cfg.H;
    ra.wait_mask |= 1u << r;
  }
  ra.flags = t.flags;
  ra.wait_seq = t.seq;
}

// in_planes / next_gain / next_planes as in decode_batch_layer.  The row
// kernels after each all-reduce requantize the summed partials on load
// (row_norm_kernel's i64 input), apply the norm and residual, and write the
// next GEMM's activation planes.
static const int32_t* decode_batch_layer_tp(Ctx& c, int B, int maxcap, int l, int32_t* cur, ActPlanes* in_planes,
                                            const int32_t* next_gain, ActPlanes* next_planes) {
  const ModelCfg& m = c.cfg;
  const LayerDev& L = c.layers[l];
  const LayerCfg& lc = L.cfg;
  const TpLayer& T = c.tp.layers[l];
  PrefillWs& w = c.pw;
  auto& bw = c.bw;
  cudaStream_t s = c.stream;
  const int H = m.H, d = lc.head_dim, Hql = c.tp.Hql;
  int32_t* other = cur == w.xa ? w.xb : w.xa;
  // sums of a column-sliced GEMM -> i32 rows, for the unfused fallbacks
  auto requantized = [&](int32_t* y) {
    REQUIRE(!c.tp.p2p, RDET_E_STATE, "the NVLink reduction needs 16-byte aligned rows");
    launch_requantize_rows(c.tp.part, (size_t)B * H, y, s);
    return y;
  };
  ActPlanes nrm_planes;
  if (in_planes && in_planes->ready) {
    nrm_planes = *in_planes;
  } else if (!in_planes || !in_planes->normed) {
    RowNormArgs ra;
    ra.a = cur; ra.g1 = L.in_ln; ra.n = H; ra.eps = c.eps; ra.y_out = w.nrm;
    if (!row_norm(c, ra, B, &nrm_planes)) launch_rmsnorm_rows(cur, B, H, L.in_ln, c.eps, w.nrm, s);
  }
  // this rank's query heads and the full K/V projections read the same planes
  TcOut oq;
  oq.y = w.q;
  tp_linear(c, w.nrm, B, H, T.q, oq, &nrm_planes);
  QkvPostArgs qa;
  qa.S = B; qa.Hq = Hql; qa.Hkv = lc.kv_heads; qa.d = d; qa.rotary = lc.rotary; qa.inv_freq = L.inv_freq;
  qa.q_in = w.q; qa.q_norm = L.q_norm; qa.k_norm = L.k_norm; qa.eps = c.eps; qa.q_out = w.qo;
  qa.pos_rows = bw.pos; qa.cap_rows = bw.caps;
  qa.rope_cs = rope_table_of(c, L.inv_freq);
  if (lc.donor < 0) {
    prefill_linear(c, w.nrm, B, L.k, L.tk, w.kraw, kEpiPlain, nullptr, &nrm_planes);
    const int32_t* vsrc = w.kraw;  // k_eq_v: V is the raw K projection
    if (L.v.p) { prefill_linear(c, w.nrm, B, L.v, L.tv, w.vraw, kEpiPlain, nullptr, &nrm_planes); vsrc = w.vraw; }
    qa.k_in = w.kraw; qa.v_in = vsrc;
    qa.kc_rows = bw.kc + (size_t)l * bw.rows;
    qa.vc_rows = bw.vc + (size_t)l * bw.rows;
  }
  launch_qkv_post(qa, s);
  AttnDecodeArgs aa;
  aa.Hq = Hql; aa.Hkv = lc.kv_heads; aa.group = m.Hq / lc.kv_heads; aa.head0 = c.tp.head0;
  aa.d = d; aa.window = lc.window; aa.q = w.qo; aa.out = w.comb;
  aa.cap = maxcap; aa.batch = B; aa.pos_rows = bw.pos; aa.cap_rows = bw.caps;
  aa.kc_rows = bw.kc + (size_t)l * bw.rows;
  aa.vc_rows = bw.vc + (size_t)l * bw.rows;
  aa.row_order = bw.order;
  aa.map_rows = bw.maps_ok ? bw.maps : nullptr;
  aa.map_layer = lc.donor < 0 ? l : lc.donor;
  launch_attn_decode_cluster(aa, s);
  tp_linear_sum(c, w.comb, B, Hql * d, T.o);
  const bool ple = m.P > 0;
  // post-attention norm + residual, then the MLP input norm and its planes
  ActPlanes ff_planes;
  {
    RowNormArgs ra;
    tp_sum_input(c, ra); ra.res = cur; ra.g1 = L.post_attn_ln; ra.g2 = L.pre_ff_ln; ra.n = H; ra.eps = c.eps;
    ra.t_out = other; ra.y_out = w.nrm;
    if (!row_norm(c, ra, B, &ff_planes)) {
      launch_norm_residual_rows(requantized(w.attn), cur, B, H, L.post_attn_ln, c.eps, false, 0, other, s);
      launch_rmsnorm_rows(other, B, H, L.pre_ff_ln, c.eps, w.nrm, s);
    }
  }
  TcOut og;
  og.y = w.hbuf;
  tp_linear(c, w.nrm, B, H, T.gu, og, &ff_planes);
  tp_linear_sum(c, w.hbuf, B, c.tp.Fl, T.down);
  // post-MLP norm + residual: the layer output, or the per-layer-input GEMM's input
  ActPlanes pg_planes;
  bool scattered = false;
  {
    RowNormArgs ra;
    tp_sum_input(c, ra); ra.res = other; ra.g1 = L.post_ff_ln; ra.n = H; ra.eps = c.eps;
    ra.has_scalar = !ple && L.has_scalar; ra.scalar = L.scalar; ra.t_out = cur;
    if (!ple) {
      ra.scatter = bw.dec_out; ra.scatter_off = (size_t)l * H;
      if (next_gain) { ra.g2 = next_gain; ra.y_out = w.nrm; }
    }
    if (row_norm(c, ra, B, ple ? &pg_planes : (next_gain ? next_planes : nullptr))) {
      scattered = !ple;
      if (!ple && next_gain) next_planes->normed = true;
    } else {
      launch_norm_residual_rows(requantized(w.attn), other, B, H, L.post_ff_ln, c.eps, !ple && L.has_scalar,
                                L.scalar, cur, s);
    }
  }
  int32_t* result = cur;
  if (ple) {
    TcOut op;
    op.y = w.g;
    op.epi = kEpiGeluMul;
    op.vec = w.ple_all + (size_t)l * B * m.P + (size_t)c.tp.rank * c.tp.Pl;
    op.ldv = m.P;
    tp_linear(c, cur, B, H, T.pg, op, &pg_planes);
    tp_linear_sum(c, w.g, B, c.tp.Pl, T.pp);
    RowNormArgs ra;
    tp_sum_input(c, ra); ra.res = cur; ra.g1 = L.ple_norm; ra.n = H; ra.eps = c.eps;
    ra.has_scalar = L.has_scalar; ra.scalar = L.scalar; ra.t_out = other;
    ra.scatter = bw.dec_out; ra.scatter_off = (size_t)l * H;
    if (next_gain) { ra.g2 = next_gain; ra.y_out = w.nrm; }
    if (row_norm(c, ra, B, next_gain ? next_planes : nullptr)) {
      scattered = true;
      if (next_gain) next_planes->normed = true;
    } else {
      launch_norm_residual_rows(requantized(w.pr), cur, B, H, L.ple_norm, c.eps, L.has_scalar, L.scalar, other, s);
    }
    result = other;
  }
  if (!scattered) launch_scatter_rows(result, B, H, bw.dec_out, (size_t)l * H, s);
  return result;
}

static void tp_buffers(Ctx& c, int B) {
  TpState& t = c.tp;
  if (t.rows >= B) return;
  const int rows = std::max(B, 8);
  t.part = c.dalloc_n<int64_t>((size_t)rows * c.cfg.H);
  t.lgl = c.dalloc_n<int32_t>((size_t)rows * t.Vl);
  t.lga = c.dalloc_n<int32_t>((size_t)t.world * rows * t.Vl);
  t.rows = rows;
}

static void tp_init(Ctx& c, int rank, int world, const ncclUniqueId& id) {
  const ModelCfg& m = c.cfg;
  TpState& t = c.tp;
  REQUIRE(t.comm == nullptr, RDET_E_STATE, "tensor-parallel decode is already set up on this context");
  REQUIRE(world >= 1 && rank >= 0 && rank < world, RDET_E_INVALID, "invalid tensor-parallel rank or world size");
  REQUIRE(c.tc, RDET_E_STATE, "tensor-parallel decode runs on the tensor-core linear (sm_100, i16 weights)");
  REQUIRE(nccl_api().ok, RDET_E_STATE, "libnccl.so.2 could not be loaded");
  REQUIRE(m.Hq % world == 0, RDET_E_INVALID, "num_attention_heads must be a multiple of the world size");
  const int Hql = m.Hq / world;
  for (const LayerDev& L : c.layers) {
    const int G = m.Hq / L.cfg.kv_heads;
    REQUIRE(Hql % G == 0 || G % Hql == 0, RDET_E_INVALID, "each rank's query heads must cover whole KV groups");
    REQUIRE((Hql * L.cfg.head_dim) % 16 == 0, RDET_E_INVALID, "head slice width must be a multiple of 16");
    REQUIRE(L.F % world == 0 && (L.F / world) % 16 == 0, RDET_E_INVALID,
            "intermediate_size / world must be a multiple of 16");
    REQUIRE(L.tq.planes && L.to.planes && L.tgu.planes && L.tdown.planes, RDET_E_STATE,
            "tensor-parallel decode needs i16 projection weights");
  }
  if (m.P > 0)
    REQUIRE(m.P % world == 0 && (m.P / world) % 16 == 0, RDET_E_INVALID,
            "hidden_size_per_layer_input / world must be a multiple of 16");
  REQUIRE(m.V % world == 0 && c.t_lm_head.planes, RDET_E_INVALID, "vocab_size must be a multiple of the world size");
  t.rank = rank;
  t.world = world;
  t.Hql = Hql;
  t.head0 = rank * Hql;
  t.Fl = c.F / world;
  t.Pl = m.P > 0 ? m.P / world : 0;
  t.Vl = m.V / world;
  t.layers.assign(m.L, TpLayer());
  auto slice = [&](TcWeight& tw, const DevMat& g, const DevMat* u, int row0, int rows, int col0, int cols) {
    void* mem = c.dalloc(tc_weight_bytes(rows, cols, u != nullptr));
    REQUIRE(tc_prepare_weight_slice(tw, g, u, row0, rows, col0, cols, mem, c.stream), RDET_E_CUDA,
            "tensor map encoding failed");
  };
  for (int l = 0; l < m.L; ++l) {
    const LayerDev& L = c.layers[l];
    TpLayer& T = t.layers[l];
    const int d = L.cfg.head_dim, Fl = L.F / world;
    slice(T.q, L.q, nullptr, t.head0 * d, Hql * d, 0, m.H);
    slice(T.o, L.o, nullptr, 0, m.H, t.head0 * d, Hql * d);
    slice(T.gu, L.gate, &L.up, rank * Fl, Fl, 0, m.H);
    slice(T.down, L.down, nullptr, 0, m.H, rank * Fl, Fl);
    if (m.P > 0) {
      slice(T.pg, L.ple_gate, nullptr, rank * t.Pl, t.Pl, 0, m.H);
      slice(T.pp, L.ple_proj, nullptr, 0, m.H, rank * t.Pl, t.Pl);
    }
  }
  slice(t.lm, c.lm_head, nullptr, rank * t.Vl, t.Vl, 0, m.H);
  CK(cudaStreamSynchronize(c.stream));
  CK(cudaGetLastError());
  NCK(nccl_api().commInitRank(&t.comm, world, id, rank));
}

static void decode_batch_tp(Ctx& c, Seq* const* seqs, const uint32_t* tokens, int B, int row0) {
  const ModelCfg& m = c.cfg;
  PrefillWs& w = c.pw;
  cudaStream_t s = c.stream;
  batch_tables(c, seqs, B);
  batch_rope_tables(c, B);
  tp_buffers(c, B);
  auto& bw = c.bw;
  int maxcap = 0;
  for (int i = 0; i < B; ++i) maxcap = std::max(maxcap, seqs[i]->cap);
  CK(cudaMemcpyAsync(bw.ids, tokens, (size_t)B * 4, cudaMemcpyHostToDevice, s));
  launch_embed(bw.ids, B, c.emb, c.emb_scale, w.xa, c.d_err, s);
  if (m.P > 0) {
    prefill_linear(c, w.xa, B, c.ple_model_proj, c.t_ple_model, w.ple_proj, kEpiPlain, nullptr);
    PleArgs pa;
    pa.S = B; pa.L = m.L; pa.P = m.P; pa.ids = bw.ids; pa.proj = w.ple_proj; pa.table = c.ple_table;
    pa.norm = c.ple_proj_norm; pa.eps = c.eps; pa.emb_scale = c.ple_emb_scale; pa.proj_scale = c.ple_proj_scale;
    pa.in_scale = c.ple_in_scale; pa.out = w.ple_all; pa.err = c.d_err;
    launch_ple(pa, s);
  }
  int32_t* cur = w.xa;
  ActPlanes carry;  // the next layer's (or lm_head's) normalized input, made by the previous layer
  for (int l = 0; l < m.L; ++l) {
    ActPlanes next;
    const int32_t* gain = l + 1 < m.L ? c.layers[l + 1].in_ln : c.final_norm;
    cur = const_cast<int32_t*>(decode_batch_layer_tp(c, B, maxcap, l, cur, &carry, gain, &next));
    carry = next;
  }
  if (!carry.normed) launch_rmsnorm_rows(cur, B, m.H, c.final_norm, c.eps, w.nrm, s);
  TcOut ol;
  ol.y = c.tp.lgl;
  tp_linear(c, w.nrm, B, m.H, c.tp.lm, ol, carry.ready ? &carry : nullptr);
  if (m.has_softcap) launch_softcap(c.tp.lgl, B * c.tp.Vl, c.softcap, s);
  TpState& t = c.tp;
  if (t.shard_logits) {
    // global argmax over the vocab-sharded logits: each rank's first max per
    // chunk of its rows as (value, global index), all-gathered (8 bytes per
    // chunk and row), then reduced per row; the logit rows stay sharded
    const int chunks = t.sel_chunks;
    launch_argmax_rows(nullptr, t.lgl, B, t.Vl, (size_t)t.Vl, t.rank * t.Vl, chunks, t.lpairs, s);
    NCK(nccl_api().allGather(t.lpairs, t.gpairs, (size_t)B * chunks * 2, ncclInt32, t.comm, s));
    launch_argmax_rows_final(t.gpairs, t.world, B, chunks, t.tokens + row0, s);
  } else {
    NCK(nccl_api().allGather(t.lgl, t.lga, (size_t)B * t.Vl, ncclInt32, t.comm, s));
    launch_gather_vocab(t.lga, t.world, B, t.Vl, bw.logits_dst, s);
  }
  launch_add_i32_rows(bw.pos, B, 1, s);
  CK(cudaGetLastError());
  for (int i = 0; i < B; ++i) {
    seqs[i]->pos += 1;
    seqs[i]->last_was_prefill = false;
    seqs[i]->logits_sharded = t.shard_logits;
    seqs[i]->sel_row = row0 + i;
    seqs[i]->sel_epoch = t.epoch;
  }
}

// Capacity of the vocab-sharded selection buffers for a decode of nseq rows.
static void tp_select_buffers(Ctx& c, int nseq) {
  TpState& t = c.tp;
  const int B = std::min<int>(nseq, (int)c.max_prefill);
  const int chunks = std::max(1, std::min(32, std::min(256 / std::max(1, B), t.Vl / 256)));
  if (t.sel_rows >= nseq && t.sel_chunks >= chunks) return;
  const int rows = std::max(nseq, 8);
  t.sel_chunks = std::max(chunks, t.sel_chunks);
  t.lpairs = c.dalloc_n<int32_t>((size_t)rows * t.sel_chunks * 2);
  t.gpairs = c.dalloc_n<int32_t>((size_t)t.world * rows * t.sel_chunks * 2);
  t.tokens = c.dalloc_n<uint32_t>((size_t)rows);
  t.sel_rows = rows;
}

// Whether the batched path can run these sequences (distinct, and the
// batched cluster attention fits every layer's window).
static bool batch_supported(Ctx& c, Seq* const* seqs, int B) {
  if (B < 2) return false;
  for (int i = 0; i < B; ++i)
    for (int j = 0; j < i; ++j)
      if (seqs[i] == seqs[j]) return false;
  int maxcap = 0;
  for (int i = 0; i < B; ++i) maxcap = std::max(maxcap, seqs[i]->cap);
  const bool tp = c.tp.comm != nullptr;
  for (const LayerDev& L : c.layers) {
    const int hq = tp ? c.tp.Hql : c.cfg.Hq, group = tp ? c.cfg.Hq / L.cfg.kv_heads : 0;
    if (!attn_decode_cluster_fits(hq, L.cfg.kv_heads, L.cfg.head_dim, L.cfg.window, maxcap, 0, group)) return false;
  }
  return true;
}

static void decode_batch(Ctx& c, Seq* const* seqs, const uint32_t* tokens, int B) {
  const ModelCfg& m = c.cfg;
  PrefillWs& w = c.pw;
  cudaStream_t s = c.stream;
  batch_tables(c, seqs, B);
  batch_rope_tables(c, B);
  auto& bw = c.bw;
  int maxcap = 0;
  for (int i = 0; i < B; ++i) maxcap = std::max(maxcap, seqs[i]->cap);
  CK(cudaMemcpyAsync(bw.ids, tokens, (size_t)B * 4, cudaMemcpyHostToDevice, s));
  launch_embed(bw.ids, B, c.emb, c.emb_scale, w.xa, c.d_err, s);
  if (m.P > 0) {
    prefill_linear(c, w.xa, B, c.ple_model_proj, c.t_ple_model, w.ple_proj, kEpiPlain, nullptr);
    PleArgs pa;
    pa.S = B; pa.L = m.L; pa.P = m.P; pa.ids = bw.ids; pa.proj = w.ple_proj; pa.table = c.ple_table;
    pa.norm = c.ple_proj_norm; pa.eps = c.eps; pa.emb_scale = c.ple_emb_scale; pa.proj_scale = c.ple_proj_scale;
    pa.in_scale = c.ple_in_scale; pa.out = w.ple_all; pa.err = c.d_err;
    launch_ple(pa, s);
  }
  int32_t* cur = w.xa;
  ActPlanes carry;  // the next layer's (or lm_head's) normalized input, made by the previous layer
  for (int l = 0; l < m.L; ++l) {
    ActPlanes next;
    const int32_t* gain = l + 1 < m.L ? c.layers[l + 1].in_ln : c.final_norm;
    cur = const_cast<int32_t*>(decode_batch_layer(c, B, maxcap, l, cur, &carry, gain, &next));
    carry = next;
  }
  if (!carry.normed) launch_rmsnorm_rows(cur, B, m.H, c.final_norm, c.eps, w.nrm, s);
  prefill_linear(c, w.nrm, B, c.lm_head, c.t_lm_head, bw.logits, kEpiPlain, nullptr, carry.ready ? &carry : nullptr);
  launch_scatter_rows(bw.logits, B, m.V, bw.logits_dst, 0, s, m.has_softcap ? c.softcap : 0);
  launch_add_i32_rows(bw.pos, B, 1, s);
  CK(cudaGetLastError());
  for (int i = 0; i < B; ++i) {
    seqs[i]->pos += 1;
    seqs[i]->last_was_prefill = false;
  }
}

static void ensure_decode_graph(Ctx& c, Seq& q) {
  if (q.graph) return;
  cudaGraph_t g;
  CK(cudaStreamBeginCapture(c.stream, cudaStreamCaptureModeThreadLocal));
  decode_step_launch(c, q);
  cudaError_t e = cudaStreamEndCapture(c.stream, &g);
  if (e != cudaSuccess) throw Fail{RDET_E_CUDA, std::string("graph capture failed: ") + cudaGetErrorString(e)};
  size_t n = 0;
  cudaGraphGetNodes(g, nullptr, &n);
  std::vector<cudaGraphNode_t> nodes(n);
  cudaGraphGetNodes(g, nodes.data(), &n);
  int kernels = 0;
  for (auto nd : nodes) {
    cudaGraphNodeType ty;
    if (cudaGraphNodeGetType(nd, &ty) == cudaSuccess && ty == cudaGraphNodeTypeKernel) ++kernels;
  }
  q.graph_kernels = kernels;
  e = cudaGraphInstantiate(&q.graph, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) { q.graph = nullptr; throw Fail{RDET_E_CUDA, std::string("graph instantiate failed: ") + cudaGetErrorString(e)}; }
}

static void check_token(Ctx& c, uint32_t token) {
  REQUIRE(token < (uint32_t)c.emb.rows, RDET_E_RANGE, "token id " + std::to_string(token) + " is out of bounds for embedding tensor");
  if (c.cfg.P > 0) REQUIRE(token < (uint32_t)c.cfg.ple_vocab, RDET_E_RANGE, "token id is out of bounds for the PLE table");
}

// Decode-attention scratch of the kernel-level entry point: allocated on first
// use per device and grown on demand.
struct AttnScratchOwned {
  AttnScratch sc;
  int heads = 0, rows = 0, splits = 0, dim = 0;
  std::vector<void*> ptrs;
};
static std::map<int, AttnScratchOwned> g_attn_scratch;
// held from the lookup (and any regrowth) of a device's scratch until the
// kernel that uses it is enqueued, so two host threads never grow, free or
// hand out one device's scratch at the same time
static std::mutex g_attn_scratch_mu;
// byte-plane scratch of the kernel-level tensor-core linear, per device
struct LinScratch {
  void* p = nullptr;
  size_t bytes = 0;
};
static std::map<int, LinScratch> g_lin_scratch;
static std::mutex g_lin_scratch_mu;
// scratch of the kernel-level prefill attention, per device (same rules)
static std::map<int, LinScratch> g_pattn_scratch;
static std::mutex g_pattn_scratch_mu;

static void attn_entry_args(AttnDecodeArgs& a, const int32_t* q, const int32_t* k_cache, const int32_t* v_cache,
                            uint32_t cap, uint32_t num_heads, uint32_t num_kv_heads, uint32_t head_dim,
                            uint32_t position, uint32_t window, int32_t* out) {
  REQUIRE(q && k_cache && v_cache && out, RDET_E_INVALID, "null argument");
  REQUIRE(num_kv_heads > 0 && num_heads % num_kv_heads == 0 && num_heads / num_kv_heads <= 8, RDET_E_INVALID,
          "num_heads must be a multiple of num_kv_heads with at most 8 query heads per KV head");
  REQUIRE(head_dim > 0 && head_dim <= 1024, RDET_E_RANGE, "head_dim out of range");
  REQUIRE(position < cap, RDET_E_RANGE, "position must be below the cache capacity");
  a.pos = nullptr;
  a.pos_value = (int32_t)position;
  a.Hq = (int)num_heads;
  a.Hkv = (int)num_kv_heads;
  a.d = (int)head_dim;
  a.window = (int)window;
  a.q = q;
  a.k_cache = k_cache;
  a.v_cache = v_cache;
  a.cap = (int)cap;
  a.out = out;
  a.rows_per_split = 64;
}
static int attn_rows(uint32_t position, uint32_t window) {
  int len = (int)position + 1;
  return (window > 0 && len > (int)window) ? (int)window : len;
}

// ---------------------------------------------------------------------------
// Decode attention without allocation: its scratch is a fixed array compiled
// into this library (every GPU that loads the library holds it until the
// process exits).  Host code never uses the array's name as an address: the
// device address comes from cudaGetSymbolAddress, looked up once per device
// with that device current.
// ---------------------------------------------------------------------------
constexpr int kNoAllocMaxHeads = 16, kNoAllocMaxRows = 4096, kNoAllocMaxHeadDim = 512;
constexpr int kNoAllocRowsPerSplit = 64, kNoAllocMaxSplits = kNoAllocMaxRows / kNoAllocRowsPerSplit;
constexpr size_t kNaScores = 0;
constexpr size_t kNaExps = kNaScores + (size_t)kNoAllocMaxHeads * kNoAllocMaxRows * 4;
constexpr size_t kNaPmax = kNaExps + (size_t)kNoAllocMaxHeads * kNoAllocMaxRows * 8;
constexpr size_t kNaPidx = kNaPmax + (size_t)kNoAllocMaxHeads * kNoAllocMaxSplits * 4;
constexpr size_t kNaPsum = kNaPidx + (size_t)kNoAllocMaxHeads * kNoAllocMaxSplits * 4;
constexpr size_t kNaPwsum = kNaPsum + (size_t)kNoAllocMaxHeads * kNoAllocMaxSplits * 8;
constexpr size_t kNaPacc = kNaPwsum + (size_t)kNoAllocMaxHeads * kNoAllocMaxSplits * 8;
constexpr size_t kNaBytes = kNaPacc + (size_t)kNoAllocMaxHeads * kNoAllocMaxSplits * kNoAllocMaxHeadDim * 8;
static_assert(kNaExps % 256 == 0 && kNaPmax % 256 == 0 && kNaPidx % 256 == 0 && kNaPsum % 256 == 0 &&
                  kNaPwsum % 256 == 0 && kNaPacc % 256 == 0,
              "scratch sections stay 256-byte aligned");

static __device__ __align__(256) unsigned char g_attn_noalloc_scratch[kNaBytes];

static std::mutex g_noalloc_mu;
static std::map<int, unsigned char*> g_noalloc_addr;  // device ordinal -> device address of the array

static unsigned char* noalloc_scratch_current_device() {
  int dev = 0;
  CK(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  auto it = g_noalloc_addr.find(dev);
  if (it != g_noalloc_addr.end()) return it->second;
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_attn_noalloc_scratch);
  REQUIRE(e == cudaSuccess && p, RDET_E_CUDA,
          std::string("cudaGetSymbolAddress of the attention scratch failed: ") + cudaGetErrorString(e));
  g_noalloc_addr[dev] = static_cast<unsigned char*>(p);
  return static_cast<unsigned char*>(p);
}

}  // namespace rdet

// ===========================================================================
// C ABI
// ===========================================================================
using namespace rdet;

struct rdet_ctx { std::unique_ptr<Ctx> c; };
struct rdet_seq { std::unique_ptr<Seq> s; rdet_ctx* owner; };

template <typename F>
static int32_t guard(F&& f) {
  try {
    f();
    return RDET_OK;
  } catch (const Fail& e) {
    g_last_error = e.msg;
    return e.code;
  } catch (const std::bad_alloc&) {
    g_last_error = "host out of memory";
    return RDET_E_OOM;
  } catch (const std::exception& e) {
    g_last_error = e.what();
    return RDET_E_INVALID;
  }
}

static void open_common(Ctx& c, const rdet_opts* opts) {
  c.device = opts ? opts->device : 0;
  c.max_prefill = (opts && opts->max_prefill) ? opts->max_prefill : 4096;
  c.flags = opts ? opts->flags : 0;
  int ndev = 0;
  CK(cudaGetDeviceCount(&ndev));
  REQUIRE(c.device >= 0 && c.device < ndev, RDET_E_INVALID, "invalid CUDA device ordinal");
  CK(cudaSetDevice(c.device));
  CK(cudaStreamCreateWithFlags(&c.stream, cudaStreamNonBlocking));
  kernels_init();
}

static std::string read_file(const std::string& path) {
  FILE* f = fopen(path.c_str(), "rb");
  REQUIRE(f, RDET_E_IO, "failed to open " + path);
  std::string s;
  char buf[65536];
  size_t n;
  while ((n = fread(buf, 1, sizeof(buf), f)) > 0) s.append(buf, n);
  fclose(f);
  return s;
}

extern "C" {

const char* rdet_version(void) { return "rdet 0.1 (det_num spec 1, detwgt 2, sm_100a)"; }

int32_t rdet_last_error(char* buf, size_t len) {
  if (buf && len) snprintf(buf, len, "%s", g_last_error.c_str());
  return (int32_t)g_last_error.size();
}

int32_t rdet_open(const char* model_dir, const rdet_opts* opts, rdet_ctx** out) {
  return guard([&] {
    REQUIRE(model_dir && out, RDET_E_INVALID, "null argument");
    auto h = std::make_unique<rdet_ctx>();
    h->c = std::make_unique<Ctx>();
    Ctx& c = *h->c;
    // Parse and validate everything on the host before touching the GPU, so
    // malformed models fail closed with RDET_E_FORMAT on any machine.
    std::string dir(model_dir);
    c.cfg = parse_config(read_file(dir + "/config.json"));
    std::string wpath = dir + "/model.detwgt";
    int fd = open(wpath.c_str(), O_RDONLY);
    REQUIRE(fd >= 0, RDET_E_IO, "failed to open deterministic artifact " + wpath);
    struct stat st;
    fstat(fd, &st);
    MappedFile mf;
    mf.size = (size_t)st.st_size;
    mf.base = mf.size ? mmap(nullptr, mf.size, PROT_READ, MAP_PRIVATE, fd, 0) : nullptr;
    close(fd);
    REQUIRE(mf.size == 0 || mf.base != MAP_FAILED, RDET_E_IO, "failed to mmap deterministic artifact " + wpath);
    auto tab = parse_detwgt(static_cast<const uint8_t*>(mf.base), mf.size);
    {
      Ctx probe;  // dry pass: every tensor the model needs exists with the right shape
      probe.cfg = c.cfg;
      build_model(probe, tab, false, 0, true);
    }
    open_common(c, opts);
    build_model(c, tab, false, 0);
    alloc_workspaces(c);
    prepare_tensor_cores(c);
    *out = h.release();
  });
}

int32_t rdet_open_synthetic(const char* config_json, uint64_t seed, int32_t width, const rdet_opts* opts,
                            rdet_ctx** out) {
  return guard([&] {
    REQUIRE(config_json && out, RDET_E_INVALID, "null argument");
    REQUIRE(width == 16 || width == 32, RDET_E_INVALID, "width must be 16 or 32");
    auto h = std::make_unique<rdet_ctx>();
    h->c = std::make_unique<Ctx>();
    Ctx& c = *h->c;
    c.cfg = parse_config(config_json);
    json::Value root = json::parse(config_json);
    const json::Value& t = text_cfg(root);
    int F = (int)req_int(t, "intermediate_size");
    auto tab = synthetic_table(c.cfg, t, width, F);
    open_common(c, opts);
    build_model(c, tab, true, seed);
    alloc_workspaces(c);
    prepare_tensor_cores(c);
    *out = h.release();
  });
}

int32_t rdet_close(rdet_ctx* ctx) {
  return guard([&] {
    if (!ctx) return;
    // Sequences still open on this context are freed with it; their handles
    // must not be used afterwards.
    std::vector<void*> live = ctx->c->live_seqs;
    for (void* p : live) delete static_cast<rdet_seq*>(p);
    delete ctx;
  });
}

int32_t rdet_get_model_info(rdet_ctx* ctx, rdet_model_info* out) {
  return guard([&] {
    REQUIRE(ctx && out, RDET_E_INVALID, "null argument");
    const Ctx& c = *ctx->c;
    out->hidden_size = c.cfg.H;
    out->vocab_size = c.cfg.V;
    out->num_layers = c.cfg.L;
    out->num_heads = c.cfg.Hq;
    out->ple_dim = c.cfg.P;
    out->intermediate_size = c.F;
    out->weight_bytes = c.weight_bytes;
  });
}

int32_t rdet_seq_new(rdet_ctx* ctx, uint32_t max_ctx, rdet_seq** out) {
  return guard([&] {
    REQUIRE(ctx && out, RDET_E_INVALID, "null argument");
    REQUIRE(max_ctx > 0, RDET_E_INVALID, "max_ctx must be positive");
    CK(cudaSetDevice(ctx->c->device));
    auto h = std::make_unique<rdet_seq>();
    h->s = std::make_unique<Seq>();
    h->owner = ctx;
    seq_alloc(*ctx->c, *h->s, (int)max_ctx);
    ctx->c->live_seqs.push_back(h.get());
    *out = h.release();
  });
}

int32_t rdet_seq_free(rdet_seq* seq) {
  return guard([&] {
    if (!seq) return;
    Ctx& c = *seq->owner->c;
    if (c.prefill_owner == seq->s.get()) c.prefill_owner = nullptr;
    if (c.decode_owner == seq->s.get()) c.decode_owner = nullptr;
    auto it = std::find(c.live_seqs.begin(), c.live_seqs.end(), (void*)seq);
    REQUIRE(it != c.live_seqs.end(), RDET_E_INVALID, "unknown sequence handle");
    c.live_seqs.erase(it);
    delete seq;
  });
}

int32_t rdet_seq_position(rdet_seq* seq, uint32_t* position) {
  return guard([&] {
    REQUIRE(seq && position, RDET_E_INVALID, "null argument");
    *position = (uint32_t)seq->s->pos;
  });
}

int32_t rdet_embed(rdet_ctx* ctx, const uint32_t* ids, size_t n, int32_t* act_out) {
  return guard([&] {
    REQUIRE(ctx && ids && act_out, RDET_E_INVALID, "null argument");
    Ctx& c = *ctx->c;
    CK(cudaSetDevice(c.device));
    REQUIRE(n > 0, RDET_E_INVALID, "transformer embedding requires at least one token id");
    REQUIRE(n <= c.max_prefill, RDET_E_RANGE, "too many token ids");
    REQUIRE(c.prefill_owner == nullptr, RDET_E_STATE, "a routine-granular prefill is in flight on this context");
    for (size_t i = 0; i < n; ++i)
      REQUIRE(ids[i] < (uint32_t)c.emb.rows, RDET_E_RANGE, "token id " + std::to_string(ids[i]) + " is out of bounds for embedding tensor");
    CK(cudaMemcpyAsync(c.pw.ids, ids, n * 4, cudaMemcpyHostToDevice, c.stream));
    launch_embed(c.pw.ids, (int)n, c.emb, c.emb_scale, c.pw.x0, c.d_err, c.stream);
    CK(cudaGetLastError());
    CK(cudaMemcpyAsync(act_out, c.pw.x0, n * c.cfg.H * 4, cudaMemcpyDeviceToHost, c.stream));
    check_err_flag(c, "embed");
  });
}

int32_t rdet_prefill_begin(rdet_ctx* ctx, rdet_seq* seq, const uint32_t* ids, size_t n) {
  return guard([&] {
    REQUIRE(ctx && seq && ids, RDET_E_INVALID, "null argument");
    Ctx& c = *ctx->c;
    CK(cudaSetDevice(c.device));
    REQUIRE(seq->owner == ctx, RDET_E_INVALID, "sequence belongs to another context");
    REQUIRE(c.prefill_owner == nullptr || c.prefill_owner == seq->s.get(), RDET_E_STATE, "another prefill is in flight on this context");
    prefill_begin(c, *seq->s, ids, n);
  });
}

int32_t rdet_prefill_range(rdet_ctx* ctx, rdet_seq* seq, uint32_t layer_start, uint32_t layer_end) {
  return guard([&] {
    REQUIRE(ctx && seq, RDET_E_INVALID, "null argument");
    Ctx& c = *ctx->c;
    Seq& q = *seq->s;
    CK(cudaSetDevice(c.device));
    REQUIRE(c.prefill_owner == &q, RDET_E_STATE, "prefill.range requires prefill_begin on this sequence");
    REQUIRE((int)layer_start == q.prefill_next, RDET_E_STATE, "prefill.range must continue at the next layer");
    REQUIRE(layer_end >= layer_start && (int)layer_end <= c.cfg.L, RDET_E_RANGE, "layer range out of bounds");
    struct JoinAtExit {  // no layer hash outlives the call, whatever happens
      Ctx& c;
      ~JoinAtExit() { commit_join(c, false); }
    } join{c};
    for (uint32_t l = layer_start; l < layer_end; ++l) {
      prefill_layer(c, q, (int)l);
      q.prefill_next = (int)l + 1;
    }
    CK(cudaStreamSynchronize(c.stream));
    commit_join(c, true);
  });
}

int32_t rdet_prefill_finalize(rdet_ctx* ctx, rdet_seq* seq) {
  return guard([&] {
    REQUIRE(ctx && seq, RDET_E_INVALID, "null argument");
    Ctx& c = *ctx->c;
    CK(cudaSetDevice(c.device));
    REQUIRE(c.prefill_owner == seq->s.get(), RDET_E_STATE, "prefill.finalize requires prefill_begin on this sequence");
    prefill_finalize(c, *seq->s);
  });
}

int32_t rdet_prefill(rdet_ctx* ctx, rdet_seq* seq, const uint32_t* ids, size_t n) {
  int32_t rc = rdet_prefill_begin(ctx, seq, ids, n);
  if (rc != RDET_OK) return rc;
  rc = rdet_prefill_range(ctx, seq, 0, ctx->c->cfg.L);
  if (rc != RDET_OK) { ctx->c->prefill_owner = nullptr; return rc; }
  rc = rdet_prefill_finalize(ctx, seq);
  if (rc != RDET_OK) ctx->c->prefill_owner = nullptr;
  return rc;
}

int32_t rdet_select(rdet_ctx* ctx, rdet_seq* seq, uint32_t* token_out) {
  return guard([&] {
    REQUIRE(ctx && seq && token_out, RDET_E_INVALID, "null argument");
    Ctx& c = *ctx->c;
    Seq& q = *seq->s;
    CK(cudaSetDevice(c.device));
    require_logits(q);
    select_launch(c, q);
    CK(cudaGetLastError());
    CK(cudaMemcpyAsync(token_out, q.d_token, 4, cudaMemcpyDeviceToHost, c.stream));
    CK(cudaStreamSynchronize(c.stream));
  });
}

int32_t rdet_select_batch(rdet_ctx* ctx, rdet_seq* const* seqs, size_t n, uint32_t* tokens_out) {
  return guard([&] {
    REQUIRE(ctx && (n == 0 || (seqs && tokens_out)), RDET_E_INVALID, "null argument");
    Ctx& c = *ctx->c;
    CK(cudaSetDevice(c.device));
    REQUIRE(n <= (1u << 20), RDET_E_RANGE, "at most 2^20 sequences per call");
    std::vector<int> full;           // positions whose logit rows are on this device
    std::vector<int> sharded;        // positions selected by the last vocab-sharded decode
    for (size_t i = 0; i < n; ++i) {
      REQUIRE(seqs[i] && seqs[i]->owner == ctx, RDET_E_INVALID, "sequence belongs to another context");
      const Seq& q = *seqs[i]->s;
      REQUIRE(q.prefilled, RDET_E_STATE, "no logits available (run prefill first)");
      if (q.logits_sharded) {
        REQUIRE(q.sel_epoch == c.tp.epoch && q.sel_row >= 0 && q.sel_row < c.tp.sel_rows, RDET_E_STATE,
                "a later batched decode replaced this sequence's selected token: select before the next decode");
        sharded.push_back((int)i);
      } else {
        full.push_back((int)i);
      }
    }
    cudaStream_t s = c.stream;
    const int nf = (int)full.size();
    const int chunks = std::max(1, std::min(32, 256 / std::max(1, nf)));
    if (nf > 0) {
      if (c.sel_rows < nf) {
        const int rows = std::max(nf, 64);
        c.sel_tab = reinterpret_cast<int32_t**>(c.dalloc((size_t)rows * 8));
        c.sel_part = c.dalloc_n<int32_t>((size_t)rows * 32 * 2);
        c.sel_tok = c.dalloc_n<uint32_t>((size_t)rows);
        c.sel_rows = rows;
      }
      std::vector<int32_t*> tab(nf);
      for (int j = 0; j < nf; ++j) tab[j] = seqs[full[j]]->s->logits;
      CK(cudaMemcpyAsync(c.sel_tab, tab.data(), (size_t)nf * 8, cudaMemcpyHostToDevice, s));
      launch_argmax_rows(c.sel_tab, nullptr, nf, c.cfg.V, 0, 0, chunks, c.sel_part, s);
      launch_argmax_rows_final(c.sel_part, 1, nf, chunks, c.sel_tok, s);
      CK(cudaGetLastError());
    }
    std::vector<uint32_t> ftok(nf), stok;
    if (nf > 0) CK(cudaMemcpyAsync(ftok.data(), c.sel_tok, (size_t)nf * 4, cudaMemcpyDeviceToHost, s));
    if (!sharded.empty()) {
      stok.resize(c.tp.sel_rows);
      CK(cudaMemcpyAsync(stok.data(), c.tp.tokens, stok.size() * 4, cudaMemcpyDeviceToHost, s));
    }
    CK(cudaStreamSynchronize(s));
    for (int j = 0; j < nf; ++j) tokens_out[full[j]] = ftok[j];
    for (int i : sharded) tokens_out[i] = stok[seqs[i]->s->sel_row];
  });
}

int32_t rdet_tp_shard_logits(rdet_ctx* ctx, int32_t on) {
  return guard([&] {
    REQUIRE(ctx, RDET_E_INVALID, "null argument");
    Ctx& c = *ctx->c;
    REQUIRE(c.tp.comm != nullptr, RDET_E_STATE, "rdet_tp_shard_logits needs rdet_tp_init first");
    c.tp.shard_logits = on != 0;
  });
}

int32_t rdet_decode_begin(rdet_ctx* ctx, rdet_seq* seq, uint32_t token) {
  return guard([&] {
    REQUIRE(ctx && seq, RDET_E_INVALID, "null argument");
    Ctx& c = *ctx->c;
    Seq& q = *seq->s;
    CK(cudaSetDevice(c.device));
    check_decode_ready(c, q);
    REQUIRE(c.decode_owner == nullptr || c.decode_owner == &q, RDET_E_STATE, "another decode is in flight on this context");
    check_token(c, token);
    CK(cudaMemcpyAsync(q.d_token, &token, 4, cudaMemcpyHostToDevice, c.stream));
    decode_embed(c, q, q.d_token);
    CK(cudaGetLastError());
    q.decode_next = 0;
    q.decode_cur = c.dw.x0;
    c.decode_owner = &q;
  });
}

int32_t rdet_decode_range(rdet_ctx* ctx, rdet_seq* seq, uint32_t layer_start, uint32_t layer_end) {
  return guard([&] {
    REQUIRE(ctx && seq, RDET_E_INVALID, "null argument");
    Ctx& c = *ctx->c;
    Seq& q = *seq->s;
    CK(cudaSetDevice(c.device));
    REQUIRE(c.decode_owner == &q, RDET_E_STATE, "decode.layer_range requires decode_begin on this sequence");
    REQUIRE((int)layer_start == q.decode_next, RDET_E_STATE, "decode.layer_range must continue at the next layer");
    REQUIRE(layer_end >= layer_start && (int)layer_end <= c.cfg.L, RDET_E_RANGE, "layer range out of bounds");
    for (uint32_t l = layer_start; l < layer_end; ++l) {
      q.decode_cur = const_cast<int32_t*>(decode_layer(c, q, (int)l, q.decode_cur));
      q.decode_next = (int)l + 1;
    }
    CK(cudaGetLastError());
    CK(cudaStreamSynchronize(c.stream));
  });
}

int32_t rdet_decode_finalize(rdet_ctx* ctx, rdet_seq* seq) {
  return guard([&] {
    REQUIRE(ctx && seq, RDET_E_INVALID, "null argument");
    Ctx& c = *ctx->c;
    Seq& q = *seq->s;
    CK(cudaSetDevice(c.device));
    REQUIRE(c.decode_owner == &q && q.decode_next == c.cfg.L, RDET_E_STATE,
            "decode.transition_finalize requires all layers");
    decode_finalize_launch(c, q, q.decode_cur);
    CK(cudaGetLastError());
    CK(cudaStreamSynchronize(c.stream));
    check_err_flag(c, "decode");
    q.logits_sharded = false;
    q.pos += 1;
    q.last_was_prefill = false;
    q.decode_next = -1;
    c.decode_owner = nullptr;
  });
}

int32_t rdet_decode(rdet_ctx* ctx, rdet_seq* const* seqs, const uint32_t* tokens, size_t nseq) {
  return guard([&] {
    REQUIRE(ctx && (nseq == 0 || (seqs && tokens)), RDET_E_INVALID, "null argument");
    Ctx& c = *ctx->c;
    CK(cudaSetDevice(c.device));
    REQUIRE(c.decode_owner == nullptr, RDET_E_STATE, "a routine-granular decode is in flight on this context");
    for (size_t i = 0; i < nseq; ++i) {
      REQUIRE(seqs[i] && seqs[i]->owner == ctx, RDET_E_INVALID, "sequence belongs to another context");
      check_decode_ready(c, *seqs[i]->s);
      check_token(c, tokens[i]);
    }
    std::vector<Seq*> batch(nseq);
    for (size_t i = 0; i < nseq; ++i) {
      batch[i] = seqs[i]->s.get();
      batch[i]->logits_sharded = false;  // every path below but the sharded one writes the logits
    }
    if (batch_supported(c, batch.data(), (int)nseq)) {
      if (c.tp.comm && c.tp.shard_logits) {
        tp_select_buffers(c, (int)nseq);
        c.tp.epoch += 1;
      }
      // chunks of at most max_prefill rows (the row workspaces' size)
      for (size_t i0 = 0; i0 < nseq; i0 += c.max_prefill) {
        const int B = (int)std::min<size_t>(c.max_prefill, nseq - i0);
        if (B >= 2) {
          if (c.tp.comm) decode_batch_tp(c, batch.data() + i0, tokens + i0, B, (int)i0);
          else decode_batch(c, batch.data() + i0, tokens + i0, B);
          continue;
        }
        Seq& q = *batch[i0];
        ensure_decode_graph(c, q);
        CK(cudaMemcpyAsync(q.d_token, tokens + i0, 4, cudaMemcpyHostToDevice, c.stream));
        CK(cudaGraphLaunch(q.graph, c.stream));
        q.pos += 1;
        q.last_was_prefill = false;
      }
    } else {
      for (size_t i = 0; i < nseq; ++i) {
        Seq& q = *batch[i];
        ensure_decode_graph(c, q);
        CK(cudaMemcpyAsync(q.d_token, tokens + i, 4, cudaMemcpyHostToDevice, c.stream));
        CK(cudaGraphLaunch(q.graph, c.stream));
        q.pos += 1;
        q.last_was_prefill = false;
      }
    }
    CK(cudaStreamSynchronize(c.stream));
    check_err_flag(c, "decode");
  });
}

int32_t rdet_generate(rdet_ctx* ctx, rdet_seq* seq, uint32_t n_tokens, uint32_t* tokens_out) {
  return guard([&] {
    REQUIRE(ctx && seq && (tokens_out || n_tokens == 0), RDET_E_INVALID, "null argument");
    Ctx& c = *ctx->c;
    Seq& q = *seq->s;
    CK(cudaSetDevice(c.device));
    check_decode_ready(c, q);
    REQUIRE(c.decode_owner == nullptr, RDET_E_STATE, "a routine-granular decode is in flight on this context");
    REQUIRE(q.pos + (int)n_tokens <= q.cap, RDET_E_RANGE, "generation would overflow the sequence KV cache");
    require_logits(q);
    ensure_decode_graph(c, q);
    if (q.hist_cap < (int)n_tokens) {
      q.d_hist = static_cast<uint32_t*>(q.dalloc((size_t)std::max<uint32_t>(n_tokens, 1) * 4));
      q.hist_cap = (int)n_tokens;
    }
    for (uint32_t i = 0; i < n_tokens; ++i) {
      select_launch(c, q);
      CK(cudaMemcpyAsync(q.d_hist + i, q.d_token, 4, cudaMemcpyDeviceToDevice, c.stream));
      CK(cudaGraphLaunch(q.graph, c.stream));
    }
    if (n_tokens) CK(cudaMemcpyAsync(tokens_out, q.d_hist, (size_t)n_tokens * 4, cudaMemcpyDeviceToHost, c.stream));
    CK(cudaStreamSynchronize(c.stream));
    check_err_flag(c, "generate");
    q.pos += (int)n_tokens;
    q.last_was_prefill = false;
  });
}

int32_t rdet_get_stream(rdet_ctx* ctx, void** stream) {
  return guard([&] {
    REQUIRE(ctx && stream, RDET_E_INVALID, "null argument");
    *stream = ctx->c->stream;
  });
}

int32_t rdet_seq_kernels_per_step(rdet_seq* seq, uint32_t* kernels) {
  return guard([&] {
    REQUIRE(seq && kernels, RDET_E_INVALID, "null argument");
    Seq& q = *seq->s;
    REQUIRE(q.graph, RDET_E_STATE, "no decode graph captured yet");
    *kernels = (uint32_t)q.graph_kernels;
  });
}

int32_t rdet_read(rdet_ctx* ctx, rdet_seq* seq, int32_t which, int32_t layer, int32_t arg, void* dst, size_t bytes,
                  size_t* size_out) {
  return guard([&] {
    REQUIRE(ctx && seq, RDET_E_INVALID, "null argument");
    Ctx& c = *ctx->c;
    Seq& q = *seq->s;
    CK(cudaSetDevice(c.device));
    const int H = c.cfg.H;
    std::vector<int32_t> v;
    switch (which) {
      case RDET_BUF_EMBEDDING:
        REQUIRE(q.embd && q.last_S > 0, RDET_E_STATE, "no prefill embedding available");
        v = d2h(c, q.embd, (size_t)q.last_S * H);
        break;
      case RDET_BUF_HIDDEN:
        if (q.last_was_prefill) {
          REQUIRE(q.hid && q.last_S > 0, RDET_E_STATE, "no hidden states available");
          v = d2h(c, q.hid, (size_t)q.last_S * H);
        } else {
          v = d2h(c, q.dec_out + (size_t)(c.cfg.L - 1) * H, H);
        }
        break;
      case RDET_BUF_LOGITS:
        require_logits(q);
        v = d2h(c, q.logits, c.cfg.V);
        break;
      case RDET_BUF_LAYER_OUTPUT:
        REQUIRE(layer >= 0 && layer < c.cfg.L, RDET_E_RANGE, "layer out of range");
        REQUIRE(!q.last_was_prefill, RDET_E_STATE, "prefill layer outputs are available as commitments only");
        v = d2h(c, q.dec_out + (size_t)layer * H, H);
        break;
      case RDET_BUF_KV_K:
      case RDET_BUF_KV_V:
        REQUIRE(layer >= 0 && layer < c.cfg.L, RDET_E_RANGE, "layer out of range");
        REQUIRE(q.kc[layer], RDET_E_STATE, "layer shares the KV cache of an earlier layer");
        REQUIRE(arg >= 0 && arg < c.cfg.layers[layer].kv_heads, RDET_E_RANGE, "kv head out of range");
        v = kv_read(c, q, layer, arg, which == RDET_BUF_KV_K);
        break;
      default:
        throw Fail{RDET_E_INVALID, "unknown buffer"};
    }
    if (size_out) *size_out = v.size() * 4;
    if (dst) memcpy(dst, v.data(), std::min(bytes, v.size() * 4));
  });
}

int32_t rdet_commitment(rdet_ctx* ctx, rdet_seq* seq, int32_t which, int32_t layer, char* hex_out) {
  int32_t none = 0;
  int32_t rc = guard([&] {
    REQUIRE(ctx && seq && hex_out, RDET_E_INVALID, "null argument");
    Ctx& c = *ctx->c;
    Seq& q = *seq->s;
    CK(cudaSetDevice(c.device));
    const int H = c.cfg.H;
    std::string hx;
    switch (which) {
      case RDET_BUF_EMBEDDING: {
        REQUIRE(q.embd && q.last_S > 0, RDET_E_STATE, "no prefill embedding available");
        auto v = d2h(c, q.embd, (size_t)q.last_S * H);
        hx = act_hash_rows(v.data(), q.last_S, H);
        break;
      }
      case RDET_BUF_HIDDEN: {
        if (q.last_was_prefill) {
          REQUIRE(q.hid && q.last_S > 0, RDET_E_STATE, "no hidden states available");
          auto v = d2h(c, q.hid, (size_t)q.last_S * H);
          hx = act_hash_rows(v.data(), q.last_S, H);
        } else {
          auto v = d2h(c, q.dec_out + (size_t)(c.cfg.L - 1) * H, H);
          hx = act_hash_rows(v.data(), 1, H);
        }
        break;
      }
      case RDET_BUF_LOGITS: {
        require_logits(q);
        auto v = d2h(c, q.logits, c.cfg.V);
        Sha256 h;
        h.put("raster-det-num-act-vector-v1", 28);
        h.put_u64(v.size());
        h.put(v.data(), v.size() * 4);
        hx = h.hex();
        break;
      }
      case RDET_BUF_LAYER_OUTPUT: {
        REQUIRE(layer >= 0 && layer < c.cfg.L, RDET_E_RANGE, "layer out of range");
        if (q.last_was_prefill) {
          REQUIRE(!q.layer_hashes.empty() && !q.layer_hashes[layer].empty(), RDET_E_STATE,
                  "per-layer prefill commitments need RDET_FLAG_LAYER_COMMITMENTS");
          hx = q.layer_hashes[layer];
        } else {
          auto v = d2h(c, q.dec_out + (size_t)layer * H, H);
          hx = act_hash_rows(v.data(), 1, H);
        }
        break;
      }
      case RDET_BUF_KV:
        REQUIRE(layer >= 0 && layer <= c.cfg.L, RDET_E_RANGE, "KV layer count out of range");
        if (!kv_commitment(c, q, &hx, layer > 0 ? layer : c.cfg.L)) { none = 1; return; }
        break;
      default:
        throw Fail{RDET_E_INVALID, "unknown buffer"};
    }
    memcpy(hex_out, hx.c_str(), 65);
  });
  if (rc == RDET_OK && none) { hex_out[0] = 0; return RDET_NONE; }
  return rc;
}

int32_t rdet_kv_prefix_commitments(rdet_ctx* ctx, rdet_seq* seq, uint32_t n, char* hex_out) {
  return guard([&] {
    REQUIRE(ctx && seq && (hex_out || n == 0), RDET_E_INVALID, "null argument");
    Ctx& c = *ctx->c;
    Seq& q = *seq->s;
    CK(cudaSetDevice(c.device));
    REQUIRE(n <= (uint32_t)c.cfg.L, RDET_E_RANGE, "more prefixes than layers");
    std::vector<std::string> hx;
    kv_prefix_commitments(c, q, (int)n, &hx);
    for (uint32_t p = 0; p < n; ++p) {
      if (hx[p].empty()) hex_out[65 * (size_t)p] = 0;
      else memcpy(hex_out + 65 * (size_t)p, hx[p].c_str(), 65);
    }
  });
}

int32_t rdet_nccl_unique_id(void* id_out, size_t len) {
  return guard([&] {
    REQUIRE(id_out && len >= sizeof(ncclUniqueId), RDET_E_INVALID, "the id buffer needs 128 bytes");
    REQUIRE(nccl_api().ok, RDET_E_STATE, "libnccl.so.2 could not be loaded");
    ncclUniqueId id;
    NCK(nccl_api().getUniqueId(&id));
    memcpy(id_out, &id, sizeof(id));
  });
}

int32_t rdet_tp_init(rdet_ctx* ctx, int32_t rank, int32_t world, const void* id, size_t len) {
  return guard([&] {
    REQUIRE(ctx && id && len >= sizeof(ncclUniqueId), RDET_E_INVALID, "null argument or short id");
    Ctx& c = *ctx->c;
    CK(cudaSetDevice(c.device));
    ncclUniqueId uid;
    memcpy(&uid, id, sizeof(uid));
    tp_init(c, rank, world, uid);
  });
}

// IPC handles of recv and flags, then the row count of recv's slots as a u64.
constexpr size_t kTpIpcBlob = 2 * sizeof(cudaIpcMemHandle_t) + 8;

int32_t rdet_tp_ipc_export(rdet_ctx* ctx, uint32_t max_batch, void* out, size_t cap, size_t* len) {
  return guard([&] {
    REQUIRE(ctx && out && len, RDET_E_INVALID, "null argument");
    Ctx& c = *ctx->c;
    TpState& t = c.tp;
    REQUIRE(t.comm != nullptr, RDET_E_STATE, "rdet_tp_ipc_export needs rdet_tp_init first");
    REQUIRE(t.recv == nullptr, RDET_E_STATE, "the NVLink reduction buffers are already exported");
    REQUIRE(max_batch >= 1 && max_batch <= 65536, RDET_E_INVALID, "max_batch must be in [1, 65536]");
    REQUIRE(t.world <= 8, RDET_E_INVALID, "the NVLink reduction supports at most 8 ranks");
    REQUIRE(cap >= kTpIpcBlob, RDET_E_INVALID, "the export buffer needs " + std::to_string(kTpIpcBlob) + " bytes");
    CK(cudaSetDevice(c.device));
    t.p2p_rows = (int)max_batch;
    t.recv = c.dalloc_n<int64_t>((size_t)t.world * 2 * t.p2p_rows * c.cfg.H);
    t.flags = c.dalloc_n<uint32_t>(32);
    CK(cudaMemset(t.flags, 0, 32 * sizeof(uint32_t)));
    cudaIpcMemHandle_t h[2];
    CK(cudaIpcGetMemHandle(&h[0], t.recv));
    CK(cudaIpcGetMemHandle(&h[1], t.flags));
    const uint64_t rows = (uint64_t)t.p2p_rows;
    memcpy(out, h, sizeof(h));
    memcpy(static_cast<unsigned char*>(out) + sizeof(h), &rows, 8);
    *len = kTpIpcBlob;
  });
}

int32_t rdet_tp_ipc_connect(rdet_ctx* ctx, const void* blobs, size_t len_each, int32_t world) {
  return guard([&] {
    REQUIRE(ctx && blobs, RDET_E_INVALID, "null argument");
    Ctx& c = *ctx->c;
    TpState& t = c.tp;
    REQUIRE(t.recv != nullptr, RDET_E_STATE, "rdet_tp_ipc_connect needs rdet_tp_ipc_export first");
    REQUIRE(!t.p2p, RDET_E_STATE, "the NVLink reduction is already connected");
    REQUIRE(world == t.world && len_each == kTpIpcBlob, RDET_E_INVALID, "one export blob per rank, in rank order");
    CK(cudaSetDevice(c.device));
    // every rank's buffers hold the sums of the same rows: same batch limit
    CK(cudaDeviceSynchronize());
    const unsigned char* b = static_cast<const unsigned char*>(blobs);
    for (int r = 0; r < world; ++r) {
      if (r == t.rank) continue;
      cudaIpcMemHandle_t h[2];
      uint64_t rows = 0;
      memcpy(h, b + (size_t)r * kTpIpcBlob, sizeof(h));
      memcpy(&rows, b + (size_t)r * kTpIpcBlob + sizeof(h), 8);
      REQUIRE(rows == (uint64_t)t.p2p_rows, RDET_E_INVALID, "every rank must export the same max_batch");
      void* p[2] = {nullptr, nullptr};
      for (int i = 0; i < 2; ++i) {
        CK(cudaIpcOpenMemHandle(&p[i], h[i], cudaIpcMemLazyEnablePeerAccess));
        t.ipc_opened.push_back(p[i]);
      }
      t.peer_recv[r] = static_cast<int64_t*>(p[0]);
      t.peer_flags.f[r] = static_cast<uint32_t*>(p[1]);
    }
    t.p2p = true;
  });
}

int32_t rdet_tp_world(rdet_ctx* ctx) {
  if (!ctx || !ctx->c) return 0;
  return ctx->c->tp.comm ? ctx->c->tp.world : 1;
}

int32_t rdet_tensor_core_prefill(rdet_ctx* ctx) {
  if (!ctx || !ctx->c) return 0;
  return ctx->c->tc ? 1 : 0;
}

int32_t rdet_det_gemv(const int32_t* x, const void* w, int32_t width, uint32_t rows, uint32_t cols, int32_t* y,
                      void* stream) {
  return guard([&] {
    kernels_init();
    REQUIRE(x && w && y, RDET_E_INVALID, "null argument");
    REQUIRE(width == 16 || width == 32, RDET_E_INVALID, "width must be 16 or 32");
    REQUIRE(rows > 0 && cols > 0 && cols <= 49152, RDET_E_RANGE, "unsupported GEMV shape");
    REQUIRE(((uintptr_t)w & 15) == 0 && ((uintptr_t)x & 15) == 0, RDET_E_INVALID,
            "weights and input must be 16-byte aligned");
    GemvArgs g;
    g.K = (int)cols;
    g.seg[0].w.p = w;
    g.seg[0].w.width = width;
    g.seg[0].w.rows = (int)rows;
    g.seg[0].w.cols = (int)cols;
    g.seg[0].y = y;
    g.a = x;
    launch_gemv(g, static_cast<cudaStream_t>(stream));
    CK(cudaGetLastError());
  });
}

int32_t rdet_det_attention_decode(const int32_t* q, const int32_t* k_cache, const int32_t* v_cache,
                                             uint32_t cap, uint32_t num_heads, uint32_t num_kv_heads,
                                             uint32_t head_dim, uint32_t position, uint32_t window, int32_t* out,
                                             void* stream) {
  return guard([&] {
    kernels_init();
    AttnDecodeArgs a;
    attn_entry_args(a, q, k_cache, v_cache, cap, num_heads, num_kv_heads, head_dim, position, window, out);
    int dev = 0;
    CK(cudaGetDevice(&dev));
    int rows = attn_rows(position, window);
    std::lock_guard<std::mutex> lk(g_attn_scratch_mu);
    AttnScratchOwned& o = g_attn_scratch[dev];
    if (o.heads < (int)num_heads || o.rows < rows || o.dim < (int)head_dim) {
      if (!o.ptrs.empty()) CK(cudaDeviceSynchronize());  // earlier launches may still read the old scratch
      for (void* p : o.ptrs) CK(cudaFree(p));
      o = AttnScratchOwned();
      o.heads = std::max<int>(num_heads, 8);
      o.rows = std::max(rows, 1024);
      o.dim = std::max<int>(head_dim, 256);
      o.splits = (o.rows + a.rows_per_split - 1) / a.rows_per_split;
      auto al = [&](size_t bytes) {
        void* p = nullptr;
        CK(cudaMalloc(&p, bytes));
        o.ptrs.push_back(p);
        return p;
      };
      o.sc.scores = static_cast<int32_t*>(al((size_t)o.heads * o.rows * 4));
      o.sc.exps = static_cast<int64_t*>(al((size_t)o.heads * o.rows * 8));
      o.sc.pmax = static_cast<int32_t*>(al((size_t)o.heads * o.splits * 4));
      o.sc.pidx = static_cast<int32_t*>(al((size_t)o.heads * o.splits * 4));
      o.sc.psum = static_cast<int64_t*>(al((size_t)o.heads * o.splits * 8));
      o.sc.pwsum = static_cast<int64_t*>(al((size_t)o.heads * o.splits * 8));
      o.sc.pacc = static_cast<int64_t*>(al((size_t)o.heads * o.splits * o.dim * 8));
      o.sc.max_splits = o.splits;
      o.sc.stride = o.rows;
    }
    a.sc = o.sc;
    launch_attn_decode_cluster(a, static_cast<cudaStream_t>(stream));
    CK(cudaGetLastError());
  });
}

// Same computation as rdet_det_attention_decode with no device allocation:
// the scratch is the library's fixed array (see noalloc_scratch_current_device).
// Every scratch value is written before it is read, so nothing is cleared.
int32_t rdet_det_attention_decode_noalloc(const int32_t* q, const int32_t* k_cache, const int32_t* v_cache,
                                          uint32_t cap, uint32_t num_heads, uint32_t num_kv_heads,
                                          uint32_t head_dim, uint32_t position, uint32_t window, int32_t* out,
                                          void* stream) {
  return guard([&] {
    kernels_init();
    AttnDecodeArgs a;
    attn_entry_args(a, q, k_cache, v_cache, cap, num_heads, num_kv_heads, head_dim, position, window, out);
    const int rows = attn_rows(position, window);
    REQUIRE(num_heads <= (uint32_t)kNoAllocMaxHeads, RDET_E_RANGE,
            "rdet_det_attention_decode_noalloc supports at most 16 query heads");
    REQUIRE(head_dim <= (uint32_t)kNoAllocMaxHeadDim, RDET_E_RANGE,
            "rdet_det_attention_decode_noalloc supports head_dim <= 512");
    REQUIRE(rows <= kNoAllocMaxRows, RDET_E_RANGE,
            "rdet_det_attention_decode_noalloc attends at most 4096 rows (min(position + 1, window))");
    unsigned char* base = noalloc_scratch_current_device();
    a.rows_per_split = kNoAllocRowsPerSplit;
    a.sc.scores = reinterpret_cast<int32_t*>(base + kNaScores);
    a.sc.exps = reinterpret_cast<int64_t*>(base + kNaExps);
    a.sc.pmax = reinterpret_cast<int32_t*>(base + kNaPmax);
    a.sc.pidx = reinterpret_cast<int32_t*>(base + kNaPidx);
    a.sc.psum = reinterpret_cast<int64_t*>(base + kNaPsum);
    a.sc.pwsum = reinterpret_cast<int64_t*>(base + kNaPwsum);
    a.sc.pacc = reinterpret_cast<int64_t*>(base + kNaPacc);
    a.sc.max_splits = (rows + kNoAllocRowsPerSplit - 1) / kNoAllocRowsPerSplit;
    a.sc.stride = kNoAllocMaxRows;
    launch_attn_decode(a, static_cast<cudaStream_t>(stream));
    CK(cudaGetLastError());
  });
}

int32_t rdet_det_attention_prefill(const int32_t* q, const int32_t* k_cache, const int32_t* v_cache, uint32_t cap,
                                   uint32_t n_tokens, uint32_t num_heads, uint32_t num_kv_heads, uint32_t head_dim,
                                   uint32_t window, uint32_t flags, int32_t* out, void* stream) {
  return guard([&] {
    kernels_init();
    REQUIRE(q && k_cache && v_cache && out, RDET_E_INVALID, "null argument");
    REQUIRE(n_tokens > 0 && n_tokens <= cap, RDET_E_RANGE, "n_tokens must be in [1, cap]");
    REQUIRE(num_kv_heads > 0 && num_heads % num_kv_heads == 0, RDET_E_INVALID,
            "num_heads must be a multiple of num_kv_heads");
    REQUIRE(head_dim > 0 && head_dim <= 512 && head_dim % 4 == 0, RDET_E_RANGE,
            "head_dim must be a multiple of 4, at most 512");
    REQUIRE((((uintptr_t)q | (uintptr_t)k_cache | (uintptr_t)v_cache | (uintptr_t)out) & 15) == 0, RDET_E_INVALID,
            "q, caches and out must be 16-byte aligned");
    AttnPrefillArgs a;
    a.S = (int)n_tokens;
    a.Hq = (int)num_heads;
    a.Hkv = (int)num_kv_heads;
    a.d = (int)head_dim;
    a.window = (int)window;
    a.q = q;
    a.k_cache = k_cache;
    a.v_cache = v_cache;
    a.cap = (int)cap;
    a.out = out;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const bool tc = !(flags & RDET_FLAG_NO_TENSOR_CORES) &&
                    tc_attn_eligible(a.S, a.Hq, a.Hkv, a.d);
    const int rowlen = a.window > 0 ? std::min(a.window, a.S) : a.S;
    const size_t cuda_elems = (size_t)a.Hq * a.S * rowlen;
    const size_t need = tc ? tc_attn_ws_bytes(a.S, a.Hq, a.Hkv, a.d) : cuda_elems * 12 + 256;
    int dev = 0;
    CK(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lk(g_pattn_scratch_mu);
    LinScratch& sc = g_pattn_scratch[dev];
    if (sc.bytes < need) {
      if (sc.p) {
        CK(cudaDeviceSynchronize());  // earlier launches may still read the old scratch
        CK(cudaFree(sc.p));
        sc.p = nullptr;
        sc.bytes = 0;
      }
      CK(cudaMalloc(&sc.p, need));
      sc.bytes = need;
    }
    if (tc) {
      REQUIRE(launch_attn_prefill_tc(a, sc.p, sc.bytes, s), RDET_E_CUDA, "tensor-core attention launch failed");
    } else {
      a.scores = static_cast<int32_t*>(sc.p);
      a.exps = reinterpret_cast<int64_t*>(static_cast<unsigned char*>(sc.p) + ((cuda_elems * 4 + 255) & ~(size_t)255));
      a.scratch_elems = (int64_t)cuda_elems;
      launch_attn_prefill(a, s);
    }
    CK(cudaGetLastError());
  });
}

int32_t rdet_convert_to_wgt(const void* src, int32_t dtype, uint64_t rows, uint64_t row_len, int32_t* out,
                            uint64_t* row_mass, uint32_t* stats, void* stream) {
  return guard([&] {
    kernels_init();
    REQUIRE(dtype == kSrcF32 || dtype == kSrcBF16 || dtype == kSrcF16, RDET_E_INVALID,
            "dtype must be RDET_SRC_F32, RDET_SRC_BF16 or RDET_SRC_F16");
    REQUIRE(rows == 0 || (src && out && row_mass && stats), RDET_E_INVALID, "null argument");
    REQUIRE(rows == 0 || row_len > 0, RDET_E_RANGE, "row_len must be positive");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (stats) CK(cudaMemsetAsync(stats, 0, 2 * sizeof(uint32_t), s));
    launch_convert_wgt(src, dtype, rows, row_len, out, row_mass, stats, s);
    CK(cudaGetLastError());
  });
}

int32_t rdet_det_linear(const int32_t* x, uint32_t n_rows_x, const void* w, int32_t width, uint32_t rows,
                        uint32_t cols, int32_t* y, void* stream) {
  return guard([&] {
    kernels_init();
    REQUIRE(x && w && y, RDET_E_INVALID, "null argument");
    REQUIRE(width == 16 || width == 32, RDET_E_INVALID, "width must be 16 or 32");
    REQUIRE(rows > 0 && cols > 0 && n_rows_x > 0, RDET_E_RANGE, "unsupported linear shape");
    DevMat m;
    m.p = w;
    m.width = width;
    m.rows = (int)rows;
    m.cols = (int)cols;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if ((int)n_rows_x >= kTcMinRows && tc_weight_eligible(m) && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
        tc_supported()) {
      // byte planes of w and x in the per-device scratch, then the tensor-core GEMM
      int dev = 0;
      CK(cudaGetDevice(&dev));
      const size_t wb = (tc_weight_bytes((int)rows, (int)cols, false) + 255) & ~(size_t)255;
      const size_t ab = (tc_act_bytes((int)n_rows_x, (int)cols) + 255) & ~(size_t)255;
      const size_t need = wb + ab + kTcSplitScratch;
      std::lock_guard<std::mutex> lk(g_lin_scratch_mu);
      LinScratch& sc = g_lin_scratch[dev];
      if (sc.bytes < need) {
        if (sc.p) {
          CK(cudaDeviceSynchronize());
          CK(cudaFree(sc.p));
          sc.p = nullptr;
          sc.bytes = 0;
        }
        CK(cudaMalloc(&sc.p, need));
        sc.bytes = need;
      }
      TcWeight tw;
      TcAct ta;
      unsigned char* base = static_cast<unsigned char*>(sc.p);
      REQUIRE(tc_prepare_weight(tw, m, nullptr, base, s), RDET_E_CUDA, "tensor map encoding failed");
      REQUIRE(tc_prepare_act(ta, x, (int)n_rows_x, (int)cols, base + wb, s), RDET_E_CUDA,
              "tensor map encoding failed");
      TcOut o;
      o.y = y;
      o.scratch = base + wb + ab;
      o.scratch_bytes = kTcSplitScratch;
      launch_tc_linear(ta, tw, o, s);
    } else {
      launch_linear(x, (int)n_rows_x, m, y, kEpiPlain, nullptr, s);
    }
    CK(cudaGetLastError());
  });
}

}  // extern "C"
