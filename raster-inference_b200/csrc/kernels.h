// Launch interface of the det kernels (sm_100a).  Host code in runtime.cu
// composes these into the prefill / decode / select routines.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

namespace rdet {

enum WeightWidth : int32_t { kW16 = 16, kW32 = 32 };

// A weight matrix resident in HBM: row-major [rows, cols], i16 or i32.
struct DevMat {
  const void* p = nullptr;
  int32_t width = 16;
  int32_t rows = 0, cols = 0;
};

// ---- decode GEMV -----------------------------------------------------------
// Epilogues applied to requantize(dot) of output row r.
enum GemvEpi : int32_t {
  kEpiPlain = 0,      // y[r] = v
  kEpiSoftcap = 1,    // y[r] = softcap(v, cap)
  kEpiGeluMul = 2,    // y[r] = mul_sat(gelu(v), vec[r])
};
// Prologues that build the input vector x (length K) in shared memory.
enum GemvPro : int32_t {
  kProNone = 0,       // x = a
  kProNorm = 1,       // x = rmsnorm(a, g1)
  kProResNorm = 2,    // t = add_sat(res, rmsnorm(a, g1)); x = rmsnorm(t, g2); block 0 stores t
  kProResScale = 3,   // t = scale?(add_sat(res, rmsnorm(a, g1))); x = t; block 0 stores t
  kProResScaleNorm = 4,  // t as kProResScale; x = rmsnorm(t, g2); block 0 stores t
};
struct GemvSeg {
  DevMat w;
  int32_t* y = nullptr;
  int32_t epi = kEpiPlain;
  const int32_t* vec = nullptr;
};
struct GemvArgs {
  int32_t K = 0;
  int32_t nseg = 1;
  GemvSeg seg[3];
  bool pair_geglu = false;  // seg[0]=gate, seg[1]=up: seg[0].y[r] = mul_sat(gelu(g), u)
  int32_t softcap = 0;
  // prologue.  g1/g2 are model constants: the kernel reads them before
  // waiting on the preceding grid, so no earlier kernel in the stream may
  // write them.
  int32_t pro = kProNone;
  const int32_t* a = nullptr;
  const int32_t* res = nullptr;
  const int32_t* g1 = nullptr;
  const int32_t* g2 = nullptr;
  int64_t eps = 0;
  int32_t scalar = 0;
  bool has_scalar = false;
  int32_t* t_out = nullptr;
};
void launch_gemv(const GemvArgs& a, cudaStream_t s);

// ---- prefill linear (Y[S,N] = requantize(X[S,K] W^T)) -------------------------
void launch_linear(const int32_t* X, int32_t S, const DevMat& w, int32_t* Y, int32_t epi, const int32_t* vec,
                   cudaStream_t s);
// geglu pair: Y = mul_sat(gelu(X Wg^T), X Wu^T)
void launch_linear_geglu(const int32_t* X, int32_t S, const DevMat& wg, const DevMat& wu, int32_t* Y,
                         cudaStream_t s);

// ---- prefill linear on tcgen05 int8 tensor cores (tc_gemm.cu) ------------------
// Exact: X + 2^31 and W + 2^15 split into unsigned byte planes, byte products
// on the tensor cores, recombined with row-sum corrections in wrapping i64.
// Bit-exact with launch_linear / launch_linear_geglu for i16 weights with
// K a multiple of 16 and K <= kTcMaxK.
constexpr int kTcMaxK = 32768;
struct TcWeight {           // byte planes of one weight matrix (or a gate/up pair)
  alignas(64) unsigned char map[128];  // TMA tensor map of the planes (96-row boxes)
  alignas(64) unsigned char map_m[128];  // the same planes in 128-row boxes (short-row-count kernel)
  uint8_t* planes = nullptr;           // [2][nrows][K]
  uint64_t* rowsum = nullptr;          // [nrows] sum over k of W + 2^15
  int32_t N = 0, K = 0, nrows = 0;
  bool pair = false;                   // rows interleave gate and up in blocks of 48
};
struct TcAct {              // byte planes of one activation matrix
  alignas(64) unsigned char map[128];    // 128-row boxes
  alignas(64) unsigned char map_t[128];  // 64-row boxes (S <= 64: short-row-count kernel)
  uint8_t* planes = nullptr;           // [4][S][K] byte limbs of X + 2^e (e per row: 23 or 31)
  uint64_t* rowsum = nullptr;          // [S] sum over k of X + 2^e; top bit set when e = 23
  uint32_t* tile4 = nullptr;           // [S / 256] 1 when a 256-row tile has a row with e = 31 (or null)
  int32_t S = 0, K = 0;
};
bool tc_supported();                         // current device is sm_100
bool tc_weight_eligible(const DevMat& w);
size_t tc_weight_bytes(int rows, int K, bool pair);
// Builds the planes of g (and u, for the gate/up pair) into `mem`
// (tc_weight_bytes); returns false if the tensor map cannot be encoded.
bool tc_prepare_weight(TcWeight& t, const DevMat& g, const DevMat* u, void* mem, cudaStream_t s);
// Same for the block rows [row0, row0 + rows) x columns [col0, col0 + cols) of
// g (and u); row0/rows select gate/up rows of a pair.  col0 and cols are
// multiples of 16.  Memory: tc_weight_bytes(rows, cols, pair).
bool tc_prepare_weight_slice(TcWeight& t, const DevMat& g, const DevMat* u, int row0, int rows, int col0, int cols,
                             void* mem, cudaStream_t s);
size_t tc_act_bytes(int S, int K);
// X [S, K] (16-byte aligned, K % 16 == 0) -> planes in `mem` (tc_act_bytes)
// Byte planes of n matrices with the same column count in one buffer
// ([2][sum of rows][K], then the row sums): views[i] covers matrix i alone,
// whole covers all rows in order (one GEMM producing [S][sum of rows]).
size_t tc_weight_group_bytes(const DevMat* mats, int n);
bool tc_prepare_weight_group(TcWeight* views, const DevMat* mats, int n, TcWeight& whole, void* mem, cudaStream_t s);
bool tc_prepare_act(TcAct& a, const int32_t* X, int S, int K, void* mem, cudaStream_t s);
// Attaches planes already written at `mem` (layout of tc_prepare_act: [4][S][K]
// bytes of X + 2^e, then S u64 row sums, then the tile flags) and encodes
// their tensor maps.  with_tile4: the producer zeroed and set the tile flags
// (tc_act_tile4(mem, S, K)); else every tile multiplies all four limbs.
bool tc_attach_act(TcAct& a, int S, int K, void* mem, bool with_tile4 = false);
// The tile flags of the activation layout at `mem`: one u32 per
// kTcFlagRows rows, nonzero when a row of that tile has offset 2^31.
uint32_t* tc_act_tile4(void* mem, int S, int K);
constexpr int kTcFlagRows = 256;
// Up to this many rows the linear takes its short-row kernel, which
// multiplies all four limbs and reads no tile flags.
constexpr int kTcShortRows = 64;
// Output of the tensor-core linear.  y: Y [S, N] = epilogue(requantize(X W^T))
// (a pair writes mul_sat(gelu(gate), up); kEpiGeluMul multiplies by
// vec[s * ldv + n]).  y64 instead: the exact wrapping i64 sums before
// requantize (needs scratch).  With scratch the K loop may be split across
// CTAs when the output tiles alone would leave SMs idle.
// Copies of the i64 sums written into other GPUs' memory (peer pointers of
// the tensor-parallel NVLink reduction), each [S, N] like y64.
struct TcMirrors {
  int64_t* p[7] = {};
  int32_t n = 0;
};
struct TcOut {
  int32_t* y = nullptr;
  int64_t* y64 = nullptr;
  TcMirrors y64_mirror;         // y64 is also stored to these (the split-K finish only)
  int32_t epi = 0;
  const int32_t* vec = nullptr;
  int32_t ldv = 0;              // 0: N
  void* scratch = nullptr;      // split-K partials, [splits][S][rows] u64
  size_t scratch_bytes = 0;
};
// false when y64 is asked for and the scratch cannot hold the partial sums
bool launch_tc_linear(const TcAct& a, const TcWeight& w, const TcOut& o, cudaStream_t s);
void tc_init();  // per-device kernel attributes (called by kernels_init)
int tc_error_flag(bool reset);  // nonzero when a tensor-core pipeline wait gave up

// ---- row ops -------------------------------------------------------------------
// y[s] = rmsnorm(x[s], g)   (g == nullptr: weightless value norm)
void launch_rmsnorm_rows(const int32_t* x, int32_t S, int32_t n, const int32_t* g, int64_t eps, int32_t* y,
                         cudaStream_t s);
// out[s] = scale?(add_sat(res[s], rmsnorm(a[s], g)))
void launch_norm_residual_rows(const int32_t* a, const int32_t* res, int32_t S, int32_t n, const int32_t* g,
                               int64_t eps, bool has_scalar, int32_t scalar, int32_t* out, cudaStream_t s);
// Fused per-row norms (one block per row, n % 4 == 0), covering the row
// kernels between the GEMMs of a batched decode step and of a prefill layer:
//   with res: t = res + norm(a) * g1 (then * scalar), stored to t_out (and
//             copied to scatter[r] + scatter_off when scatter is set);
//   with g2:  y = norm(t) * g2 stored to y_out;
//   without res: y = norm(a) * g1 stored to y_out;
//   planes:   the tensor-core activation planes and row sums (the layout of
//             tc_prepare_act) of y, or of t when res is set without g2.
struct RowNormArgs {
  const int32_t* a = nullptr;
  // instead of a: exact i64 sums (a tensor-parallel all-reduce's output),
  // requantized as they are loaded
  const int64_t* a64 = nullptr;
  // the tensor-parallel NVLink reduction: a64 plus the same rows of the
  // peers' sums (peer memory), read once flags[r] >= wait_seq for every rank
  // r in wait_mask (flags in this GPU's memory, written by the peers; the
  // wait is bounded and sets the pipeline error flag when it gives up)
  const int64_t* a64_peer[7] = {};
  int32_t npeer = 0;
  const uint32_t* flags = nullptr;
  uint32_t wait_mask = 0, wait_seq = 0;
  const int32_t* res = nullptr;
  const int32_t* g1 = nullptr;
  const int32_t* g2 = nullptr;
  int32_t n = 0;
  int64_t eps = 0;
  bool has_scalar = false;
  int32_t scalar = 0;
  int32_t* t_out = nullptr;
  int32_t* y_out = nullptr;
  int32_t* const* scatter = nullptr;
  size_t scatter_off = 0;
  // tensor-core operand of the output row y: byte planes of y + 2^e (e = 23
  // when the row fits 24 bits, flagged in the row sum's top bit, else 31;
  // the tensor-core linear's activation layout) and tile4[row / 256] set for
  // a row with e = 31 (tile4 zeroed by the caller; may be null)
  uint8_t* planes = nullptr;
  uint64_t* rowsum = nullptr;
  uint32_t* tile4 = nullptr;
};
void launch_row_norm(const RowNormArgs& a, int32_t rows, cudaStream_t s);

// ---- attention inputs -------------------------------------------------------------
struct QkvPostArgs {
  int32_t S = 1;              // rows (tokens)
  const int32_t* pos = nullptr;  // device: position of row 0
  int32_t Hq = 0, Hkv = 0, d = 0, rotary = 0;
  const int64_t* inv_freq = nullptr;  // [rotary/2] Q32.32 recurrence table
  // prefill: (cos, sin) of row s's position for every rotary pair, [S][rotary/2][2]
  // (launch_rope_table), or nullptr to compute them from inv_freq
  const int32_t* rope_cs = nullptr;
  const int32_t* q_in = nullptr;      // [S, Hq*d]
  const int32_t* k_in = nullptr;      // [S, Hkv*d] raw K (nullptr: no own KV)
  const int32_t* v_in = nullptr;      // [S, Hkv*d] raw V (== k_in for k_eq_v)
  int32_t ld = 0;                     // row stride of q_in / k_in / v_in in ints (0: Hq*d, Hkv*d)
  const int32_t* q_norm = nullptr;
  const int32_t* k_norm = nullptr;
  int64_t eps = 0;
  int32_t* q_out = nullptr;           // [S, Hq*d]
  int32_t* k_cache = nullptr;         // [Hkv, cap, d]
  int32_t* v_cache = nullptr;
  int32_t cap = 0;
  // batched decode: row s is its own sequence (position *pos_rows[s], caches
  // kc_rows[s] / vc_rows[s] of capacity cap_rows[s]); pos, k_cache, v_cache and
  // cap are then unused
  const int32_t* const* pos_rows = nullptr;
  int32_t* const* kc_rows = nullptr;
  int32_t* const* vc_rows = nullptr;
  const int32_t* cap_rows = nullptr;
};
void launch_qkv_post(const QkvPostArgs& a, cudaStream_t s);
// cs[p][i] = (cos, sin) of pos_angle(p, inv_freq[i]) for positions p in [0, S)
// and pairs i in [0, half): the RoPE factors of a prompt, once per distinct
// inverse-frequency table instead of once per (row, head, layer)
void launch_rope_table(const int64_t* inv_freq, int half, int S, int32_t* cs, cudaStream_t s);
// The same layout for batch rows at their own positions: row r at *pos_rows[r].
void launch_rope_rows(const int64_t* inv_freq, int half, int rows, const int32_t* const* pos_rows, int32_t* cs,
                      cudaStream_t s);

// ---- attention -----------------------------------------------------------------
struct AttnScratch {
  int32_t* scores = nullptr;  // [Hq, cap]
  int64_t* exps = nullptr;    // [Hq, cap]
  int32_t* pmax = nullptr;    // [Hq, nsplit]
  int32_t* pidx = nullptr;    // [Hq, nsplit]
  int64_t* psum = nullptr;    // [Hq, nsplit]
  int64_t* pwsum = nullptr;   // [Hq, nsplit]
  int64_t* pacc = nullptr;    // [Hq, nsplit, d]
  int32_t max_splits = 0;
  int32_t stride = 0;         // row stride of scores / exps (>= attended rows)
};
// Optional prologue of the cluster decode attention: q/k head RMSNorm, RoPE,
// value RMSNorm and the KV-cache append of the current token (the work of
// qkv_post), done inside the attention kernel.
struct AttnFuse {
  const int32_t* q_in = nullptr;   // raw q [Hq*d]; nullptr: a.q is already normed/rotated
  const int32_t* k_in = nullptr;   // raw k [Hkv*d]; nullptr: no own cache (KV-sharing layer)
  const int32_t* v_in = nullptr;   // raw v [Hkv*d] (== k_in for k_eq_v)
  const int32_t* q_norm = nullptr;
  const int32_t* k_norm = nullptr;
  int64_t eps = 0;
  int32_t rotary = 0;
  const int64_t* inv_freq = nullptr;
  int32_t* k_out = nullptr;        // own cache [Hkv, cap, d] written at row pos
  int32_t* v_out = nullptr;
};
struct AttnDecodeArgs {
  const int32_t* pos = nullptr;  // device: position of the current token
  int32_t pos_value = 0;         // used when pos == nullptr
  int32_t Hq = 0, Hkv = 0, d = 0;
  int32_t window = 0;            // 0 = full attention
  const int32_t* q = nullptr;    // [Hq, d]
  const int32_t* k_cache = nullptr;
  const int32_t* v_cache = nullptr;
  int32_t cap = 0;
  int32_t* out = nullptr;        // [Hq, d]
  AttnScratch sc;
  int32_t rows_per_split = 64;
  AttnFuse fuse;                 // used by the cluster kernel only
  // batched decode (cluster kernel, not fused): `batch` query rows, row b
  // attends with position *pos_rows[b] over kc_rows[b] / vc_rows[b] (capacity
  // cap_rows[b]); q and out hold [batch, Hq, d]; cap is the largest capacity
  int32_t batch = 1;
  // tensor-parallel shard: q / out hold Hq local heads, global index head0 + h;
  // group = query heads per KV head of the model (0: Hq / Hkv), caches keep
  // all Hkv KV heads
  int32_t head0 = 0, group = 0;
  const int32_t* const* pos_rows = nullptr;
  const int32_t* const* kc_rows = nullptr;
  const int32_t* const* vc_rows = nullptr;
  const int32_t* cap_rows = nullptr;
  // batched: the rows in launch order (longest context first, so that the
  // longest rows' clusters start in the first wave); null = row order
  const int32_t* row_order = nullptr;
  // batched, tensor-core attention: each row's tensor maps of its caches
  // ([layer][K, V], 128 bytes each; td_encode_cache_map) and the layer whose
  // caches this launch reads; null: the CUDA-core kernel runs
  const unsigned char* const* map_rows = nullptr;
  int32_t map_layer = 0;
};
void launch_attn_decode(const AttnDecodeArgs& a, cudaStream_t s);
// Same computation in one kernel: one thread-block cluster per query head
// splits the window across its CTAs and combines the exact softmax statistics
// through distributed shared memory (no global scratch).
void launch_attn_decode_cluster(const AttnDecodeArgs& a, cudaStream_t s);
// Batched decode attention on the tensor cores (tc_attn_dec.cu): false when
// the shape does not qualify (then the cluster kernel runs).
bool launch_attn_decode_tc(const AttnDecodeArgs& a, int sms, cudaStream_t s);
// The tensor map (128 bytes at out, 64-byte aligned) of one KV cache
// [rows][d] i32 that launch_attn_decode_tc reads: 32 x 64 boxes, 128-byte
// swizzle.  False when d is not a multiple of 128 or encoding fails.
bool td_encode_cache_map(void* out, const int32_t* base, int rows, int d);
int tc_attn_dec_error_flag(bool reset);
void tc_attn_dec_init();
// Whether launch_attn_decode_cluster runs the cluster kernel for this shape
// (rotary: the fused prologue's rotary width, 0 when not fused).  When it
// does not, it falls back to launch_attn_decode, which needs a.sc and does
// not fuse the prologue.
bool attn_decode_cluster_fits(int Hq, int Hkv, int d, int window, int cap, int rotary, int group = 0);

struct AttnPrefillArgs {
  int32_t S = 0;
  int32_t Hq = 0, Hkv = 0, d = 0;
  int32_t window = 0;            // 0 = full (causal)
  const int32_t* q = nullptr;    // [S, Hq*d]
  const int32_t* k_cache = nullptr;  // [Hkv, cap, d], rows 0..S-1
  const int32_t* v_cache = nullptr;
  int32_t cap = 0;
  int32_t* out = nullptr;        // [S, Hq*d]
  int32_t* scores = nullptr;     // scratch [Hq, S, S] (or window)
  int64_t* exps = nullptr;       // scratch same count
  int64_t scratch_elems = 0;
};
void launch_attn_prefill(const AttnPrefillArgs& a, cudaStream_t s);
// The same attention on the tcgen05 tensor cores (tc_attn.cu): exact byte-limb
// products for q k^T and for the weighted values, the exact softmax on the CUDA
// cores between them.  Eligible when head_dim is a multiple of 64, the query
// heads per KV head divide 128 and S <= 32768.  Workspace: tc_attn_ws_bytes
// (0 when not eligible).  Returns false, launching nothing, when the shape,
// alignment or workspace does not qualify.
size_t tc_attn_ws_bytes(int S, int Hq, int Hkv, int d);
bool tc_attn_eligible(int S, int Hq, int Hkv, int d);
bool launch_attn_prefill_tc(const AttnPrefillArgs& a, void* ws, size_t ws_bytes, cudaStream_t s);
void tc_attn_init();                 // per-device kernel attributes (called by kernels_init)
int tc_attn_error_flag(bool reset);  // nonzero when one of its pipeline waits gave up

// ---- embedding / PLE / logits ------------------------------------------------------
void launch_embed(const uint32_t* ids, int32_t S, const DevMat& emb, int32_t scale, int32_t* out, int32_t* err,
                  cudaStream_t s);
struct PleArgs {
  int32_t S = 0, L = 0, P = 0;
  const uint32_t* ids = nullptr;
  const int32_t* proj = nullptr;   // [S, L*P] = requantize(x0 Wproj^T)
  DevMat table;                    // [ple_vocab, L*P]
  const int32_t* norm = nullptr;   // [P]
  int64_t eps = 0;
  int32_t emb_scale = 0, proj_scale = 0, in_scale = 0;
  int32_t* out = nullptr;          // [L, S, P]
  int32_t* err = nullptr;
};
void launch_ple(const PleArgs& a, cudaStream_t s);

// argmax_first over n values; result index written to *idx (u32).  `part`
// holds at least 2*blocks ints of scratch.
void launch_argmax(const int32_t* x, int32_t n, int32_t* part, int32_t blocks, uint32_t* idx, cudaStream_t s);
// argmax_first of B rows: (value, idx0 + column) of each chunk's first max
// into part [B][chunks][2]; then each row's token from [world][B][chunks][2]
void launch_argmax_rows(const int32_t* const* rows, const int32_t* base, int32_t B, int32_t n, size_t ld,
                        int32_t idx0, int32_t chunks, int32_t* part, cudaStream_t s);
void launch_argmax_rows_final(const int32_t* part, int32_t world, int32_t B, int32_t chunks, uint32_t* tokens,
                              cudaStream_t s);
void launch_softcap(int32_t* x, int32_t n, int32_t cap, cudaStream_t s);

// ---- misc ---------------------------------------------------------------------------
void launch_add_i32(int32_t* p, int32_t v, cudaStream_t s);  // *p += v
void launch_add_i32_rows(int32_t* const* p, int32_t n, int32_t v, cudaStream_t s);  // *p[i] += v
void launch_requantize_rows(const int64_t* x, size_t n, int32_t* y, cudaStream_t s);  // y = requantize(x)
// Publishes reduction number `value` of rank `rank` to the other ranks:
// peer_flags[r][rank] = value (system-scope release) for r != rank, after the
// sums written by the preceding kernels.
struct TpPeerFlags {
  uint32_t* f[8] = {};
};
void launch_tp_signal(const TpPeerFlags& peers, int32_t world, int32_t rank, uint32_t value, cudaStream_t s);
// vocab-sharded logits: src [world][rows][vl] -> dst[r][w * vl + j]
// ---- model ingestion: safetensors values -> Q16.16 weights (convert.cu) --------------
enum SrcDtype : int32_t { kSrcF32 = 0, kSrcBF16 = 1, kSrcF16 = 2 };
// out[r * row_len + k] = f32_to_wgt(src value), row_mass[r] = sum_k |out|;
// stats[0] += non-finite values (written as 0), stats[1] |= 1 when a value
// does not fit i16.  stats must start at zero.
void launch_convert_wgt(const void* src, int dtype, uint64_t rows, uint64_t row_len, int32_t* out,
                        uint64_t* row_mass, uint32_t* stats, cudaStream_t s);

void launch_gather_vocab(const int32_t* src, int32_t world, int32_t rows, int32_t vl, int32_t* const* dst,
                         cudaStream_t s);
// dst[r] + off <- src row r (n ints), for r < rows; cap > 0 applies the
// logit softcap (softcap_act) to every value copied
void launch_scatter_rows(const int32_t* src, int32_t rows, int32_t n, int32_t* const* dst, size_t off,
                         cudaStream_t s, int32_t cap = 0);
void launch_copy_rows(const int32_t* src, int32_t* dst, size_t n, cudaStream_t s);
// synthetic weights (counter-based generator, see detwgt.py)
void launch_synth(void* dst, int32_t width, int32_t rank, int64_t n, int64_t cols, uint64_t key, cudaStream_t s);

int sm_count();
// one-time kernel attributes of the current device (idempotent; call outside
// stream capture before the first launch on a device)
void kernels_init();
// nonzero when a bounded pipeline wait in a streamed kernel gave up (reset: clear it)
int stream_error_flag(bool reset);

}  // namespace rdet
