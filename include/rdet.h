/*
 * rdet — B200-native deterministic integer-weight transformer path.
 *
 * C ABI of the drop-in CUDA executor for casettek/raster-inference's det
 * path.  A Rust executor `src/runtime/executors/cuda.rs` beside the
 * reference's `native.rs` binds these symbols through a thin FFI.  Every
 * call returns an int32 status (RDET_OK or a negative RDET_E_* code); the
 * message of the last failure on the calling thread is available from
 * rdet_last_error().  No exception or panic crosses this boundary.  All
 * results are bit-exact with the reference det path (det_num spec v1).
 *
 * Threading: one host thread drives one context at a time.  The
 * kernel-level entry points (rdet_det_gemv, rdet_det_linear,
 * rdet_det_attention_decode) may be called from several host threads; their
 * per-device scratch is handed out under a lock.
 */
#ifndef RDET_H_
#define RDET_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RDET_OK 0
#define RDET_NONE 1 /* commitment is None (reference returns Option::None) */
#define RDET_E_INVALID (-1)
#define RDET_E_IO (-2)
#define RDET_E_FORMAT (-3)
#define RDET_E_CUDA (-4)
#define RDET_E_STATE (-5)
#define RDET_E_RANGE (-6)
#define RDET_E_OOM (-7)

typedef struct rdet_ctx rdet_ctx;
typedef struct rdet_seq rdet_seq;

/* Options for rdet_open / rdet_open_synthetic. */
typedef struct rdet_opts {
  int32_t device;        /* CUDA device ordinal */
  uint32_t max_prefill;  /* largest prompt per prefill call (workspace sizing); 0 -> 4096 */
  uint32_t flags;        /* RDET_FLAG_* */
} rdet_opts;
#define RDET_FLAG_LAYER_COMMITMENTS 1u /* keep per-layer prefill commitments */
#define RDET_FLAG_NO_TENSOR_CORES 2u   /* prefill on CUDA cores only: no weight byte planes
                                          (saves one extra copy of the projection weights) */

typedef struct rdet_model_info {
  uint32_t hidden_size, vocab_size, num_layers, num_heads, ple_dim, intermediate_size;
  uint64_t weight_bytes; /* bytes of all weight tensors resident in HBM */
} rdet_model_info;

/* Buffers readable with rdet_read / rdet_commitment. */
#define RDET_BUF_EMBEDDING 0    /* [S,H] embedded prompt of the last prefill */
#define RDET_BUF_HIDDEN 1       /* [S,H] final hidden states (prefill) or [1,H] (decode) */
#define RDET_BUF_LOGITS 2       /* [V] last logits */
#define RDET_BUF_LAYER_OUTPUT 3 /* layer `layer` output of the last prefill ([S,H]) or decode ([1,H]) */
#define RDET_BUF_KV 4           /* whole KV cache (commitment only) */
#define RDET_BUF_KV_K 5         /* [rows,d] logical K rows of (layer, kv head = arg) */
#define RDET_BUF_KV_V 6

/* ---- model ---------------------------------------------------------------
 * Replaces load_transformer_state_model_from_det_num_wgt_path
 * (reference src/shared/model/gemma/io.rs:1043-1123): parses
 * <model_dir>/config.json and the fail-closed detwgt v2 artifact
 * <model_dir>/model.detwgt (io.rs:230-395) and uploads every tensor to HBM
 * once. */
int32_t rdet_open(const char* model_dir, const rdet_opts* opts, rdet_ctx** out);
/* Seeded random-init model of a config (JSON text); weights are generated in
 * HBM by the counter-based generator documented in detwgt.py, identical to
 * the artifact that detwgt.write_synthetic_model writes.  width: 16 or 32. */
int32_t rdet_open_synthetic(const char* config_json, uint64_t seed, int32_t width, const rdet_opts* opts,
                            rdet_ctx** out);
int32_t rdet_close(rdet_ctx* ctx);
int32_t rdet_get_model_info(rdet_ctx* ctx, rdet_model_info* out);

/* ---- sequences (TransformerDecodeState: per-layer KV cache in HBM) --------
 * Replaces TransformerDecodeState / LayerKvCache (model/transformer.rs:278-399). */
int32_t rdet_seq_new(rdet_ctx* ctx, uint32_t max_ctx, rdet_seq** out);
int32_t rdet_seq_free(rdet_seq* seq);
int32_t rdet_seq_position(rdet_seq* seq, uint32_t* position);

/* ---- routines ---------------------------------------------------------------
 * input.embedding (src/routines/input_embedding/mod.rs:17; io.rs:2446-2518). */
int32_t rdet_embed(rdet_ctx* ctx, const uint32_t* ids, size_t n, int32_t* act_out);

/* prefill_layer: input.embedding + prefill.prepare_aux + prefill.range over all
 * layers + prefill.finalize (native.rs:153-257 ->
 * prefill_range/native/deterministic_tiles.rs:69-199,
 * prefill_finalize/native/tiles.rs:11-107).  Logits stay resident. */
int32_t rdet_prefill(rdet_ctx* ctx, rdet_seq* seq, const uint32_t* ids, size_t n);
/* Routine-granular prefill: begin (embedding + PLE inputs), range over
 * [layer_start, layer_end), finalize (final norm, lm_head, softcap). */
int32_t rdet_prefill_begin(rdet_ctx* ctx, rdet_seq* seq, const uint32_t* ids, size_t n);
int32_t rdet_prefill_range(rdet_ctx* ctx, rdet_seq* seq, uint32_t layer_start, uint32_t layer_end);
int32_t rdet_prefill_finalize(rdet_ctx* ctx, rdet_seq* seq);

/* select_output_token: argmax_first over the resident logits, lowest index on
 * ties (decode_select_token/native/tiles.rs:22-38, det_num/ops.rs:463). */
int32_t rdet_select(rdet_ctx* ctx, rdet_seq* seq, uint32_t* token_out);
/* select_output_token for n sequences at once (the per-sequence routine of
 * decode_select_token/native/tiles.rs:22-38 applied to each):
 * tokens_out[i] = argmax_first of seqs[i]'s logits, lowest index on ties,
 * in one launch over all rows.  A sequence whose last batched decode ran
 * with vocab-sharded logits (rdet_tp_shard_logits) gets the token that
 * decode's global argmax selected; select it before its next decode. */
int32_t rdet_select_batch(rdet_ctx* ctx, rdet_seq* const* seqs, size_t n, uint32_t* tokens_out);

/* decode_transition for a (ragged) batch: for each sequence, embed its token
 * at its own position, run every layer (appending to its KV cache) and
 * project to logits (decode_layer_range/native/tiles.rs:133-197,
 * decode_transition_finalize/native/tiles.rs:9-65). */
int32_t rdet_decode(rdet_ctx* ctx, rdet_seq* const* seqs, const uint32_t* tokens, size_t nseq);
/* Routine-granular decode for one sequence (decode_layer_range init_state /
 * run_range / decode_transition_finalize). */
int32_t rdet_decode_begin(rdet_ctx* ctx, rdet_seq* seq, uint32_t token);
int32_t rdet_decode_range(rdet_ctx* ctx, rdet_seq* seq, uint32_t layer_start, uint32_t layer_end);
int32_t rdet_decode_finalize(rdet_ctx* ctx, rdet_seq* seq);

/* Greedy generation on the device (native.rs:265-450 loop: select ->
 * decode_transition, n_tokens times), each decode_transition replayed as the
 * sequence's CUDA graph.  Writes the n_tokens selected ids; logits of the
 * last decode stay resident. */
int32_t rdet_generate(rdet_ctx* ctx, rdet_seq* seq, uint32_t n_tokens, uint32_t* tokens_out);

/* ---- canonical bytes and commitments ----------------------------------------
 * rdet_read copies the canonical little-endian i32 values of a buffer into
 * dst (up to `bytes`) and reports the full size in *size_out.
 * rdet_commitment computes the reference's SHA-256 det commitment
 * (transformer_kernels.rs:1395-1482) as 64 lowercase hex chars + NUL:
 *   EMBEDDING, HIDDEN, LAYER_OUTPUT: build_det_activation_commitment (rows)
 *   LOGITS: build_det_vector_commitment
 *   KV: build_det_kv_cache_commitment over the caches of layers [0, layer)
 *       (layer 0: all layers); returns RDET_NONE when one of them has no
 *       cache of its own (KV-sharing layers), like the reference's None. */
int32_t rdet_read(rdet_ctx* ctx, rdet_seq* seq, int32_t which, int32_t layer, int32_t arg, void* dst, size_t bytes,
                  size_t* size_out);
int32_t rdet_commitment(rdet_ctx* ctx, rdet_seq* seq, int32_t which, int32_t layer, char* hex_out);
/* The KV commitments of the layer prefixes [0, p) for p = 1..n at once: what
 * n calls rdet_commitment(RDET_BUF_KV, p) return, i.e. det_layer_caches_sha256
 * of prefill.range_finalize after each layer (prefill_range_finalize/mod.rs:
 * 38-72 in the reference).  The caches download once and the n independent
 * hashes run on host threads.  hex_out holds n * 65 bytes; entry p-1 is the
 * hex + NUL, or an empty string where that prefix is RDET_NONE.  n <= layers. */
int32_t rdet_kv_prefix_commitments(rdet_ctx* ctx, rdet_seq* seq, uint32_t n, char* hex_out);

/* ---- kernel-level entry points on caller-owned device memory -----------------
 * det GEMV / linear: y[s, r] = requantize(sum_k x[s, k] * w[r, k]) with exact
 * wrapping i64 accumulation (det_kernels.rs:108-203 det_linear_rows_into /
 * det_linear_slab).  w is row-major [rows, cols], i16 (width 16) or i32
 * (width 32).  stream: a cudaStream_t or NULL.
 * rdet_det_linear with at least 32 rows of x, an i16 w whose cols are a
 * multiple of 16 (at most 32768) and 16-byte aligned x and w runs on the
 * tensor cores (exact byte-limb decomposition, same result); the byte planes
 * live in a per-device scratch that the library allocates on first use and
 * grows as needed, shared by all such calls on the device (calls that overlap
 * on the GPU race on it). */
int32_t rdet_det_gemv(const int32_t* x, const void* w, int32_t width, uint32_t rows, uint32_t cols, int32_t* y,
                      void* stream);
int32_t rdet_det_linear(const int32_t* x, uint32_t n_rows_x, const void* w, int32_t width, uint32_t rows,
                        uint32_t cols, int32_t* y, void* stream);

/* det decode attention of one token for every query head
 * (attention_output_into, det_kernels.rs:340-367, as driven by
 * det_layer_decode :1000-1053): q [num_heads, head_dim] holds the normed,
 * rotated queries; k_cache / v_cache [num_kv_heads, cap, head_dim] hold the
 * cache rows by position; rows [max(0, position + 1 - window), position] are
 * attended (window 0 = full attention); out [num_heads, head_dim].  Query head
 * h reads KV head h / (num_heads / num_kv_heads).  Scratch memory is allocated
 * by the library on first use per device and reused.  stream: cudaStream_t or
 * NULL. */
int32_t rdet_det_attention_decode(const int32_t* q, const int32_t* k_cache, const int32_t* v_cache, uint32_t cap,
                                  uint32_t num_heads, uint32_t num_kv_heads, uint32_t head_dim, uint32_t position,
                                  uint32_t window, int32_t* out, void* stream);

/* det prefill attention of n_tokens prompt positions for every query head
 * (det_attention_prefill, det_kernels.rs:525-671): q [n_tokens, num_heads,
 * head_dim] holds the normed, rotated queries; k_cache / v_cache [num_kv_heads,
 * cap, head_dim] hold the prompt's keys and values in rows [0, n_tokens);
 * query i attends to keys [max(0, i + 1 - window), i] (window 0 = causal over
 * the whole prompt); out [n_tokens, num_heads, head_dim].  Runs on the tcgen05
 * tensor cores when head_dim is a multiple of 64 and num_heads / num_kv_heads
 * divides 128 (flags RDET_FLAG_NO_TENSOR_CORES forces the CUDA-core kernel);
 * the result is the same either way.  Scratch memory is allocated by the
 * library on first use per device and grown as needed.  stream: cudaStream_t
 * or NULL. */
int32_t rdet_det_attention_prefill(const int32_t* q, const int32_t* k_cache, const int32_t* v_cache, uint32_t cap,
                                   uint32_t n_tokens, uint32_t num_heads, uint32_t num_kv_heads, uint32_t head_dim,
                                   uint32_t window, uint32_t flags, int32_t* out, void* stream);

/* Model ingestion on the GPU: safetensors values to det Q16.16 weights
 * (f32_to_wgt, det_num/convert.rs:77-93, as the reference's
 * gemma-det-num-wgt-converter applies it, tools/gemma-det-num-wgt-converter/
 * main.rs:218-388).  src holds rows * row_len little-endian values of dtype
 * RDET_SRC_*; out[i] = round half to even of value * 2^16, saturated to i32
 * (0 for a non-finite value); row_mass[r] = sum over the row of |out| (the
 * converter's overflow-bound input); stats[0] = the number of non-finite
 * values (the reference rejects the tensor when it is not 0), stats[1] = 1
 * when some value does not fit i16 (the tensor is then stored at width 32).
 * All pointers are device memory; stats is zeroed by the call. */
#define RDET_SRC_F32 0
#define RDET_SRC_BF16 1
#define RDET_SRC_F16 2
int32_t rdet_convert_to_wgt(const void* src, int32_t dtype, uint64_t rows, uint64_t row_len, int32_t* out,
                            uint64_t* row_mass, uint32_t* stats, void* stream);

/* Decode attention that allocates nothing.  Same arguments and the same
 * bit-exact result as rdet_det_attention_decode, for callers that cannot
 * allocate device memory while they run: a serving process that hands all of
 * HBM to weights and KV caches at start-up has none left to give, and an
 * executor that keeps its device footprint fixed across decode steps must not
 * allocate inside the step.  Its scratch is a fixed 4.8 MiB array inside the
 * library, which every GPU that loads the library holds until the process
 * exits.  Limits: num_heads <= 16, head_dim <= 512, and at most 4096 attended
 * rows (min(position + 1, window)); larger requests fail with RDET_E_RANGE.
 * The first call on a device looks up the array's address on that device
 * (with that device current) and should come before any stream capture.  All
 * calls share the one array, which keeps the previous call's contents: calls
 * that overlap on the GPU (other streams, other host threads) race.  The
 * array's address is looked up once per device ordinal and kept: after
 * cudaDeviceReset (or a release and re-creation of the device's primary
 * context) the kept address is stale, so do not call this entry point in a
 * process that resets the device after its first call.  This entry point has
 * no counterpart in the reference. */
int32_t rdet_det_attention_decode_noalloc(const int32_t* q, const int32_t* k_cache, const int32_t* v_cache,
                                          uint32_t cap, uint32_t num_heads, uint32_t num_kv_heads,
                                          uint32_t head_dim, uint32_t position, uint32_t window, int32_t* out,
                                          void* stream);

/* Tensor-parallel batched decode (no counterpart in the reference, which runs
 * one process on the CPU).  Every rank
 * opens the same model on its own GPU; rank 0 creates an id with
 * rdet_nccl_unique_id (128 bytes), the caller hands it to every rank, and each
 * calls rdet_tp_init with its rank.  Afterwards rdet_decode on two or more
 * sequences shards query heads, the MLP intermediate rows, the per-layer-input
 * rows and the vocabulary across the ranks: column-slice projections give exact
 * i64 partial sums that an NCCL int64 all-reduce completes before requantize,
 * and logits are all-gathered, so each rank's results are identical to an
 * unsharded decode.  All ranks must call rdet_decode with the same sequences
 * and tokens.  Prefill, single-sequence decode and commitments are unchanged
 * (every rank keeps the whole model and complete KV caches).  Needs the
 * tensor-core path (sm_100, i16 weights) and libnccl.so.2 at run time. */
int32_t rdet_nccl_unique_id(void* id_out, size_t len);
int32_t rdet_tp_init(rdet_ctx* ctx, int32_t rank, int32_t world, const void* id, size_t len);
int32_t rdet_tp_world(rdet_ctx* ctx); /* 1 when not sharded */
/* Vocab-sharded selection for the tensor-parallel batched decode (the
 * global argmax over a vocab-sharded lm_head; argmax_first,
 * det_num/ops.rs:463-478).  With on != 0, rdet_decode on two or more
 * sequences no longer all-gathers the logit rows: each rank finds the first
 * maximum of its own vocab rows per sequence, the ranks exchange those
 * (value, global index) pairs (8 bytes per row and chunk) and every rank
 * reduces them to the same tokens, which rdet_select_batch returns.  The
 * sequences' full logits are then not assembled on any rank: rdet_select,
 * rdet_generate, and reading or committing RDET_BUF_LOGITS fail with
 * RDET_E_STATE until their next prefill or unsharded decode.  on = 0
 * restores the default (logits all-gathered).  Needs rdet_tp_init. */
int32_t rdet_tp_shard_logits(rdet_ctx* ctx, int32_t on);

/* NVLink reduction for the tensor-parallel batched decode (no counterpart in
 * the reference).  After rdet_tp_init, every rank calls rdet_tp_ipc_export,
 * which allocates its reduction buffers for batches of up to max_batch
 * sequences and writes an opaque blob (*len = 136 bytes; cap must hold it;
 * every rank passes the same max_batch);
 * the caller gathers the blobs of all ranks in rank order (one process per
 * GPU) and every rank calls rdet_tp_ipc_connect with them.  From then on each
 * column-slice projection's i64 partial sums are stored by each rank into
 * every other rank's reduction buffer over NVLink (CUDA IPC peer memory,
 * plain stores) and summed there once the per-reduction flags are published,
 * instead of an NCCL all-reduce: same results bit for bit.  The flag waits are bounded; a rank that stops
 * publishing makes the others' rdet_decode fail with RDET_E_CUDA.  All ranks
 * must decode in lockstep and close their contexts only after every rank has
 * finished its last rdet_decode.  At most 8 ranks. */
int32_t rdet_tp_ipc_export(rdet_ctx* ctx, uint32_t max_batch, void* out, size_t cap, size_t* len);
int32_t rdet_tp_ipc_connect(rdet_ctx* ctx, const void* blobs, size_t len_each, int32_t world);

/* 1 when this context's prefill linears run on the tcgen05 tensor cores (an
 * sm_100 device, the context opened without RDET_FLAG_NO_TENSOR_CORES and at
 * least one eligible weight), else 0.  Prompts shorter than 32 tokens use the
 * CUDA-core linear either way.  No counterpart in the reference. */
int32_t rdet_tensor_core_prefill(rdet_ctx* ctx);
/* The CUDA stream (cudaStream_t) on which the context launches all of its
 * work, for callers that order their own work or CUDA events against it. */
int32_t rdet_get_stream(rdet_ctx* ctx, void** stream);
/* Number of kernels in one captured decode_transition (the sequence's decode
 * CUDA graph; captured on the first rdet_decode / rdet_generate). */
int32_t rdet_seq_kernels_per_step(rdet_seq* seq, uint32_t* kernels);

int32_t rdet_last_error(char* buf, size_t len);
const char* rdet_version(void);

#ifdef __cplusplus
}
#endif

#endif /* RDET_H_ */
