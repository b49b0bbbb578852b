"""B200-native deterministic integer-weight transformer path (rdet).

Host-side mirror of casettek/raster-inference's det routine API over the
C ABI in ``include/rdet.h`` (``librdet.so`` in this directory).  The names
follow the reference routines:

    load_transformer_state_model_from_det_num_wgt_path   io.rs:1043
    input_embedding                                      routines/input_embedding/mod.rs:17
    run_prefill (prefill_layer routine family)            executors/native.rs:153
    select_output_token                                  decode_select_token/native/tiles.rs:22
    decode_transition                                    executors/native.rs:339-437
    run_output_decode                                    executors/native.rs:265

There is no CPU fallback: every entry point raises ImportError when the CUDA
library is missing, and fails with ``RdetError`` carrying the reference's
error message when the C ABI reports a failure.
"""
from __future__ import annotations

import ctypes as C
import json
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "librdet.so")

RDET_OK, RDET_NONE = 0, 1
BUF_EMBEDDING, BUF_HIDDEN, BUF_LOGITS, BUF_LAYER_OUTPUT, BUF_KV, BUF_KV_K, BUF_KV_V = range(7)
FLAG_LAYER_COMMITMENTS = 1
FLAG_NO_TENSOR_CORES = 2

# Exported symbols, in the order include/rdet.h declares them.
SYMBOLS = [
    "rdet_open", "rdet_open_synthetic", "rdet_close", "rdet_get_model_info", "rdet_seq_new", "rdet_seq_free",
    "rdet_seq_position", "rdet_embed", "rdet_prefill", "rdet_prefill_begin", "rdet_prefill_range",
    "rdet_prefill_finalize", "rdet_select", "rdet_select_batch", "rdet_decode", "rdet_decode_begin", "rdet_decode_range",
    "rdet_decode_finalize", "rdet_generate", "rdet_read", "rdet_commitment", "rdet_kv_prefix_commitments",
    "rdet_det_gemv", "rdet_det_linear",
    "rdet_det_attention_decode", "rdet_det_attention_decode_noalloc", "rdet_det_attention_prefill", "rdet_convert_to_wgt", "rdet_get_stream", "rdet_tensor_core_prefill", "rdet_nccl_unique_id", "rdet_tp_init", "rdet_tp_world", "rdet_tp_shard_logits", "rdet_tp_ipc_export", "rdet_tp_ipc_connect", "rdet_seq_kernels_per_step", "rdet_last_error",
    "rdet_version",
]


class RdetError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"rdet error {code}: {msg}")
        self.code = code
        self.msg = msg


class Opts(C.Structure):
    _fields_ = [("device", C.c_int32), ("max_prefill", C.c_uint32), ("flags", C.c_uint32)]


class ModelInfo(C.Structure):
    _fields_ = [("hidden_size", C.c_uint32), ("vocab_size", C.c_uint32), ("num_layers", C.c_uint32),
                ("num_heads", C.c_uint32), ("ple_dim", C.c_uint32), ("intermediate_size", C.c_uint32),
                ("weight_bytes", C.c_uint64)]


_lib = None


def lib() -> C.CDLL:
    """Load librdet.so (raises if it was not built — there is no fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: build it with `make -C {_HERE}` (no CPU fallback exists)")
    L = C.CDLL(LIB_PATH)
    p, i32, u32, u64, sz = C.c_void_p, C.c_int32, C.c_uint32, C.c_uint64, C.c_size_t
    sig = {
        "rdet_open": [C.c_char_p, p, p],
        "rdet_open_synthetic": [C.c_char_p, u64, i32, p, p],
        "rdet_close": [p],
        "rdet_get_model_info": [p, p],
        "rdet_seq_new": [p, u32, p],
        "rdet_seq_free": [p],
        "rdet_seq_position": [p, p],
        "rdet_embed": [p, p, sz, p],
        "rdet_prefill": [p, p, p, sz],
        "rdet_prefill_begin": [p, p, p, sz],
        "rdet_prefill_range": [p, p, u32, u32],
        "rdet_prefill_finalize": [p, p],
        "rdet_select": [p, p, p],
        "rdet_select_batch": [p, p, sz, p],
        "rdet_tp_shard_logits": [p, i32],
        "rdet_decode": [p, p, p, sz],
        "rdet_decode_begin": [p, p, u32],
        "rdet_decode_range": [p, p, u32, u32],
        "rdet_decode_finalize": [p, p],
        "rdet_generate": [p, p, u32, p],
        "rdet_read": [p, p, i32, i32, i32, p, sz, p],
        "rdet_commitment": [p, p, i32, i32, C.c_char_p],
        "rdet_kv_prefix_commitments": [p, p, C.c_uint32, C.c_char_p],
        "rdet_det_gemv": [p, p, i32, u32, u32, p, p],
        "rdet_det_linear": [p, u32, p, i32, u32, u32, p, p],
        "rdet_det_attention_decode": [p, p, p, u32, u32, u32, u32, u32, u32, p, p],
        "rdet_det_attention_decode_noalloc": [p, p, p, u32, u32, u32, u32, u32, u32, p, p],
        "rdet_det_attention_prefill": [p, p, p, u32, u32, u32, u32, u32, u32, u32, p, p],
        "rdet_convert_to_wgt": [p, i32, C.c_uint64, C.c_uint64, p, p, p, p],
        "rdet_get_stream": [p, p],
        "rdet_tensor_core_prefill": [p],
        "rdet_nccl_unique_id": [p, sz],
        "rdet_tp_init": [p, i32, i32, p, sz],
        "rdet_tp_world": [p],
        "rdet_tp_ipc_export": [p, u32, p, sz, p],
        "rdet_tp_ipc_connect": [p, p, sz, i32],
        "rdet_seq_kernels_per_step": [p, p],
        "rdet_last_error": [C.c_char_p, sz],
    }
    for name, args in sig.items():
        f = getattr(L, name)
        f.argtypes = args
        f.restype = i32
    L.rdet_version.restype = C.c_char_p
    L.rdet_version.argtypes = []
    _lib = L
    return L


def _check(rc: int):
    if rc < 0:
        buf = C.create_string_buffer(4096)
        lib().rdet_last_error(buf, 4096)
        raise RdetError(rc, buf.value.decode(errors="replace"))
    return rc


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


class Model:
    """Gemma-4 det model resident in HBM (Gemma4TransformerModel, model/gemma/transformer.rs:560)."""

    def __init__(self, handle, config: dict | None):
        self._h = handle
        self.config = config
        info = ModelInfo()
        _check(lib().rdet_get_model_info(self._h, C.byref(info)))
        self.H, self.V, self.L = info.hidden_size, info.vocab_size, info.num_layers
        self.Hq, self.P, self.F = info.num_heads, info.ple_dim, info.intermediate_size
        self.weight_bytes = info.weight_bytes

    @classmethod
    def open(cls, model_dir: str, device: int = 0, max_prefill: int = 0, layer_commitments: bool = False,
             tensor_cores: bool = True):
        flags = (FLAG_LAYER_COMMITMENTS if layer_commitments else 0) | (0 if tensor_cores else FLAG_NO_TENSOR_CORES)
        opts = Opts(device, max_prefill, flags)
        h = C.c_void_p()
        _check(lib().rdet_open(model_dir.encode(), C.byref(opts), C.byref(h)))
        with open(os.path.join(model_dir, "config.json")) as f:
            cfg = json.load(f)
        return cls(h, cfg)

    @classmethod
    def synthetic(cls, config: dict, seed: int, width: int = 16, device: int = 0, max_prefill: int = 0,
                  layer_commitments: bool = False, tensor_cores: bool = True):
        flags = (FLAG_LAYER_COMMITMENTS if layer_commitments else 0) | (0 if tensor_cores else FLAG_NO_TENSOR_CORES)
        opts = Opts(device, max_prefill, flags)
        h = C.c_void_p()
        _check(lib().rdet_open_synthetic(json.dumps(config).encode(), seed, width, C.byref(opts), C.byref(h)))
        return cls(h, config)

    def close(self):
        if getattr(self, "_h", None):
            lib().rdet_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def tp_init(self, rank: int, world: int, uid: bytes):
        """Shard the batched decode over `world` ranks (rdet_tp_init); every rank
        opened the same model and passes the same id from nccl_unique_id()."""
        buf = C.create_string_buffer(bytes(uid), len(uid))
        _check(lib().rdet_tp_init(self._h, rank, world, buf, len(uid)))

    def tp_shard_logits(self, on: bool = True) -> None:
        """Vocab-sharded selection (rdet_tp_shard_logits): batched decodes end
        with a global argmax over (value, index) pairs instead of gathering
        the logit rows; take the tokens with select_batch."""
        _check(lib().rdet_tp_shard_logits(self._h, 1 if on else 0))

    def tp_ipc_export(self, max_batch: int) -> bytes:
        """This rank's NVLink reduction buffers for batches of up to max_batch
        sequences (rdet_tp_ipc_export): an opaque blob for every other rank."""
        buf = C.create_string_buffer(256)
        n = C.c_size_t(0)
        _check(lib().rdet_tp_ipc_export(self._h, max_batch, buf, 256, C.byref(n)))
        return buf.raw[: n.value]

    def tp_ipc_connect(self, blobs) -> None:
        """Map the other ranks' reduction buffers (all ranks' export blobs in
        rank order, rdet_tp_ipc_connect): the sharded decode then reduces over
        NVLink instead of NCCL."""
        each = len(blobs[0])
        assert all(len(b) == each for b in blobs)
        buf = C.create_string_buffer(b"".join(blobs), each * len(blobs))
        _check(lib().rdet_tp_ipc_connect(self._h, buf, each, len(blobs)))

    @property
    def tp_world(self) -> int:
        return int(lib().rdet_tp_world(self._h))

    @property
    def tensor_core_prefill(self) -> bool:
        """Whether prefill linears of >= 32 tokens run on the tcgen05 tensor cores."""
        return bool(lib().rdet_tensor_core_prefill(self._h))

    @property
    def stream(self) -> int:
        """cudaStream_t (as an int) on which this model launches its work."""
        v = C.c_void_p()
        _check(lib().rdet_get_stream(self._h, C.byref(v)))
        return v.value or 0

    def new_sequence(self, max_ctx: int) -> "Sequence":
        h = C.c_void_p()
        _check(lib().rdet_seq_new(self._h, max_ctx, C.byref(h)))
        return Sequence(self, h)

    def embed(self, ids) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        out = np.zeros((ids.size, self.H), dtype=np.int32)
        _check(lib().rdet_embed(self._h, _ptr(ids), ids.size, _ptr(out)))
        return out


class Sequence:
    """One sequence's decode state (TransformerDecodeState) with its KV cache in HBM."""

    def __init__(self, model: Model, handle):
        self.model = model
        self._h = handle

    def free(self):
        if getattr(self, "_h", None):
            if getattr(self.model, "_h", None):  # closing the model already freed it
                lib().rdet_seq_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass

    @property
    def position(self) -> int:
        v = C.c_uint32()
        _check(lib().rdet_seq_position(self._h, C.byref(v)))
        return v.value

    # -- routines -------------------------------------------------------------
    def prefill(self, ids):
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        _check(lib().rdet_prefill(self.model._h, self._h, _ptr(ids), ids.size))

    def prefill_begin(self, ids):
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        _check(lib().rdet_prefill_begin(self.model._h, self._h, _ptr(ids), ids.size))

    def prefill_range(self, start: int, end: int):
        _check(lib().rdet_prefill_range(self.model._h, self._h, start, end))

    def prefill_finalize(self):
        _check(lib().rdet_prefill_finalize(self.model._h, self._h))

    def select(self) -> int:
        t = C.c_uint32()
        _check(lib().rdet_select(self.model._h, self._h, C.byref(t)))
        return t.value

    def decode(self, token: int):
        arr = (C.c_void_p * 1)(self._h)
        toks = np.array([token], dtype=np.uint32)
        _check(lib().rdet_decode(self.model._h, arr, _ptr(toks), 1))

    def decode_begin(self, token: int):
        _check(lib().rdet_decode_begin(self.model._h, self._h, token))

    def decode_range(self, start: int, end: int):
        _check(lib().rdet_decode_range(self.model._h, self._h, start, end))

    def decode_finalize(self):
        _check(lib().rdet_decode_finalize(self.model._h, self._h))

    def generate(self, n: int) -> list[int]:
        out = np.zeros(max(n, 1), dtype=np.uint32)
        _check(lib().rdet_generate(self.model._h, self._h, n, _ptr(out)))
        return [int(v) for v in out[:n]]

    def kernels_per_step(self) -> int:
        v = C.c_uint32()
        _check(lib().rdet_seq_kernels_per_step(self._h, C.byref(v)))
        return v.value

    # -- canonical bytes / commitments -------------------------------------------
    def read(self, which: int, layer: int = 0, arg: int = 0) -> np.ndarray:
        size = C.c_size_t()
        _check(lib().rdet_read(self.model._h, self._h, which, layer, arg, None, 0, C.byref(size)))
        out = np.zeros(size.value // 4, dtype=np.int32)
        _check(lib().rdet_read(self.model._h, self._h, which, layer, arg, _ptr(out), size.value, C.byref(size)))
        return out

    def commitment(self, which: int, layer: int = 0):
        buf = C.create_string_buffer(65)
        rc = _check(lib().rdet_commitment(self.model._h, self._h, which, layer, buf))
        return None if rc == RDET_NONE else buf.value.decode()

    def kv_prefix_commitments(self, n: int) -> list:
        """commitment(BUF_KV, p) for p = 1..n in one call (None where a
        prefix holds a KV-sharing layer)."""
        buf = C.create_string_buffer(65 * max(n, 1))
        _check(lib().rdet_kv_prefix_commitments(self.model._h, self._h, n, buf))
        out = []
        for p in range(n):
            h = buf.raw[65 * p:65 * p + 64]
            out.append(None if h[0] == 0 else h.decode())
        return out

    def logits(self) -> np.ndarray:
        return self.read(BUF_LOGITS)


def nccl_unique_id() -> bytes:
    """A fresh NCCL id (128 bytes) for Model.tp_init on every rank."""
    buf = C.create_string_buffer(128)
    _check(lib().rdet_nccl_unique_id(buf, 128))
    return buf.raw


def decode_batch(model: Model, seqs, tokens):
    """decode_transition over a ragged batch (one token per sequence)."""
    arr = (C.c_void_p * len(seqs))(*[s._h for s in seqs])
    toks = np.ascontiguousarray(tokens, dtype=np.uint32)
    _check(lib().rdet_decode(model._h, arr, _ptr(toks), len(seqs)))


def select_batch(model: Model, seqs) -> list[int]:
    """select_output_token for every sequence in one launch (argmax_first of
    each sequence's logits; after a vocab-sharded tensor-parallel decode,
    the tokens its global argmax selected)."""
    n = len(seqs)
    arr = (C.c_void_p * max(n, 1))(*[s._h for s in seqs])
    out = np.zeros(max(n, 1), dtype=np.uint32)
    _check(lib().rdet_select_batch(model._h, arr, n, _ptr(out)))
    return [int(v) for v in out[:n]]


# ---- reference-named entry points ---------------------------------------------------
def load_transformer_state_model_from_det_num_wgt_path(model_dir: str, **kw) -> Model:
    return Model.open(model_dir, **kw)


def input_embedding(model: Model, prompt_token_ids) -> np.ndarray:
    return model.embed(prompt_token_ids)


def run_prefill(model: Model, prompt_token_ids, max_ctx: int) -> Sequence:
    seq = model.new_sequence(max_ctx)
    seq.prefill(prompt_token_ids)
    return seq


def select_output_token(seq: Sequence) -> int:
    return seq.select()


def decode_transition(seq: Sequence, next_token: int):
    seq.decode(next_token)


def run_output_decode(seq: Sequence, max_new_tokens: int) -> list[int]:
    """Greedy loop of executors/native.rs:265-450 (select, then decode)."""
    return seq.generate(max_new_tokens)


def det_gemv(x_ptr: int, w_ptr: int, width: int, rows: int, cols: int, y_ptr: int, stream: int = 0):
    """GEMV on caller-owned device pointers (integers, e.g. torch data_ptr())."""
    _check(lib().rdet_det_gemv(C.c_void_p(x_ptr), C.c_void_p(w_ptr), width, rows, cols, C.c_void_p(y_ptr),
                               C.c_void_p(stream) if stream else None))


def det_linear(x_ptr: int, s: int, w_ptr: int, width: int, rows: int, cols: int, y_ptr: int, stream: int = 0):
    _check(lib().rdet_det_linear(C.c_void_p(x_ptr), s, C.c_void_p(w_ptr), width, rows, cols, C.c_void_p(y_ptr),
                                 C.c_void_p(stream) if stream else None))


def det_attention_decode(q_ptr: int, k_ptr: int, v_ptr: int, cap: int, num_heads: int, num_kv_heads: int,
                         head_dim: int, position: int, window: int, out_ptr: int, stream: int = 0):
    """Decode attention of one token on caller-owned device memory (rdet_det_attention_decode)."""
    _check(lib().rdet_det_attention_decode(C.c_void_p(q_ptr), C.c_void_p(k_ptr), C.c_void_p(v_ptr), cap, num_heads,
                                           num_kv_heads, head_dim, position, window, C.c_void_p(out_ptr),
                                           C.c_void_p(stream) if stream else None))


def det_attention_prefill(q_ptr: int, k_ptr: int, v_ptr: int, cap: int, n_tokens: int, num_heads: int,
                          num_kv_heads: int, head_dim: int, window: int, out_ptr: int, tensor_cores: bool = True,
                          stream: int = 0):
    """Prefill attention of a prompt on caller-owned device memory
    (rdet_det_attention_prefill); tensor_cores=False forces the CUDA-core kernel."""
    _check(lib().rdet_det_attention_prefill(C.c_void_p(q_ptr), C.c_void_p(k_ptr), C.c_void_p(v_ptr), cap, n_tokens,
                                            num_heads, num_kv_heads, head_dim, window,
                                            0 if tensor_cores else FLAG_NO_TENSOR_CORES, C.c_void_p(out_ptr),
                                            C.c_void_p(stream) if stream else None))


SRC_DTYPES = {"F32": 0, "BF16": 1, "F16": 2}


def convert_to_wgt(src_ptr: int, dtype: str, rows: int, row_len: int, out_ptr: int, row_mass_ptr: int,
                   stats_ptr: int, stream: int = 0):
    """safetensors values -> Q16.16 weights on the GPU (rdet_convert_to_wgt):
    out = f32_to_wgt(value), row_mass = sum |out| per row, stats = [non-finite
    count, does not fit i16]; all device pointers."""
    _check(lib().rdet_convert_to_wgt(C.c_void_p(src_ptr), SRC_DTYPES[dtype], rows, row_len, C.c_void_p(out_ptr),
                                     C.c_void_p(row_mass_ptr), C.c_void_p(stats_ptr),
                                     C.c_void_p(stream) if stream else None))


def det_attention_decode_noalloc(q_ptr: int, k_ptr: int, v_ptr: int, cap: int, num_heads: int, num_kv_heads: int,
                                 head_dim: int, position: int, window: int, out_ptr: int, stream: int = 0):
    """rdet_det_attention_decode without any device allocation, for callers
    that cannot allocate device memory while they run (all of HBM handed to
    weights and KV caches up front, or a fixed per-step footprint).  Scratch
    is the library's fixed 4.8 MiB array; limits: 16 heads, head_dim 512,
    4096 attended rows.  Calls that overlap on the GPU race on that array."""
    _check(lib().rdet_det_attention_decode_noalloc(C.c_void_p(q_ptr), C.c_void_p(k_ptr), C.c_void_p(v_ptr), cap,
                                                   num_heads, num_kv_heads, head_dim, position, window,
                                                   C.c_void_p(out_ptr), C.c_void_p(stream) if stream else None))
