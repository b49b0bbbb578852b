"""CPU ORACLE — TEST INFRASTRUCTURE ONLY.

ctypes binding for ``oracle/_build/libdet_oracle.so``, the C++ restatement of
casettek/raster-inference's deterministic integer-weight path (see the header
of ``det_oracle.cpp`` for the reference file:line map).  Imported only by
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (cpu_baseline leg and
the ``--impl reference`` arm), always as the checker or the timed CPU
baseline, never as the product path.

Parity status: pinned.  The scalar arithmetic is checked against the
reference's known-answer vectors (src/shared/numerics/det_num/tests.rs) and
the whole path against both det fixtures of
testdata/det_commitment_goldens.json (tests/test_oracle_goldens.py).
"""
from __future__ import annotations

import ctypes as C
import json
import math
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_build", "libdet_oracle.so")
_lib = None


class Config(C.Structure):
    _fields_ = [
        ("hidden_size", C.c_int32), ("num_hidden_layers", C.c_int32),
        ("num_attention_heads", C.c_int32), ("num_key_value_heads", C.c_int32),
        ("head_dim", C.c_int32), ("global_head_dim", C.c_int32),
        ("num_global_key_value_heads", C.c_int32), ("hidden_size_per_layer_input", C.c_int32),
        ("vocab_size", C.c_int32), ("vocab_size_per_layer_input", C.c_int32),
        ("sliding_window", C.c_int32), ("num_kv_shared_layers", C.c_int32),
        ("attention_k_eq_v", C.c_int32), ("tie_word_embeddings", C.c_int32),
        ("bidirectional_all", C.c_int32), ("enable_moe_block", C.c_int32),
        ("hidden_activation_is_gelu_tanh", C.c_int32), ("has_softcap", C.c_int32),
        ("final_logit_softcapping", C.c_float), ("rms_norm_eps", C.c_float),
        ("has_full_partial", C.c_int32), ("has_full_theta", C.c_int32),
        ("has_sliding_theta", C.c_int32), ("has_global_theta", C.c_int32),
        ("full_partial_rotary_factor", C.c_float), ("full_rope_theta", C.c_float),
        ("sliding_rope_theta", C.c_float), ("global_rope_theta", C.c_float),
        ("n_layer_types", C.c_int32), ("layer_is_sliding", C.c_int32 * 1024),
    ]


def build(quiet: bool = True) -> str:
    """Compile the oracle library with its Makefile (checker build only)."""
    out = subprocess.run(["make", "-C", _HERE], capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + out.stdout + out.stderr)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        i32, i64, u32, sz, p = C.c_int32, C.c_int64, C.c_uint32, C.c_size_t, C.c_void_p
        sig = {
            "dor_set_threads": (None, [C.c_int]),
            "dor_get_threads": (C.c_int, []),
            "dor_model_open": (p, [C.c_char_p, C.POINTER(Config), C.c_char_p, sz]),
            "dor_detwgt_validate": (C.c_long, [p, sz, C.c_char_p, sz]),
            "dor_model_close": (None, [p]),
            "dor_model_open_synthetic": (p, [C.POINTER(Config), C.c_uint64, C.c_int, C.c_int, C.c_int, C.c_char_p, sz]),
            "dor_model_info": (C.c_int, [p, p, sz]),
            "dor_seq_new": (p, [p]),
            "dor_seq_free": (None, [p]),
            "dor_seq_position": (i64, [p]),
            "dor_embed": (C.c_int, [p, p, sz, p, C.c_char_p, sz]),
            "dor_prefill": (C.c_int, [p, p, p, sz, p, p, p, C.c_char_p, sz]),
            "dor_decode": (C.c_int, [p, p, u32, p, p, p, C.c_char_p, sz]),
            "dor_seq_fill_synthetic": (C.c_int, [p, p, sz, C.c_uint64]),
            "dor_kv_commitment": (C.c_int, [p, C.c_char_p]),
            "dor_kv_commitment_prefix": (C.c_int, [p, sz, C.c_char_p]),
            "dor_kv_read": (C.c_long, [p, C.c_int, C.c_int, C.c_int, p, sz]),
            "dor_argmax_first": (u32, [p, sz]),
            "dor_attention_one": (None, [p, p, p, sz, sz, p]),
            "dor_act_commitment": (None, [p, sz, sz, C.c_char_p]),
            "dor_vec_commitment": (None, [p, sz, C.c_char_p]),
            "dor_sha256_hex": (None, [p, sz, C.c_char_p]),
            "dor_gemv": (None, [p, p, C.c_int, sz, sz, p]),
            "dor_linear": (None, [p, sz, p, C.c_int, sz, sz, p]),
            "dor_requantize": (i32, [i64]),
            "dor_rshift_rte": (i64, [i64, u32]),
            "dor_mac_bits": (i64, [i64, i32, i32]),
            "dor_acc_combine": (i64, [i64, i64]),
            "dor_add_sat": (i32, [i32, i32]),
            "dor_sub_sat": (i32, [i32, i32]),
            "dor_acc_add_sat": (i64, [i64, i64]),
            "dor_mul_sat": (i32, [i32, i32]),
            "dor_div_act": (i32, [i32, i32]),
            "dor_div_acc_by_u32": (i64, [i64, u32]),
            "dor_tanh": (i32, [i32]),
            "dor_softcap": (i32, [i32, i32]),
            "dor_gelu": (i32, [i32]),
            "dor_f32_to_act": (i32, [C.c_float]),
            "dor_f32_to_acc": (i64, [C.c_float]),
            "dor_rms_norm_scale": (i32, [p, sz, i64]),
            "dor_rms_norm": (None, [p, p, sz, i64]),
            "dor_value_rms_norm": (None, [p, sz, i64]),
            "dor_softmax": (None, [p, sz, p]),
            "dor_softmax_exp_term": (i64, [i32, i32]),
            "dor_rope_step": (i64, [i64, sz]),
            "dor_rope": (None, [p, sz, sz, i64, sz]),
            "dor_sin_cos": (None, [i64, p, p]),
            "dor_attention_score": (i32, [p, p, sz]),
            "dor_weighted_sum": (None, [p, sz, p, sz, p]),
        }
        for name, (res, args) in sig.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def config_from_dict(cfg: dict) -> Config:
    """Mirror of the reference's GemmaTextConfigFile fields (io.rs:61-83)."""
    t = cfg.get("text_config", cfg)
    c = Config()

    def opt(key, default=-1):
        v = t.get(key)
        return default if v is None else v

    c.hidden_size = t["hidden_size"]
    c.num_hidden_layers = t["num_hidden_layers"]
    c.num_attention_heads = t["num_attention_heads"]
    c.num_key_value_heads = t["num_key_value_heads"]
    c.head_dim = t["head_dim"]
    c.global_head_dim = opt("global_head_dim")
    c.num_global_key_value_heads = opt("num_global_key_value_heads")
    c.hidden_size_per_layer_input = opt("hidden_size_per_layer_input")
    c.vocab_size = t["vocab_size"]
    c.vocab_size_per_layer_input = opt("vocab_size_per_layer_input")
    c.sliding_window = t["sliding_window"]
    c.num_kv_shared_layers = opt("num_kv_shared_layers")
    kv = t.get("attention_k_eq_v")
    c.attention_k_eq_v = -1 if kv is None else int(bool(kv))
    tie = t.get("tie_word_embeddings")
    c.tie_word_embeddings = -1 if tie is None else int(bool(tie))
    c.bidirectional_all = int(t.get("use_bidirectional_attention") == "all")
    c.enable_moe_block = int(bool(t["enable_moe_block"]))
    c.hidden_activation_is_gelu_tanh = int(t["hidden_activation"] == "gelu_pytorch_tanh")
    sc = t.get("final_logit_softcapping")
    c.has_softcap = int(sc is not None)
    c.final_logit_softcapping = float(sc) if sc is not None else 0.0
    c.rms_norm_eps = float(t["rms_norm_eps"])
    rp = t.get("rope_parameters") or {}
    full = rp.get("full_attention") or {}
    slid = rp.get("sliding_attention") or {}
    c.has_full_partial = int(full.get("partial_rotary_factor") is not None)
    c.full_partial_rotary_factor = float(full.get("partial_rotary_factor") or 0.0)
    c.has_full_theta = int(full.get("rope_theta") is not None)
    c.full_rope_theta = float(full.get("rope_theta") or 0.0)
    c.has_sliding_theta = int(slid.get("rope_theta") is not None)
    c.sliding_rope_theta = float(slid.get("rope_theta") or 0.0)
    c.has_global_theta = int(rp.get("rope_theta") is not None)
    c.global_rope_theta = float(rp.get("rope_theta") or 0.0)
    lt = t["layer_types"]
    c.n_layer_types = len(lt)
    for i, s in enumerate(lt):
        c.layer_is_sliding[i] = int(s == "sliding_attention")
    return c


class OracleError(RuntimeError):
    pass


class Model:
    """A det model loaded by the oracle from ``model_dir`` (config.json + model.detwgt)."""

    def __init__(self, model_dir: str | None, threads: int | None = None, synthetic: tuple | None = None):
        """Load ``model_dir`` (config.json + model.detwgt), or with
        ``synthetic=(config_dict, seed, width)`` generate the seeded synthetic
        model of raster-inference_b200/detwgt.py in host memory."""
        L = lib()
        if threads is not None:
            L.dor_set_threads(threads)
        err = C.create_string_buffer(1024)
        if synthetic is not None:
            cfg, seed, width = synthetic
            self.config = cfg
            self._cfg = config_from_dict(cfg)
            t = cfg.get("text_config", cfg)
            h = L.dor_model_open_synthetic(C.byref(self._cfg), seed, width, t["intermediate_size"],
                                           int(t.get("_synthetic_layer_scalar", True)), err, 1024)
        else:
            with open(os.path.join(model_dir, "config.json")) as f:
                self.config = json.load(f)
            self._cfg = config_from_dict(self.config)
            h = L.dor_model_open(os.path.join(model_dir, "model.detwgt").encode(), C.byref(self._cfg), err, 1024)
        if not h:
            raise OracleError(err.value.decode())
        self._h = h
        info = np.zeros(8 + 8 * 1024, dtype=np.int64)
        n = L.dor_model_info(h, _ptr(info), info.size)
        self.H, self.V, self.L, self.Hq, self.P = (int(v) for v in info[:5])
        self.layers = [dict(zip(["head_dim", "kv_heads", "rotary_dim", "sliding", "window", "cache_trim", "donor", "k_eq_v"],
                                (int(v) for v in info[5 + 8 * i: 13 + 8 * i]))) for i in range(self.L)]
        assert n == 5 + 8 * self.L

    def close(self):
        if getattr(self, "_h", None):
            lib().dor_model_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def embed(self, ids) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        out = np.zeros((ids.size, self.H), dtype=np.int32)
        err = C.create_string_buffer(1024)
        if lib().dor_embed(self._h, _ptr(ids), ids.size, _ptr(out), err, 1024) != 0:
            raise OracleError(err.value.decode())
        return out

    def seq(self) -> "Seq":
        return Seq(self)


class Seq:
    def __init__(self, model: Model):
        self.m = model
        self._h = lib().dor_seq_new(model._h)

    def __del__(self):
        try:
            lib().dor_seq_free(self._h)
        except Exception:
            pass

    @property
    def position(self) -> int:
        return int(lib().dor_seq_position(self._h))

    def prefill(self, ids, want_hidden=True, want_layer_hashes=True):
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        m = self.m
        hidden = np.zeros((ids.size, m.H), dtype=np.int32) if want_hidden else None
        logits = np.zeros(m.V, dtype=np.int32)
        hashes = C.create_string_buffer(65 * m.L) if want_layer_hashes else None
        err = C.create_string_buffer(1024)
        rc = lib().dor_prefill(m._h, self._h, _ptr(ids), ids.size,
                               _ptr(hidden) if hidden is not None else None, _ptr(logits),
                               hashes, err, 1024)
        if rc != 0:
            raise OracleError(err.value.decode())
        lh = [hashes.raw[65 * i: 65 * i + 64].decode() for i in range(m.L)] if hashes is not None else None
        return hidden, logits, lh

    def decode(self, token: int, want_layer_hashes=True):
        m = self.m
        hidden = np.zeros(m.H, dtype=np.int32)
        logits = np.zeros(m.V, dtype=np.int32)
        hashes = C.create_string_buffer(65 * m.L) if want_layer_hashes else None
        err = C.create_string_buffer(1024)
        rc = lib().dor_decode(m._h, self._h, int(token), _ptr(hidden), _ptr(logits), hashes, err, 1024)
        if rc != 0:
            raise OracleError(err.value.decode())
        lh = [hashes.raw[65 * i: 65 * i + 64].decode() for i in range(m.L)] if hashes is not None else None
        return hidden, logits, lh

    def fill_synthetic(self, ctx: int, seed: int = 1):
        lib().dor_seq_fill_synthetic(self.m._h, self._h, ctx, seed)

    def kv_commitment(self, layers: int | None = None):
        """KV commitment over every layer's cache, or over layers [0, layers)."""
        out = C.create_string_buffer(65)
        rc = (lib().dor_kv_commitment(self._h, out) if layers is None else
              lib().dor_kv_commitment_prefix(self._h, layers, out))
        return None if rc != 0 else out.value.decode()

    def kv_rows(self, layer: int, head: int, kind: int) -> np.ndarray | None:
        d = self.m.layers[layer]["head_dim"]
        cap = 1 << 24
        buf = np.zeros(cap, dtype=np.int32)
        n = lib().dor_kv_read(self._h, layer, head, kind, _ptr(buf), cap)
        if n < 0:
            return None
        return buf[: n * d].reshape(n, d).copy()


def argmax_first(x) -> int:
    x = np.ascontiguousarray(x, dtype=np.int32)
    return int(lib().dor_argmax_first(_ptr(x), x.size))


def act_commitment(x) -> str:
    x = np.ascontiguousarray(x, dtype=np.int32)
    if x.ndim == 1:
        x = x.reshape(1, -1)
    out = C.create_string_buffer(65)
    lib().dor_act_commitment(_ptr(x), x.shape[0], x.shape[1], out)
    return out.value.decode()


def vec_commitment(x) -> str:
    x = np.ascontiguousarray(x, dtype=np.int32).ravel()
    out = C.create_string_buffer(65)
    lib().dor_vec_commitment(_ptr(x), x.size, out)
    return out.value.decode()


def gemv(x, w) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.int32)
    w = np.ascontiguousarray(w)
    width = {np.dtype(np.int16): 16, np.dtype(np.int32): 32}[w.dtype]
    N, K = w.shape
    y = np.zeros(N, dtype=np.int32)
    lib().dor_gemv(_ptr(x), _ptr(w), width, N, K, _ptr(y))
    return y


def linear(X, w) -> np.ndarray:
    X = np.ascontiguousarray(X, dtype=np.int32)
    w = np.ascontiguousarray(w)
    width = {np.dtype(np.int16): 16, np.dtype(np.int32): 32}[w.dtype]
    N, K = w.shape
    Y = np.zeros((X.shape[0], N), dtype=np.int32)
    lib().dor_linear(_ptr(X), X.shape[0], _ptr(w), width, N, K, _ptr(Y))
    return Y


def set_threads(n: int):
    lib().dor_set_threads(int(n))


def cpu_count() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def validate_detwgt(b: bytes):
    err = C.create_string_buffer(1024)
    arr = np.frombuffer(b, dtype=np.uint8)
    n = lib().dor_detwgt_validate(_ptr(arr) if arr.size else None, arr.size, err, 1024)
    if n < 0:
        raise OracleError(err.value.decode())
    return int(n)


def attention_one(q, keys, values) -> np.ndarray:
    """attention_output_into for one query row over explicit key/value rows."""
    q = np.ascontiguousarray(q, dtype=np.int32)
    keys = np.ascontiguousarray(keys, dtype=np.int32)
    values = np.ascontiguousarray(values, dtype=np.int32)
    out = np.zeros(q.size, dtype=np.int32)
    lib().dor_attention_one(_ptr(q), _ptr(keys), _ptr(values), keys.shape[0], q.size, _ptr(out))
    return out
