"""detwgt v2 writer and seeded synthetic Gemma-4 det models.

The byte layout restates the reference encoder
(casettek/raster-inference src/shared/numerics/det_num/artifact.rs:61-206,
docs/plans/DETWGT_V2_FORMAT.md): a 24-byte file header, then per tensor
``name_len u32 | name | rank u32 | dims u64* | element_count u64 |
element_width u32 (16|32) | payload_len u64 | max_row_mass u64 | zero padding
to a 64-byte file offset | payload (LE i16 or i32)``.  Width policy ``auto``
stores a tensor as i16 exactly when every value fits i16.

Synthetic models ("random-init weights of the named shapes") use a
counter-based generator so any element can be produced independently on the
host (this module) or on the GPU (``rdet_open_synthetic`` in the C ABI) with
identical bits:

    key = fnv1a64(tensor_name) ^ seed
    z   = splitmix64_mix(key + (i + 1) * 0x9E3779B97F4A7C15)      (mod 2^64)

    rank-2, width 16:  value = (z >> 48) - 32768        uniform over i16
    rank-2, width 32:  value = (z mod (2B + 1)) - B,  B = (2^31 - 1) // cols
    rank-1 (gains):    value = 32768 + (z >> 48)        Q16.16 in [0.5, 1.5)

The i32 bound keeps every row mass below 2^31, the loader's overflow check
(src/shared/model/gemma/io.rs:341-347).
"""
from __future__ import annotations

import json
import os
import struct

import numpy as np

MAGIC = b"DNWGTV0\0"
FORMAT_VERSION = 2
SPEC_VERSION = 1
ALIGN = 64
GOLDEN = np.uint64(0x9E3779B97F4A7C15)


def fnv1a64(s: str) -> int:
    h = 0xCBF29CE484222325
    for b in s.encode():
        h ^= b
        h = (h * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    return h


def _mix(z: np.ndarray) -> np.ndarray:
    z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
    z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    return z ^ (z >> np.uint64(31))


def synth_values(name: str, shape, seed: int, width: int) -> np.ndarray:
    """Seeded values of one tensor as canonical i32 bit patterns."""
    n = int(np.prod(shape))
    key = np.uint64((fnv1a64(name) ^ seed) & 0xFFFFFFFFFFFFFFFF)
    with np.errstate(over="ignore"):
        idx = np.arange(1, n + 1, dtype=np.uint64)
        z = _mix(key + idx * GOLDEN)
    if len(shape) == 1:
        return (np.int64(32768) + (z >> np.uint64(48)).astype(np.int64)).astype(np.int32)
    if width == 16:
        return ((z >> np.uint64(48)).astype(np.int64) - 32768).astype(np.int32)
    cols = int(shape[-1])
    bound = (2 ** 31 - 1) // cols
    return ((z % np.uint64(2 * bound + 1)).astype(np.int64) - bound).astype(np.int32)


def max_row_mass(shape, bits: np.ndarray) -> int:
    row = int(shape[-1]) if len(shape) else 1
    row = max(row, 1)
    a = np.abs(bits.astype(np.int64)).reshape(-1, row)
    return int(a.sum(axis=1).max()) if a.size else 0


def write(f, tensors, count: int, policy: str = "auto") -> int:
    """Stream ``count`` tensors ``(name, shape, int32 array)`` (any iterable,
    consumed one at a time; a fourth element, when present, is the tensor's
    max row mass already computed) to the binary file ``f`` as a detwgt v2
    artifact; returns the bytes written."""
    head = MAGIC + struct.pack("<IIQ", FORMAT_VERSION, SPEC_VERSION, count)
    f.write(head)
    written, n = len(head), 0
    for item in tensors:
        name, shape, bits = item[:3]
        bits = np.ascontiguousarray(bits, dtype=np.int32).ravel()
        if int(np.prod(shape)) != bits.size:
            raise ValueError(f"tensor `{name}` has {bits.size} values but shape product {int(np.prod(shape))}")
        fits16 = bits.size == 0 or (bits.min() >= -32768 and bits.max() <= 32767)
        width = 16 if (policy == "auto" and fits16) else 32
        nb = name.encode()
        rec = bytearray(struct.pack("<I", len(nb)) + nb + struct.pack("<I", len(shape)))
        for d in shape:
            rec += struct.pack("<Q", int(d))
        mass = item[3] if len(item) > 3 else max_row_mass(shape, bits)
        rec += struct.pack("<QIQQ", bits.size, width, bits.size * width // 8, mass)
        rec += b"\0" * ((ALIGN - (written + len(rec)) % ALIGN) % ALIGN)
        f.write(rec)
        payload = (bits.astype("<i2") if width == 16 else bits.astype("<i4")).tobytes()
        f.write(payload)
        written += len(rec) + len(payload)
        n += 1
    if n != count:
        raise ValueError(f"{n} tensors written, {count} declared")
    return written


def encode(tensors, policy: str = "auto") -> bytes:
    """Encode ``[(name, shape, int32 array)]`` as a detwgt v2 artifact."""
    import io
    buf = io.BytesIO()
    write(buf, tensors, len(tensors), policy)
    return buf.getvalue()


def layer_shapes(cfg: dict):
    """Tensor names and shapes of a Gemma-4 det text model (io.rs:1896-2045)."""
    t = cfg.get("text_config", cfg)
    H, V, L = t["hidden_size"], t["vocab_size"], t["num_hidden_layers"]
    Hq, kv, d = t["num_attention_heads"], t["num_key_value_heads"], t["head_dim"]
    dg = t.get("global_head_dim") or d
    P = t.get("hidden_size_per_layer_input") or 0
    keqv = bool(t.get("attention_k_eq_v") or False)
    gkv = t.get("num_global_key_value_heads") or kv
    F = t["intermediate_size"]
    ple_vocab = t.get("vocab_size_per_layer_input") or V
    out = [("model.language_model.embed_tokens.weight", (V, H))]
    for l, lt in enumerate(t["layer_types"]):
        sl = lt == "sliding_attention"
        hd = d if sl else dg
        nkv = kv if sl else (gkv if keqv else kv)
        p = f"model.language_model.layers.{l}"
        out += [(f"{p}.self_attn.q_proj.weight", (Hq * hd, H)),
                (f"{p}.self_attn.k_proj.weight", (nkv * hd, H))]
        if sl or not keqv:
            out.append((f"{p}.self_attn.v_proj.weight", (nkv * hd, H)))
        out += [(f"{p}.self_attn.o_proj.weight", (H, Hq * hd)),
                (f"{p}.self_attn.q_norm.weight", (hd,)),
                (f"{p}.self_attn.k_norm.weight", (hd,))]
        for n in ("input_layernorm", "post_attention_layernorm", "pre_feedforward_layernorm",
                  "post_feedforward_layernorm"):
            out.append((f"{p}.{n}.weight", (H,)))
        out += [(f"{p}.mlp.gate_proj.weight", (F, H)), (f"{p}.mlp.up_proj.weight", (F, H)),
                (f"{p}.mlp.down_proj.weight", (H, F))]
        if P > 0:
            out += [(f"{p}.per_layer_input_gate.weight", (P, H)), (f"{p}.per_layer_projection.weight", (H, P)),
                    (f"{p}.post_per_layer_input_norm.weight", (H,))]
        if t.get("_synthetic_layer_scalar", True):
            out.append((f"{p}.layer_scalar", (1,)))
    if P > 0:
        out += [("model.language_model.embed_tokens_per_layer.weight", (ple_vocab, L * P)),
                ("model.language_model.per_layer_model_projection.weight", (L * P, H)),
                ("model.language_model.per_layer_projection_norm.weight", (P,))]
    out.append(("model.language_model.norm.weight", (H,)))
    tie = t.get("tie_word_embeddings")
    if tie is not None and not tie:
        out.append(("model.language_model.lm_head.weight", (V, H)))
    return out


def write_synthetic_model(model_dir: str, cfg: dict, seed: int, width: int = 16, policy: str = "auto") -> str:
    """Write config.json + model.detwgt for a seeded synthetic model."""
    os.makedirs(model_dir, exist_ok=True)
    tensors = [(n, s, synth_values(n, s, seed, width)) for n, s in layer_shapes(cfg)]
    with open(os.path.join(model_dir, "config.json"), "w") as f:
        json.dump(cfg, f, indent=1)
    with open(os.path.join(model_dir, "model.detwgt"), "wb") as f:
        f.write(encode(tensors, policy))
    return model_dir


# ---------------------------------------------------------------------------
# synthetic inputs of the benchmarks (the seeded token ids and activations that
# bench.py and the E4B-shape parity tests share)
# ---------------------------------------------------------------------------
def lcg_draws(n: int, seed: int) -> list[int]:
    """The reference fixture's LCG (det_goldens.rs:348-356): s <- s *
    6364136223846793005 + 1442695040888963407 mod 2^64, draw = s >> 33."""
    s, out = seed, []
    for _ in range(n):
        s = (s * 6364136223846793005 + 1442695040888963407) & 0xFFFFFFFFFFFFFFFF
        out.append(s >> 33)
    return out


def lcg_token_ids(n: int, vocab: int, seed: int) -> list[int]:
    return [d % vocab for d in lcg_draws(n, seed)]


def normal_f32(n: int, seed: int) -> np.ndarray:
    """n draws of N(0, 1) as float32: Box-Muller on pairs of LCG draws
    reduced to 30 bits, u1 in (0, 1], u2 in [0, 1)."""
    u = np.array([d % (1 << 30) for d in lcg_draws(2 * ((n + 1) // 2), seed)], dtype=np.float64)
    u1 = (u[0::2] + 1.0) / float(1 << 30)
    u2 = u[1::2] / float(1 << 30)
    r = np.sqrt(-2.0 * np.log(u1))
    z = np.empty(u1.size * 2, dtype=np.float64)
    z[0::2] = r * np.cos(2.0 * np.pi * u2)
    z[1::2] = r * np.sin(2.0 * np.pi * u2)
    return z[:n].astype(np.float32)


def f32_to_act(x: np.ndarray) -> np.ndarray:
    """det_num f32_to_act (convert.rs:52-57, :82-93) for finite float32
    values: round half to even of x * 2^16, saturated to i32.  x * 2^16 is
    exact in float64 (an exponent shift of a float32), and rint rounds half
    to even."""
    q = np.rint(np.asarray(x, dtype=np.float32).astype(np.float64) * 65536.0)
    return np.clip(q, -2.0**31, 2.0**31 - 1).astype(np.int32)


def normal_acts(n: int, seed: int) -> np.ndarray:
    """Activations of the GEMV microbenchmark: N(0, 1) quantized with f32_to_act."""
    return f32_to_act(normal_f32(n, seed))
