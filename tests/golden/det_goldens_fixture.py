"""Rebuilds the reference's two in-code det golden fixtures as model dirs.

Restates casettek/raster-inference src/runtime/det_goldens.rs:288-514: a
4-layer Gemma-4 model (H=4, d=2, 2 heads / 1 KV head, layers [s,f,s,f],
FF=8, V=9, PLE=2, sliding window 4, untied lm_head, no rope_parameters),
weights drawn from the LCG ``s = s*6364136223846793005 + 1442695040888963407``
(seed 0x5eed5eed5eed5eed) as ``((s>>33) % 33 - 16) / 64`` and norm gains as
``1 + w/4``, every value exactly representable, so ``f32_to_wgt`` is exact:
weight bits = bucket*1024, gain bits = 65536 + bucket*256.  Fixture
``donor_ple`` sets num_kv_shared_layers=1, ``no_donor_ple`` sets 0.  The
prompt "w0 w1 w2 w3 w4 w5" tokenizes to ids [0..5] with the fixture's
WordLevel vocab (det_goldens.rs:269-282); 64 greedy decode tokens follow.
"""
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", ".."))

import importlib

detwgt = importlib.import_module("raster-inference_b200.detwgt")

HIDDEN, HEAD_DIM, NUM_HEADS, NUM_KV_HEADS, LAYERS, FF, VOCAB, PLE_DIM = 4, 2, 2, 1, 4, 8, 9, 2
PROMPT_IDS = [0, 1, 2, 3, 4, 5]
DECODE_TOKENS = 64


class _Lcg:
    def __init__(self, seed):
        self.s = seed

    def _bucket(self):
        self.s = (self.s * 6364136223846793005 + 1442695040888963407) & 0xFFFFFFFFFFFFFFFF
        return ((self.s >> 33) % 33) - 16

    def weights(self, n):
        return [self._bucket() * 1024 for _ in range(n)]

    def norms(self, n):
        return [65536 + self._bucket() * 256 for _ in range(n)]


def fixture_config(donor: bool) -> dict:
    return {"text_config": {
        "enable_moe_block": False, "head_dim": HEAD_DIM, "hidden_activation": "gelu_pytorch_tanh",
        "hidden_size": HIDDEN, "hidden_size_per_layer_input": PLE_DIM,
        "layer_types": ["sliding_attention", "full_attention", "sliding_attention", "full_attention"],
        "num_attention_heads": NUM_HEADS, "num_hidden_layers": LAYERS, "num_key_value_heads": NUM_KV_HEADS,
        "num_kv_shared_layers": 1 if donor else 0, "rms_norm_eps": 0.000001, "sliding_window": 4,
        "tie_word_embeddings": False, "vocab_size": VOCAB, "vocab_size_per_layer_input": VOCAB}}


def fixture_tensors():
    import numpy as np
    rng = _Lcg(0x5EED5EED5EED5EED)
    out = []

    def push(name, shape, vals):
        out.append((name, shape, np.array(vals, dtype=np.int32)))

    push("model.language_model.embed_tokens.weight", (VOCAB, HIDDEN), rng.weights(VOCAB * HIDDEN))
    for l in range(LAYERS):
        p = f"model.language_model.layers.{l}"
        push(f"{p}.self_attn.q_proj.weight", (NUM_HEADS * HEAD_DIM, HIDDEN), rng.weights(NUM_HEADS * HEAD_DIM * HIDDEN))
        push(f"{p}.self_attn.k_proj.weight", (NUM_KV_HEADS * HEAD_DIM, HIDDEN), rng.weights(NUM_KV_HEADS * HEAD_DIM * HIDDEN))
        push(f"{p}.self_attn.v_proj.weight", (NUM_KV_HEADS * HEAD_DIM, HIDDEN), rng.weights(NUM_KV_HEADS * HEAD_DIM * HIDDEN))
        push(f"{p}.self_attn.o_proj.weight", (HIDDEN, NUM_HEADS * HEAD_DIM), rng.weights(HIDDEN * NUM_HEADS * HEAD_DIM))
        push(f"{p}.self_attn.q_norm.weight", (HEAD_DIM,), rng.norms(HEAD_DIM))
        push(f"{p}.self_attn.k_norm.weight", (HEAD_DIM,), rng.norms(HEAD_DIM))
        for n in ("input_layernorm", "post_attention_layernorm", "pre_feedforward_layernorm", "post_feedforward_layernorm"):
            push(f"{p}.{n}.weight", (HIDDEN,), rng.norms(HIDDEN))
        push(f"{p}.mlp.gate_proj.weight", (FF, HIDDEN), rng.weights(FF * HIDDEN))
        push(f"{p}.mlp.up_proj.weight", (FF, HIDDEN), rng.weights(FF * HIDDEN))
        push(f"{p}.mlp.down_proj.weight", (HIDDEN, FF), rng.weights(HIDDEN * FF))
        push(f"{p}.per_layer_input_gate.weight", (PLE_DIM, HIDDEN), rng.weights(PLE_DIM * HIDDEN))
        push(f"{p}.per_layer_projection.weight", (HIDDEN, PLE_DIM), rng.weights(HIDDEN * PLE_DIM))
        push(f"{p}.post_per_layer_input_norm.weight", (HIDDEN,), rng.norms(HIDDEN))
    push("model.language_model.embed_tokens_per_layer.weight", (VOCAB, LAYERS * PLE_DIM), rng.weights(VOCAB * LAYERS * PLE_DIM))
    push("model.language_model.per_layer_model_projection.weight", (LAYERS * PLE_DIM, HIDDEN), rng.weights(LAYERS * PLE_DIM * HIDDEN))
    push("model.language_model.per_layer_projection_norm.weight", (PLE_DIM,), rng.norms(PLE_DIM))
    push("model.language_model.norm.weight", (HIDDEN,), rng.norms(HIDDEN))
    push("model.language_model.lm_head.weight", (VOCAB, HIDDEN), rng.weights(VOCAB * HIDDEN))
    return out


def write_fixture(model_dir: str, donor: bool) -> str:
    os.makedirs(model_dir, exist_ok=True)
    with open(os.path.join(model_dir, "config.json"), "w") as f:
        json.dump(fixture_config(donor), f, indent=1)
    with open(os.path.join(model_dir, "model.detwgt"), "wb") as f:
        f.write(detwgt.encode(fixture_tensors()))
    return model_dir


def load_goldens() -> dict:
    with open(os.path.join(HERE, "det_commitment_goldens.json")) as f:
        return json.load(f)
