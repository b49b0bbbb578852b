"""Shared test helpers: imports of the product package and the oracle, and
the synthetic model configurations used by the parity tests."""
import copy
import importlib
import json
import os
import tempfile

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
rdet = importlib.import_module("raster-inference_b200")
detwgt = importlib.import_module("raster-inference_b200.detwgt")
import oracle as O  # noqa: E402  (test infrastructure only)


def load_config(name: str) -> dict:
    with open(os.path.join(ROOT, "raster-inference_b200", "configs", name)) as f:
        return json.load(f)


def mini_config(**over) -> dict:
    """A small Gemma-4-shaped config exercising every det feature."""
    t = {
        "enable_moe_block": False, "hidden_activation": "gelu_pytorch_tanh",
        "hidden_size": 64, "intermediate_size": 128, "num_hidden_layers": 6,
        "num_attention_heads": 4, "num_key_value_heads": 2, "head_dim": 16, "global_head_dim": 32,
        "layer_types": ["sliding_attention", "sliding_attention", "full_attention",
                        "sliding_attention", "sliding_attention", "full_attention"],
        "sliding_window": 8, "vocab_size": 97, "hidden_size_per_layer_input": 8,
        "num_kv_shared_layers": 2, "rms_norm_eps": 1e-6, "final_logit_softcapping": 30.0,
        "rope_parameters": {"full_attention": {"partial_rotary_factor": 0.25, "rope_theta": 1000000.0},
                            "sliding_attention": {"rope_theta": 10000.0}},
        "tie_word_embeddings": True,
    }
    t.update(over)
    return {"text_config": t}


def write_model(cfg: dict, seed: int, width: int = 16) -> str:
    d = tempfile.mkdtemp(prefix="rdet-model-")
    detwgt.write_synthetic_model(d, cfg, seed, width)
    return d


def lcg_ids(n, vocab, seed):
    from tiny_gemma_dev import lcg_token_ids
    return lcg_token_ids(n, vocab, seed)
