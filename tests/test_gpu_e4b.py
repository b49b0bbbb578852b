"""BASELINE configs 2-5 at the E4B stand-in shape, CUDA path vs the CPU det path.

The model is the one bench.py times: the seeded random-init E4B stand-in
(raster-inference_b200/configs/e4b_text_standin.json, seed 20260501, i16
weights), built on the GPU by rdet_open_synthetic.  Configs 3-5 compare
against tests/golden/e4b_fixtures.json, which the CPU oracle wrote for the
same model and inputs (tests/golden/make_e4b_fixtures.py): prefill
commitments (embedding, every layer's output, final hidden states, logits,
KV caches; det_layer_prefill / det_hidden_to_logits, det_kernels.rs:678-821
and :1217-1267), the greedy tokens (argmax_first, det_num/ops.rs:463-478) and
the caches and logits after decoding (det_layer_decode, det_kernels.rs:
866-1133).  Config 2 runs the oracle's GEMV here on the same inputs.  Every
comparison is bit-exact.
"""
import json
import os

import numpy as np
import pytest

import oracle as O  # checker only
from helpers import ROOT, detwgt, load_config, rdet

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

FIXTURES = os.path.join(ROOT, "tests", "golden", "e4b_fixtures.json")
SEED = 20260501


def lcg_ids(n, vocab, seed):
    return detwgt.lcg_token_ids(n, vocab, seed)


@pytest.fixture(scope="module")
def fx():
    with open(FIXTURES) as f:
        return json.load(f)


@pytest.fixture(scope="module")
def cfg():
    return load_config("e4b_text_standin.json")


@pytest.fixture(scope="module")
def model(cfg, fx):
    assert fx["model"]["seed"] == SEED and fx["model"]["width"] == 16
    m = rdet.Model.synthetic(cfg, SEED, width=16, device=0, max_prefill=4096, layer_commitments=True)
    yield m
    m.close()


def own_cache_layers(cfg):
    t = cfg["text_config"]
    return t["num_hidden_layers"] - t["num_kv_shared_layers"]


def check_prefill(seq, rec, cfg):
    L = cfg["text_config"]["num_hidden_layers"]
    assert seq.commitment(rdet.BUF_EMBEDDING) == rec["embedding"]
    assert [seq.commitment(rdet.BUF_LAYER_OUTPUT, l) for l in range(L)] == rec["layer_outputs"]
    assert seq.commitment(rdet.BUF_HIDDEN) == rec["final_hidden"]
    assert seq.commitment(rdet.BUF_LOGITS) == rec["logits"]
    assert seq.commitment(rdet.BUF_KV) == rec["kv"]  # None: the KV-sharing layers own no cache
    assert seq.commitment(rdet.BUF_KV, own_cache_layers(cfg)) == rec["kv_own_layers"]


@pytest.mark.parametrize("length", [512, 2048])
def test_config3_prefill(model, fx, cfg, length):
    rec = fx["config3"][str(length)]
    seq = model.new_sequence(length + 8)
    seq.prefill(lcg_ids(length, cfg["text_config"]["vocab_size"], rec["ids_seed"]))
    check_prefill(seq, rec, cfg)
    assert seq.select() == rec["next_token"]
    seq.free()


def test_config4_prefill_4096_then_256_greedy_tokens(model, fx, cfg):
    rec = fx["config4"]
    seq = model.new_sequence(rec["prompt_tokens"] + len(rec["tokens"]) + 8)
    seq.prefill(lcg_ids(rec["prompt_tokens"], cfg["text_config"]["vocab_size"], rec["ids_seed"]))
    check_prefill(seq, rec["prefill"], cfg)
    assert seq.generate(len(rec["tokens"])) == rec["tokens"]
    assert seq.commitment(rdet.BUF_LOGITS) == rec["final_logits"]
    assert seq.commitment(rdet.BUF_KV) == rec["final_kv"]
    assert seq.commitment(rdet.BUF_KV, own_cache_layers(cfg)) == rec["final_kv_own_layers"]
    seq.free()


def test_config5_ragged_batch_of_64(model, fx, cfg):
    """All 64 ragged sequences decode in one batch (rdet_decode over the
    batch, greedy select per sequence between steps); the oracle's 4-sequence
    subset is checked token for token, with each one's final logits and KV."""
    rec = fx["config5"]
    V = cfg["text_config"]["vocab_size"]
    B, steps = rec["batch"], rec["tokens_per_sequence"]
    lens = [128 + (x % 3969) for x in lcg_ids(B, 1 << 30, rec["lengths_seed"])]
    seqs = [model.new_sequence(n + steps + 8) for n in lens]
    for i, (s, n) in enumerate(zip(seqs, lens)):
        s.prefill(lcg_ids(n, V, SEED + 100 + i))
    out = [[] for _ in range(B)]
    toks = [s.select() for s in seqs]
    for step in range(steps):
        for i, t in enumerate(toks):
            out[i].append(t)
        rdet.decode_batch(model, seqs, toks)
        toks = [s.select() for s in seqs]
    for key, r in rec["sequences"].items():
        i = int(key)
        assert lens[i] == r["length"] and SEED + 100 + i == r["ids_seed"]
        if out[i] != r["tokens"]:  # what went wrong, for the failure message
            lg = seqs[i].read(rdet.BUF_LOGITS)
            first0 = sum(1 for o in out if o and o[0] == 0)
            bad = next(k for k, (a, b) in enumerate(zip(out[i], r["tokens"])) if a != b)
            raise AssertionError(f"sequence {i}: first mismatch at token {bad}; final logits min {lg.min()} "
                                 f"max {lg.max()} distinct {len(np.unique(lg))}; {first0} of {B} sequences "
                                 f"selected token 0 after prefill")
        assert seqs[i].commitment(rdet.BUF_LOGITS) == r["final_logits"], f"sequence {i}"
        assert seqs[i].commitment(rdet.BUF_KV, own_cache_layers(cfg)) == r["final_kv_own_layers"], f"sequence {i}"
    for s in seqs:
        s.free()


def e4b_projection_shapes(cfg):
    t = cfg["text_config"]
    H, F, Hq, kv, d, dg, V, P, L = (t["hidden_size"], t["intermediate_size"], t["num_attention_heads"],
                                    t["num_key_value_heads"], t["head_dim"], t["global_head_dim"],
                                    t["vocab_size"], t["hidden_size_per_layer_input"], t["num_hidden_layers"])
    return {"q": (Hq * d, H), "k": (kv * d, H), "v": (kv * d, H), "o": (H, Hq * d), "gate": (F, H), "up": (F, H),
            "down": (H, F), "q_full": (Hq * dg, H), "o_full": (H, Hq * dg), "ple_gate": (P, H),
            "ple_proj": (H, P), "ple_model_proj": (L * P, H), "lm_head": (V, H)}


def test_config2_gemv_every_e4b_projection(cfg):
    """Config 2: the det GEMV of every E4B projection, lm_head over the full
    vocabulary included, on i16 weights uniform over the format's range and
    N(0,1) activations quantized with f32_to_act."""
    rng = np.random.default_rng(2)
    for n, (name, (rows, cols)) in enumerate(sorted(e4b_projection_shapes(cfg).items())):
        w = rng.integers(-32768, 32768, (rows, cols), dtype=np.int64).astype(np.int16)
        x = detwgt.normal_acts(cols, 1000 + n)
        y = torch.zeros(rows, dtype=torch.int32, device="cuda")
        wd, xd = torch.from_numpy(w).cuda(), torch.from_numpy(x).cuda()
        rdet.det_gemv(xd.data_ptr(), wd.data_ptr(), 16, rows, cols, y.data_ptr())
        torch.cuda.synchronize()
        assert np.array_equal(y.cpu().numpy(), O.gemv(x, w)), name
