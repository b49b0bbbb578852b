"""Oracle vs the reference's det commitment goldens
(testdata/det_commitment_goldens.json, written by src/runtime/det_goldens.rs)
and the reference's checked-in tiny-gemma-dev bundle.  CPU only."""
import hashlib
import json
import tempfile

import pytest

import det_goldens_fixture as fx
import oracle as O
import tiny_gemma_dev
from helpers import detwgt

GOLD = fx.load_goldens()


@pytest.fixture(scope="module", params=["donor_ple", "no_donor_ple"])
def fixture_model(request):
    d = tempfile.mkdtemp()
    fx.write_fixture(d, request.param == "donor_ple")
    return request.param, O.Model(d)


def test_prefill_and_64_decode_steps(fixture_model):
    name, m = fixture_model
    g = GOLD[name]["det"]
    assert O.act_commitment(m.embed(fx.PROMPT_IDS)) == g["prefill"]["embedding"]
    s = m.seq()
    hid, logits, _ = s.prefill(fx.PROMPT_IDS)
    assert O.act_commitment(hid) == g["prefill"]["final_hidden"]
    assert O.vec_commitment(logits) == g["prefill"]["logits"]
    assert s.kv_commitment() == g["prefill"]["kv"]
    toks = []
    for step in range(fx.DECODE_TOKENS):
        t = O.argmax_first(logits)
        toks.append(t)
        h, logits, _ = s.decode(t)
        gs = g["decode_steps"][step]
        assert (t, O.act_commitment(h), O.vec_commitment(logits), s.kv_commitment()) == \
            (gs["token"], gs["activation"], gs["logits"], gs["kv"]), step
    e2e = g["end_to_end"]
    assert toks == e2e["generated_token_ids"]
    assert hashlib.sha256(json.dumps(toks, separators=(",", ":")).encode()).hexdigest() == e2e["generated_token_ids_sha256"]


def test_first_step_layer_outputs(fixture_model):
    name, m = fixture_model
    g = GOLD[name]["det"]
    s = m.seq()
    _, logits, _ = s.prefill(fx.PROMPT_IDS)
    _, _, layer_hashes = s.decode(O.argmax_first(logits))
    assert layer_hashes == [x["layer_output"] for x in g["first_step_layers"]]


def test_thread_count_invariance(fixture_model):
    # tests/schedule_parity.rs: identical commitments for every thread count
    name, m = fixture_model
    out = []
    for t in (1, 3, 8):
        O.set_threads(t)
        s = m.seq()
        hid, logits, lh = s.prefill(fx.PROMPT_IDS)
        out.append((O.act_commitment(hid), O.vec_commitment(logits), tuple(lh)))
    O.set_threads(1)
    assert out[0] == out[1] == out[2]


def test_tiny_gemma_dev_bundle_matches_reference_bytes():
    b = detwgt.encode(tiny_gemma_dev.tensors())
    assert hashlib.sha256(b).hexdigest() == tiny_gemma_dev.reference_record()["model_detwgt_sha256"]


def test_tiny_gemma_dev_config1_runs():
    d = tiny_gemma_dev.write_bundle(tempfile.mkdtemp(), detwgt.encode)
    m = O.Model(d)
    assert m.layers[2]["donor"] == 0 and m.layers[3]["donor"] == 1 and m.layers[1]["k_eq_v"] == 1
    ids = tiny_gemma_dev.lcg_token_ids(16, 280, 0)
    s = m.seq()
    _, logits, _ = s.prefill(ids)
    for _ in range(8):
        s.decode(O.argmax_first(logits))
    assert s.position == 24


def test_synthetic_generator_matches_artifact():
    # the oracle's in-memory synthetic model equals the detwgt artifact that
    # raster-inference_b200/detwgt.py writes for the same (config, seed, width)
    from helpers import mini_config, write_model
    for width, cfg in ((16, mini_config()), (32, mini_config(num_kv_shared_layers=0, tie_word_embeddings=False))):
        d = write_model(cfg, seed=99, width=width)
        a = O.Model(d)
        b = O.Model(None, synthetic=(cfg, 99, width))
        ids = [3, 1, 4, 1, 5, 9, 2, 6]
        _, la, ha = a.seq().prefill(ids)
        _, lb, hb = b.seq().prefill(ids)
        assert (la == lb).all() and ha == hb
