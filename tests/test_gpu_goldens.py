"""The reference's det commitment goldens reproduced by the CUDA path
(testdata/det_commitment_goldens.json from src/runtime/det_goldens.rs):
embedding, prefill final hidden / logits / KV, every per-layer output of the
first decode step, 64 decode steps (token, activation, logits, KV) and the
end-to-end generated ids."""
import hashlib
import json
import tempfile

import pytest

import det_goldens_fixture as fx
from helpers import rdet

pytestmark = pytest.mark.gpu
GOLD = fx.load_goldens()


@pytest.fixture(scope="module", params=["donor_ple", "no_donor_ple"])
def model(request):
    d = tempfile.mkdtemp()
    fx.write_fixture(d, request.param == "donor_ple")
    m = rdet.Model.open(d, max_prefill=64, layer_commitments=True)
    yield request.param, m
    m.close()


def test_prefill_matches_goldens(model):
    name, m = model
    g = GOLD[name]["det"]["prefill"]
    s = m.new_sequence(128)
    s.prefill(fx.PROMPT_IDS)
    assert s.commitment(rdet.BUF_EMBEDDING) == g["embedding"]
    assert s.commitment(rdet.BUF_HIDDEN) == g["final_hidden"]
    assert s.commitment(rdet.BUF_LOGITS) == g["logits"]
    assert s.commitment(rdet.BUF_KV) == g["kv"]


def test_decode_steps_match_goldens(model):
    name, m = model
    g = GOLD[name]["det"]
    s = m.new_sequence(128)
    s.prefill(fx.PROMPT_IDS)
    toks = []
    for step in range(fx.DECODE_TOKENS):
        t = s.select()
        toks.append(t)
        s.decode(t)
        if step == 0:
            assert [s.commitment(rdet.BUF_LAYER_OUTPUT, l) for l in range(4)] == \
                [x["layer_output"] for x in g["first_step_layers"]]
        gs = g["decode_steps"][step]
        got = (t, s.commitment(rdet.BUF_HIDDEN), s.commitment(rdet.BUF_LOGITS), s.commitment(rdet.BUF_KV))
        assert got == (gs["token"], gs["activation"], gs["logits"], gs["kv"]), step
    assert toks == g["end_to_end"]["generated_token_ids"]


def test_generate_graph_matches_goldens(model):
    name, m = model
    e2e = GOLD[name]["det"]["end_to_end"]
    s = m.new_sequence(128)
    s.prefill(fx.PROMPT_IDS)
    toks = s.generate(fx.DECODE_TOKENS)
    assert toks == e2e["generated_token_ids"]
    assert hashlib.sha256(json.dumps(toks, separators=(",", ":")).encode()).hexdigest() == \
        e2e["generated_token_ids_sha256"]
    assert s.commitment(rdet.BUF_KV) == GOLD[name]["det"]["decode_steps"][-1]["kv"]


def test_routine_granular_first_step_kv(model):
    # decode_layer_range with width 1 (det_goldens.rs:187-236): the KV
    # commitment over the effective caches after each layer
    name, m = model
    g = GOLD[name]["det"]
    s = m.new_sequence(128)
    s.prefill(fx.PROMPT_IDS)
    t = s.select()
    s.decode_begin(t)
    for l in range(4):
        s.decode_range(l, l + 1)
    s.decode_finalize()
    assert s.commitment(rdet.BUF_KV) == g["first_step_layers"][-1]["kv"]
