"""Checkpoint-trace parity on the GPU: the CUDA path, through the C ABI's
routines and commitments (rdet_prefill / rdet_select / rdet_decode /
rdet_commitment), reproduces the reference's golden trace artifacts
native-det-full and native-det-terminal entry for entry."""
import importlib
import json
import os
import tempfile

import pytest

import tiny_gemma_dev
from helpers import detwgt, rdet

trace = importlib.import_module("raster-inference_b200.trace")

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = json.load(open(os.path.join(HERE, "golden", "det_trace_goldens.json")))


def run_trace(terminal=None):
    d = tiny_gemma_dev.write_bundle(tempfile.mkdtemp(), detwgt.encode)
    m = rdet.Model.open(d, max_prefill=32, layer_commitments=True)
    seq = m.new_sequence(64)
    return trace.run(trace.SeqBackend(seq), GOLD["prompt_token_ids"], num_layers=m.L,
                     max_new_tokens=GOLD["max_new_tokens"], prompt_text=GOLD["prompt_text"],
                     temperature=GOLD["temperature"], detokenize=lambda ids: GOLD["generated_text"],
                     terminal=terminal)


def test_cuda_path_reproduces_native_det_full():
    tr, gen = run_trace()
    assert gen == GOLD["generated_token_ids"]
    assert [list(e) for e in tr.entries] == GOLD["native-det-full"]


def test_cuda_path_from_prompt_text_reproduces_native_det_full():
    # the request path: prompt bytes -> prompt.prepare (the bundle's chat
    # template and tokenizer) -> the CUDA path -> output.finalize
    prompt = importlib.import_module("raster-inference_b200.prompt")
    d = tiny_gemma_dev.write_bundle(tempfile.mkdtemp(), detwgt.encode)
    m = rdet.Model.open(d, max_prefill=32, layer_commitments=True)
    seq = m.new_sequence(64)
    tr, gen = trace.run_request(trace.SeqBackend(seq), prompt.PromptPreparer(os.path.join(HERE, "golden",
                                                                                          "tiny_gemma_dev_text")),
                                GOLD["prompt_text"].encode("utf-8"), num_layers=m.L,
                                max_new_tokens=GOLD["max_new_tokens"], temperature=GOLD["temperature"])
    assert gen == GOLD["generated_token_ids"]
    assert [list(e) for e in tr.entries] == GOLD["native-det-full"]


def test_cuda_path_reproduces_native_det_terminal():
    tr, _ = run_trace(terminal=GOLD["terminal"])
    assert [list(e) for e in tr.entries] == GOLD["native-det-terminal"]


@pytest.mark.parametrize("donor", [False, True], ids=["no_donor", "donor"])
def test_kv_prefix_commitments_match_single_calls(donor):
    # rdet_kv_prefix_commitments against n calls of rdet_commitment(KV, p):
    # after prefill and after decode steps that trim the sliding caches
    # (window 4 < 6 prompt + 5 generated rows); a KV-sharing model gives None
    # from its first shared layer on
    import det_goldens_fixture as fx
    d = tempfile.mkdtemp()
    fx.write_fixture(d, donor=donor)
    m = rdet.Model.open(d, max_prefill=16)
    s = m.new_sequence(64)
    s.prefill(fx.PROMPT_IDS)
    for steps in (0, 5):
        s.generate(steps)
        want = [s.commitment(rdet.BUF_KV, p) for p in range(1, m.L + 1)]
        assert s.kv_prefix_commitments(m.L) == want
        assert s.kv_prefix_commitments(2) == want[:2]
        assert (want[-1] is None) == donor and want[0] is not None
    m.close()
