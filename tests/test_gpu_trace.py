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


def test_cuda_path_reproduces_native_det_terminal():
    tr, _ = run_trace(terminal=GOLD["terminal"])
    assert [list(e) for e in tr.entries] == GOLD["native-det-terminal"]
