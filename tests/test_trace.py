"""Checkpoint-trace parity on the CPU: the trace builder (raster-inference_b200
/trace.py) driven by the oracle reproduces the reference's own golden trace
artifacts native-det-full and native-det-terminal (tests/golden_traces.rs),
entry for entry."""
import importlib
import json
import os
import struct
import hashlib
import tempfile

import numpy as np
import pytest

import oracle as O
import tiny_gemma_dev
from helpers import detwgt

trace = importlib.import_module("raster-inference_b200.trace")

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = json.load(open(os.path.join(HERE, "golden", "det_trace_goldens.json")))


class OracleBackend:
    """The oracle as a trace backend (test infrastructure)."""

    def __init__(self, model_dir):
        self.m = O.Model(model_dir, threads=4)
        self.s = self.m.seq()

    def prefill(self, ids):
        self.emb = self.m.embed(ids)
        self.hidden, self.logits, self.lh = self.s.prefill(ids)

    def select(self):
        return O.argmax_first(self.logits)

    def decode(self, token):
        h, self.logits, self.lh = self.s.decode(token)
        self.hidden = h.reshape(1, -1)

    def embedding_commitment(self):
        return O.act_commitment(self.emb)

    def hidden_commitment(self):
        return O.act_commitment(self.hidden)

    def logits_commitment(self):
        return O.vec_commitment(self.logits)

    def layer_output_commitment(self, layer):
        return self.lh[layer]

    def kv_commitment(self, layers):
        # build_det_kv_cache_commitment over the first `layers` caches
        # (transformer_kernels.rs:1460-1482); None when one has no det data
        h = hashlib.sha256()
        h.update(b"raster-det-num-kv-cache-v1")
        h.update(struct.pack("<Q", layers))
        for layer in range(layers):
            heads = self.m.layers[layer]["kv_heads"]
            rows = [[self.s.kv_rows(layer, hd, kind) for hd in range(heads)] for kind in (0, 1)]
            if any(r is None for rk in rows for r in rk):
                return None
            h.update(struct.pack("<Q", heads))
            for kind, rk in zip((b"k", b"v"), rows):
                h.update(kind)
                h.update(struct.pack("<Q", heads))
                for r in rk:
                    h.update(struct.pack("<Q", r.shape[0]))
                    for row in r:
                        h.update(struct.pack("<Q", row.size))
                        h.update(row.astype("<i4").tobytes())
        return h.hexdigest()


@pytest.fixture(scope="module")
def bundle():
    return tiny_gemma_dev.write_bundle(tempfile.mkdtemp(), detwgt.encode)


def run_trace(backend, terminal=None):
    return trace.run(backend, GOLD["prompt_token_ids"], num_layers=4, max_new_tokens=GOLD["max_new_tokens"],
                     prompt_text=GOLD["prompt_text"], temperature=GOLD["temperature"],
                     detokenize=lambda ids: GOLD["generated_text"], terminal=terminal)


def test_serde_json_bytes():
    # serde_json::to_vec of the shapes the payloads use
    assert trace.to_json_bytes([9, 10, 11]) == b"[9,10,11]"
    assert trace.to_json_bytes({"b": None, "a": 1.0, "c": "x\ny"}) == b'{"a":1.0,"b":null,"c":"x\\ny"}'
    assert trace.sha256_hex([1, 1]) == hashlib.sha256(b"[1,1]").hexdigest()


def test_oracle_reproduces_native_det_full(bundle):
    tr, gen = run_trace(OracleBackend(bundle))
    assert gen == GOLD["generated_token_ids"]
    assert [list(e) for e in tr.entries] == GOLD["native-det-full"]


def test_oracle_reproduces_native_det_terminal(bundle):
    tr, _ = run_trace(OracleBackend(bundle), terminal=GOLD["terminal"])
    assert [list(e) for e in tr.entries] == GOLD["native-det-terminal"]


def test_a_changed_commitment_changes_its_entry(bundle):
    # plant a mistake in the oracle backend: the entry that carries the
    # layer-2 output commitment (and only entries after it) must differ
    class Planted(OracleBackend):
        def layer_output_commitment(self, layer):
            c = super().layer_output_commitment(layer)
            return c if layer != 2 else "0" * 64

    tr, _ = run_trace(Planted(bundle))
    got = [list(e) for e in tr.entries]
    names = [n for n, _ in GOLD["native-det-full"]]
    first_bad = names.index("prefill.range", 3 + 2 * 2)
    assert got[:first_bad] == GOLD["native-det-full"][:first_bad]
    assert got[first_bad] != GOLD["native-det-full"][first_bad]
