"""Checkpoint trace of a deterministic generation run.

The reference's trace artifact is a list of ``{checkpoint_id: sha256}`` entries
in emission order, each hash being SHA-256 of ``serde_json::to_vec(payload)``
(casettek/raster-inference ``src/runtime/trace.rs:266-288`` and ``:425-430``).
This module rebuilds that list for the native deterministic executor from the
commitments this library computes, so a run here can be checked entry for
entry against a trace the reference wrote (its ``tests/goldens/native-det-*``).

Payloads restate the deterministic-mode builders field for field:

=========================== ==========================================================
checkpoint                  reference builder
=========================== ==========================================================
prompt.prepare              ``src/runtime/executors/native.rs:82-91``
input.embedding             ``src/routines/input_embedding/mod.rs:88-132``
prefill.prepare_aux         ``src/routines/prefill_prepare_aux/mod.rs:174-206``
prefill.range               ``src/routines/prefill_range/mod.rs:36-81`` (default range
                            width ``usize::MAX``: one range per layer)
prefill.range_finalize      ``src/routines/prefill_range_finalize/mod.rs:17-72``
prefill.finalize            ``src/routines/prefill_finalize/native/tiles.rs:68-92``
decode.select_token         ``src/routines/decode_select_token/mod.rs:30-47, 362-397``
decode.layer_range          ``src/routines/decode_layer_range/mod.rs:553-664`` (default
                            width: all layers in one range)
decode.transition_finalize  ``src/routines/decode_transition_finalize/mod.rs:67-96``
output.finalize             ``src/routines/output_finalize/mod.rs:20-45``
=========================== ==========================================================

``serde_json`` writes compact JSON with object keys in sorted order (its
default map is a BTreeMap) and non-ASCII text unescaped; ``json.dumps`` with
``sort_keys``, compact separators and ``ensure_ascii=False`` produces the same
bytes for the integers, strings, nulls and the ``1.0``-style floats these
payloads hold.
"""
from __future__ import annotations

import hashlib
import json
from typing import Callable, Optional, Protocol, Sequence

DET = "deterministic"


def to_json_bytes(value) -> bytes:
    """serde_json::to_vec of a serde_json::Value: compact, keys sorted."""
    return json.dumps(value, separators=(",", ":"), sort_keys=True, ensure_ascii=False).encode("utf-8")


def sha256_hex(value) -> str:
    """trace.rs:425-430 sha256_hex (also build_prompt_commitment and
    build_output_decode_commitment for token id lists)."""
    return hashlib.sha256(to_json_bytes(value)).hexdigest()


class Backend(Protocol):
    """What a run needs from an executor: the three routines and the det
    commitments of include/rdet.h (rdet_commitment)."""

    def prefill(self, token_ids: Sequence[int]) -> None: ...
    def select(self) -> int: ...
    def decode(self, token: int) -> None: ...
    def embedding_commitment(self) -> str: ...
    def hidden_commitment(self) -> str: ...
    def logits_commitment(self) -> str: ...
    def layer_output_commitment(self, layer: int) -> str: ...
    def kv_commitment(self, layers: int) -> Optional[str]: ...


class Trace:
    """Checkpoint entries in emission order."""

    def __init__(self):
        self.entries: list[tuple[str, str]] = []

    def add(self, name: str, payload) -> None:
        self.entries.append((name, sha256_hex(payload)))

    def artifact(self) -> list[dict]:
        """The entries as the reference's artifact holds them."""
        return [{name: digest} for name, digest in self.entries]


def run(backend: Backend, prompt_token_ids: Sequence[int], num_layers: int, max_new_tokens: int,
        prompt_text: Optional[str] = None, temperature: float = 1.0,
        detokenize: Optional[Callable[[list], str]] = None, terminal: Optional[str] = None):
    """Prefill, then greedy decode until max_new_tokens tokens are generated,
    recording every committed checkpoint.  Returns (trace, generated ids).

    prompt_text: when given, the prompt.prepare entry is recorded (the
    reference emits it when its executor holds the tokenizer source; the
    sampling block is {max_new_tokens, temperature, top_k: null, top_p: null}).
    detokenize: turns the generated ids into text for output.finalize
    (skipping special tokens, output_finalize/native/tiles.rs:5-13); without
    it output.finalize is not recorded.
    terminal: stop after the first entry of this checkpoint, like the
    reference's terminal checkpoint control."""
    ids = [int(t) for t in prompt_token_ids]
    S, L = len(ids), num_layers
    tr = Trace()

    def add(name, payload) -> bool:
        tr.add(name, payload)
        return terminal is not None and name == terminal

    ids_sha = sha256_hex(ids)
    if prompt_text is not None:
        sampling = {"max_new_tokens": max_new_tokens, "temperature": float(temperature), "top_k": None,
                    "top_p": None}
        if add("prompt.prepare", {"prompt_text": prompt_text, "prompt_token_ids": ids,
                                  "prompt_token_ids_sha256": ids_sha, "sampling": sampling}):
            return tr, []
    backend.prefill(ids)
    emb = backend.embedding_commitment()
    if add("input.embedding", {"det_embedded_prompt_activations_sha256": emb, "prompt_token_ids": ids,
                               "prompt_token_ids_sha256": ids_sha, "raster": None}):
        return tr, []
    if add("prefill.prepare_aux", {"det_embedded_prompt_activations_sha256": emb, "prompt_token_ids": ids,
                                   "prompt_token_ids_sha256": ids_sha}):
        return tr, []
    # a backend that computes every layer prefix's KV commitment at once
    # (one download, parallel hashes) supplies kv_prefix_commitments
    prefix_kv = backend.kv_prefix_commitments(L) if hasattr(backend, "kv_prefix_commitments") else None
    done: list = []
    for layer in range(L):
        out = backend.layer_output_commitment(layer)
        if add("prefill.range", {"det_range_activations_sha256": out, "execution_mode": DET, "layer_idx": layer,
                                 "range_end": S, "range_start": 0, "token_count": S}):
            return tr, []
        done.append(out)
        if add("prefill.range_finalize", {"completed_layer_output_det_sha256s": list(done),
                                          "det_current_activations_sha256": out,
                                          "det_layer_caches_sha256": prefix_kv[layer] if prefix_kv is not None
                                          else backend.kv_commitment(layer + 1),
                                          "execution_mode": DET, "next_layer_idx": layer + 1}):
            return tr, []
    if add("prefill.finalize", {"decode_position": S, "decode_token_count": S,
                                "det_final_hidden_states_sha256": backend.hidden_commitment(),
                                "det_layer_caches_sha256": backend.kv_commitment(L),
                                "det_prefill_logits_sha256": backend.logits_commitment()}):
        return tr, []
    full, gen, pos = list(ids), [], S
    while len(gen) < max_new_tokens:
        token = backend.select()
        full, gen = full + [token], gen + [token]
        if add("decode.select_token", {"decode_position": pos, "decode_token_count": pos,
                                       "det_current_logits_sha256": backend.logits_commitment(),
                                       "full_token_ids": full, "full_token_ids_sha256": sha256_hex(full),
                                       "generated_token_ids": gen, "generated_token_ids_sha256": sha256_hex(gen),
                                       "max_new_tokens": max_new_tokens, "selected_next_token": token}):
            return tr, gen
        backend.decode(token)
        if add("decode.layer_range", {"completed_layer_output_det_sha256s":
                                      [backend.layer_output_commitment(layer) for layer in range(L)],
                                      "decode_position": pos, "decode_token_count": pos,
                                      "det_current_activation_sha256": backend.hidden_commitment(),
                                      "det_layer_caches_sha256": backend.kv_commitment(L), "execution_mode": DET,
                                      "layer_count": L, "layer_end": L, "layer_start": 0, "next_token": token}):
            return tr, gen
        pos += 1
        if add("decode.transition_finalize", {"decode_position": pos, "decode_token_count": pos,
                                              "det_current_logits_sha256": backend.logits_commitment(),
                                              "full_token_ids": full, "full_token_ids_sha256": sha256_hex(full),
                                              "generated_token_ids": gen,
                                              "generated_token_ids_sha256": sha256_hex(gen)}):
            return tr, gen
    if detokenize is not None:
        add("output.finalize", {"full_token_ids": full, "full_token_ids_sha256": sha256_hex(full),
                                "generated_text": detokenize(gen), "generated_token_count": len(gen),
                                "generated_token_ids": gen, "generated_token_ids_sha256": sha256_hex(gen),
                                "stop_reason": "max_new_tokens"})
    return tr, gen


def run_request(backend: Backend, preparer, prompt, num_layers: int, max_new_tokens: int,
                temperature: float = 1.0, add_generation_prompt: bool = True, add_special_tokens: bool = True,
                terminal: Optional[str] = None):
    """A run from the request's prompt bytes: prompt.prepare through
    ``preparer`` (a ``prompt.PromptPreparer`` of the bundle), then ``run`` with
    the prompt text for prompt.prepare and the preparer's detokenize for
    output.finalize.  Returns (trace, generated ids)."""
    prep = preparer.prepare(prompt, add_generation_prompt=add_generation_prompt,
                            add_special_tokens=add_special_tokens)
    return run(backend, prep.prompt_token_ids, num_layers, max_new_tokens, prompt_text=prep.prompt_text,
               temperature=temperature, detokenize=preparer.detokenize, terminal=terminal)


class SeqBackend:
    """Backend over an rdet sequence (the CUDA path through the C ABI).  The
    model must be opened with layer_commitments=True (per-layer prefill
    commitments)."""

    def __init__(self, seq):
        from . import BUF_EMBEDDING, BUF_HIDDEN, BUF_KV, BUF_LAYER_OUTPUT, BUF_LOGITS
        self.seq = seq
        self._b = (BUF_EMBEDDING, BUF_HIDDEN, BUF_LOGITS, BUF_LAYER_OUTPUT, BUF_KV)

    def prefill(self, token_ids):
        self.seq.prefill(list(token_ids))

    def select(self) -> int:
        return int(self.seq.select())

    def decode(self, token: int):
        self.seq.decode(int(token))

    def embedding_commitment(self):
        return self.seq.commitment(self._b[0])

    def hidden_commitment(self):
        return self.seq.commitment(self._b[1])

    def logits_commitment(self):
        return self.seq.commitment(self._b[2])

    def layer_output_commitment(self, layer):
        return self.seq.commitment(self._b[3], layer)

    def kv_commitment(self, layers):
        return self.seq.commitment(self._b[4], layers)

    def kv_prefix_commitments(self, n):
        return self.seq.kv_prefix_commitments(n)
