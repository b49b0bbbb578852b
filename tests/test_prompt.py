"""prompt.prepare and output detokenization (raster-inference_b200/prompt.py)
on the CPU, against the reference's own prompt tests
(src/routines/prompt_prepare/native/tests.rs) and its golden trace of
tiny-gemma-dev: the trace built from the request's prompt text reproduces
native-det-full, prompt.prepare and output.finalize entries included."""
import importlib
import json
import os
import tempfile

import pytest

import tiny_gemma_dev
from helpers import detwgt
from test_trace import OracleBackend

prompt = importlib.import_module("raster-inference_b200.prompt")
trace = importlib.import_module("raster-inference_b200.trace")

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = json.load(open(os.path.join(HERE, "golden", "det_trace_goldens.json")))
TEXT = os.path.join(HERE, "golden", "tiny_gemma_dev_text")

# the template of render_prompt_uses_messages_and_generation_flag (tests.rs:31-46)
TEMPLATE = ("{{ bos_token }}{% for message in messages %}[{{ message.role }}] {{ message.content }}{% endfor %}"
            "{% if add_generation_prompt %}[assistant]{% endif %}")


def test_render_uses_messages_and_generation_flag():
    p = prompt.PromptPreparer(chat_template=TEMPLATE, bos_token="<bos>")
    assert p.render("hello", True) == "<bos>[user] hello[assistant]"
    assert p.render("hello", False) == "<bos>[user] hello"


def test_empty_prompt_is_rejected():
    with pytest.raises(ValueError, match="non-empty prompt"):
        prompt.PromptPreparer(chat_template=TEMPLATE).render("")


def test_prompt_commitment_hashes_token_ids_only():
    # build_prompt_commitment_hashes_prompt_token_ids_only (tests.rs:48-55)
    assert trace.sha256_hex([1, 2, 3]) == "a615eeaee21de5179de080de8c3052c8da901138406ba71c38c032845f7d54f4"


def test_tiny_bundle_prompt_ids_and_detokenize():
    p = prompt.PromptPreparer(TEXT)
    prep = p.prepare(GOLD["prompt_text"].encode("utf-8"))
    assert prep.prompt_text == GOLD["prompt_text"]
    assert prep.prompt_token_ids == GOLD["prompt_token_ids"]
    assert prep.prompt_token_ids_sha256 == trace.sha256_hex(GOLD["prompt_token_ids"])
    assert p.detokenize(GOLD["generated_token_ids"]) == GOLD["generated_text"]
    assert p.detokenize([]) == ""


def test_invalid_utf8_prompt_bytes_are_rejected():
    with pytest.raises(UnicodeDecodeError):
        prompt.PromptPreparer(TEXT).prepare(b"\xff\xfe")


def test_trace_from_prompt_text_reproduces_native_det_full():
    # the whole request path: prompt bytes -> prompt.prepare -> prefill and
    # decode (the oracle as executor) -> output.finalize
    d = tiny_gemma_dev.write_bundle(tempfile.mkdtemp(), detwgt.encode)
    tr, gen = trace.run_request(OracleBackend(d), prompt.PromptPreparer(TEXT), GOLD["prompt_text"].encode("utf-8"),
                                num_layers=4, max_new_tokens=GOLD["max_new_tokens"],
                                temperature=GOLD["temperature"])
    assert gen == GOLD["generated_token_ids"]
    assert [list(e) for e in tr.entries] == GOLD["native-det-full"]
