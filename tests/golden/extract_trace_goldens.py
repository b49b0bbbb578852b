"""Copies the reference's det checkpoint-trace goldens into a fixture.

Sources (casettek/raster-inference): tests/goldens/native-det-full.json and
native-det-terminal.json, written by tests/golden_traces.rs for the request
built there (golden_native_det_full / golden_native_det_terminal): prompt
"hello raster prompt", add_generation_prompt, add_special_tokens,
deterministic mode, max_new_tokens 2, temperature 1.0, on
assets/tiny-gemma-dev.  The prompt token ids come from that bundle's
chat_template.jinja and tokenizer.json (jinja2 + tokenizers, the same render
and encode calls as prompt_prepare/native/tiles.rs:48-86), and the text of the
generated ids from tokenizer.decode(ids, skip_special_tokens=True)
(output_finalize/native/tiles.rs:5-13); the generated ids come from the oracle.
The bundle's chat_template.jinja and tokenizer.json are copied beside the
output (tiny_gemma_dev_text/) for the prompt.prepare tests.
Run where the reference checkout is available; the output is committed so that
tests never read the reference at run time.

    python tests/golden/extract_trace_goldens.py /path/to/raster-inference
"""
import json
import os
import sys

import jinja2
import tokenizers

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", ".."))
sys.path.insert(0, os.path.join(HERE, ".."))

if len(sys.argv) < 2:
    sys.exit("usage: extract_trace_goldens.py <raster-inference checkout>")
ref = sys.argv[1]
bundle = os.path.join(ref, "assets/tiny-gemma-dev")
PROMPT = "hello raster prompt"
MAX_NEW = 2

tpl = open(os.path.join(bundle, "chat_template.jinja")).read()
rendered = jinja2.Environment().from_string(tpl).render(
    messages=[{"role": "user", "content": PROMPT}], add_generation_prompt=True, bos_token=None, eos_token=None,
    unk_token=None)
tok = tokenizers.Tokenizer.from_file(os.path.join(bundle, "tokenizer.json"))
ids = tok.encode(rendered, add_special_tokens=True).ids

import oracle.oracle as O  # noqa: E402  (the generated ids of the golden run)

m = O.Model(bundle, threads=4)
s = m.seq()
_, logits, _ = s.prefill(ids, want_hidden=False, want_layer_hashes=False)
gen = []
for _ in range(MAX_NEW):
    t = O.argmax_first(logits)
    gen.append(t)
    _, logits, _ = s.decode(t, want_layer_hashes=False)


def entries(name):
    with open(os.path.join(ref, "tests/goldens", name + ".json")) as f:
        return [list(e.items())[0] for e in json.load(f)]


out = {
    "source": "casettek/raster-inference tests/goldens/native-det-{full,terminal}.json (tests/golden_traces.rs)",
    "prompt_text": PROMPT,
    "prompt_token_ids": ids,
    "max_new_tokens": MAX_NEW,
    "temperature": 1.0,
    "generated_token_ids": gen,
    "generated_text": tok.decode(gen, skip_special_tokens=True),
    "terminal": "prefill.finalize",
    "native-det-full": entries("native-det-full"),
    "native-det-terminal": entries("native-det-terminal"),
}
# the bundle's chat template and tokenizer, as text fixtures for the
# prompt.prepare tests (tests/test_prompt.py)
text_dir = os.path.join(HERE, "tiny_gemma_dev_text")
os.makedirs(text_dir, exist_ok=True)
for name in ("chat_template.jinja", "tokenizer.json"):
    with open(os.path.join(bundle, name), "rb") as f_in, open(os.path.join(text_dir, name), "wb") as f_out:
        f_out.write(f_in.read())
dst = os.path.join(HERE, "det_trace_goldens.json")
with open(dst, "w") as f:
    json.dump(out, f, indent=1)
print("wrote", dst, "prompt ids", ids, "generated", gen)
