"""prompt.prepare and output detokenization for a model bundle (host glue).

The deterministic executor takes token ids; this module turns a request's
prompt bytes into those ids and generated ids back into text, so that a run
here can start from the same request the reference takes and record its
prompt.prepare and output.finalize checkpoints.  It restates
casettek/raster-inference ``src/routines/prompt_prepare/mod.rs:27-50`` with
``prompt_prepare/native/tiles.rs:24-86`` and
``output_finalize/native/tiles.rs:5-13``:

1. the prompt bytes decode as UTF-8 (``decode_prompt_bytes``);
2. they become one user message, which must not be empty
   (``build_gemma4_messages``);
3. the bundle's ``chat_template.jinja`` renders with ``messages``,
   ``add_generation_prompt`` and the bos/eos/unk tokens (``render_prompt``);
4. the bundle's ``tokenizer.json`` encodes the rendered text, with or without
   special tokens (``tokenize_prompt``);
5. the ids' commitment is SHA-256 of their compact JSON
   (``build_prompt_commitment``).

The reference renders with minijinja and tokenizes with the Rust
``tokenizers`` crate; here ``jinja2`` and the ``tokenizers`` Python package
(a binding of that same crate) do the same work.  Values the template prints
are finalized the way minijinja displays them (``none``, ``true``/``false``)
rather than Python's spelling.
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Optional, Sequence

from .trace import sha256_hex


def _minijinja_display(value):
    if value is None:
        return "none"
    if value is True:
        return "true"
    if value is False:
        return "false"
    return value


@dataclass
class PromptPreparation:
    """PromptPreparationState (prompt_prepare/mod.rs:45-49)."""
    prompt_text: str
    prompt_token_ids: list
    prompt_token_ids_sha256: str


class PromptPreparer:
    """The chat template and tokenizer of one bundle.

    model_dir: a bundle holding ``chat_template.jinja`` and ``tokenizer.json``
    (or pass ``chat_template`` / ``tokenizer_path`` directly).  bos/eos/unk:
    the ModelSpec tokens the template may print (the reference's command line
    passes none of them)."""

    def __init__(self, model_dir: Optional[str] = None, chat_template: Optional[str] = None,
                 tokenizer_path: Optional[str] = None, bos_token: Optional[str] = None,
                 eos_token: Optional[str] = None, unk_token: Optional[str] = None):
        import jinja2
        if chat_template is None:
            if model_dir is None:
                raise ValueError("a chat template or a model directory is required")
            with open(os.path.join(model_dir, "chat_template.jinja"), encoding="utf-8") as f:
                chat_template = f.read()
        if tokenizer_path is None and model_dir is not None:
            tokenizer_path = os.path.join(model_dir, "tokenizer.json")
        env = jinja2.Environment(finalize=_minijinja_display)
        self.template = env.from_string(chat_template)
        self.tokenizer = None
        if tokenizer_path is not None:
            import tokenizers
            self.tokenizer = tokenizers.Tokenizer.from_file(tokenizer_path)
        self.bos_token, self.eos_token, self.unk_token = bos_token, eos_token, unk_token

    def render(self, prompt_text: str, add_generation_prompt: bool = True) -> str:
        """build_gemma4_messages + render_prompt (tiles.rs:31-77)."""
        if not prompt_text:
            raise ValueError("input embedding requires a non-empty prompt")
        return self.template.render(messages=[{"role": "user", "content": prompt_text}],
                                    add_generation_prompt=add_generation_prompt, bos_token=self.bos_token,
                                    eos_token=self.eos_token, unk_token=self.unk_token)

    def tokenize(self, rendered: str, add_special_tokens: bool = True) -> list:
        """tokenize_prompt (tiles.rs:79-89)."""
        if self.tokenizer is None:
            raise ValueError("no tokenizer.json was given")
        return list(self.tokenizer.encode(rendered, add_special_tokens=add_special_tokens).ids)

    def prepare(self, prompt: bytes | str, add_generation_prompt: bool = True,
                add_special_tokens: bool = True) -> PromptPreparation:
        """prompt_prepare::run (mod.rs:27-50) for UTF-8 prompt bytes."""
        text = prompt.decode("utf-8") if isinstance(prompt, (bytes, bytearray)) else prompt
        ids = self.tokenize(self.render(text, add_generation_prompt), add_special_tokens)
        return PromptPreparation(text, ids, sha256_hex(ids))

    def detokenize(self, token_ids: Sequence[int]) -> str:
        """detokenize_output_tokens (output_finalize/native/tiles.rs:5-13):
        special tokens skipped; no ids, no text."""
        ids = [int(t) for t in token_ids]
        if not ids:
            return ""
        if self.tokenizer is None:
            raise ValueError("no tokenizer.json was given")
        return self.tokenizer.decode(ids, skip_special_tokens=True)
