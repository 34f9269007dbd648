"""Tokenizer loading.  Model directories with tokenizer files use AutoTokenizer (as the
reference does, mini_vllm/engine/llm_engine.py:34); a directory holding only config.json (a
random-init benchmark model) gets a token-id pass-through tokenizer whose eos id comes from the
model config."""
from __future__ import annotations

import os


class IdTokenizer:
    """Prompts are token-id lists; decode renders ids as space-separated text."""

    def __init__(self, eos_token_id: int | None):
        self.eos_token_id = eos_token_id

    def encode(self, text: str) -> list[int]:
        raise ValueError("this model directory has no tokenizer files: pass prompts as token-id lists")

    def decode(self, token_ids) -> str:
        return " ".join(str(t) for t in token_ids)


def load_tokenizer(model_dir: str, hf_config):
    has_files = any(os.path.exists(os.path.join(model_dir, f))
                    for f in ("tokenizer.json", "tokenizer_config.json", "vocab.json", "tokenizer.model"))
    if has_files:
        from transformers import AutoTokenizer
        return AutoTokenizer.from_pretrained(model_dir, use_fast=True)
    eos = getattr(hf_config, "eos_token_id", None)
    if isinstance(eos, (list, tuple)):
        eos = eos[0] if eos else None
    return IdTokenizer(eos)
