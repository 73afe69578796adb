"""Tokenizer loading.

HF tokenizers are loaded offline from the model directory (or the
``tokenizer`` path). Random-init presets have no vocabulary files, so they
get :class:`ByteTokenizer`: UTF-8 bytes mapped to ids 3..258 (0 pad, 1 bos,
2 eos); other ids decode as ``<id>``. It keeps the text API usable end to
end (server, CLI) on synthetic models.
"""

from __future__ import annotations

import os
from typing import List, Optional


class ByteTokenizer:
    pad_token_id = 0
    bos_token_id = 1
    eos_token_id = 2

    def __init__(self, vocab_size: int = 32000):
        self.vocab_size = vocab_size

    def encode(self, text: str, add_special_tokens: bool = True) -> List[int]:
        ids = [b + 3 for b in text.encode("utf-8")]
        return ([self.bos_token_id] + ids) if add_special_tokens else ids

    def decode(self, ids, skip_special_tokens: bool = True) -> str:
        out = bytearray()
        parts: List[str] = []
        for t in ids:
            t = int(t)
            if 3 <= t < 259:
                out.append(t - 3)
                continue
            if out:
                parts.append(out.decode("utf-8", errors="replace"))
                out = bytearray()
            if t < 3:
                if not skip_special_tokens:
                    parts.append(["<pad>", "<s>", "</s>"][t])
            else:
                parts.append(f"<{t}>")
        if out:
            parts.append(out.decode("utf-8", errors="replace"))
        return "".join(parts)

    def __call__(self, text: str):
        return {"input_ids": self.encode(text)}

    def apply_chat_template(self, messages, add_generation_prompt: bool = True,
                            tokenize: bool = False, **_):
        text = chat_prompt(messages)
        return self.encode(text) if tokenize else text


def chat_prompt(messages) -> str:
    """Plain-text chat layout used when the tokenizer has no template
    ("System: / User: / Assistant:", as python/swiftllm/cli.py:546-555)."""
    parts = []
    for m in messages:
        role = m.get("role", "user") if isinstance(m, dict) else getattr(m, "role", "user")
        content = m.get("content", "") if isinstance(m, dict) else getattr(m, "content", "")
        parts.append(f"{role.capitalize()}: {content}")
    parts.append("Assistant:")
    return "\n".join(parts)


def load_tokenizer(path: Optional[str], vocab_size: int, trust_remote_code: bool = False):
    if path and os.path.isdir(path) and any(
            os.path.exists(os.path.join(path, f))
            for f in ("tokenizer.json", "tokenizer.model", "tokenizer_config.json")):
        try:
            from transformers import AutoTokenizer
            return AutoTokenizer.from_pretrained(path, trust_remote_code=trust_remote_code,
                                                 local_files_only=True)
        except Exception:  # pragma: no cover - depends on local files
            pass
    return ByteTokenizer(vocab_size)
