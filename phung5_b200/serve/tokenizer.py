"""Tokenizers for the HTTP layer.

`ByteTokenizer` maps UTF-8 bytes to ids 0..255 (plus BOS/EOS specials) so the server works with any
random-init model offline. `load_tokenizer(path)` loads an HF tokenizer directory (tokenizer.json)
through `transformers` when a real checkpoint is served.
"""
from __future__ import annotations

from typing import List, Optional, Sequence


class ByteTokenizer:
    bos_id = 256
    eos_id = 257
    stop_ids = [257]
    vocab_size = 258

    def encode(self, text: str, add_bos: bool = False) -> List[int]:
        ids = list(text.encode("utf-8"))
        return ([self.bos_id] if add_bos else []) + ids

    def decode(self, ids: Sequence[int]) -> str:
        return bytes(i for i in ids if 0 <= i < 256).decode("utf-8", errors="replace")

    def apply_chat_template(self, messages: List[dict]) -> str:
        parts = []
        for m in messages:
            c = m.get("content", "")
            if isinstance(c, list):  # OpenAI content parts: keep the text ones
                c = "".join(p.get("text", "") for p in c if isinstance(p, dict))
            parts.append(f"<|{m.get('role', 'user')}|>\n{c}\n")
        return "".join(parts) + "<|assistant|>\n"


class HFTokenizer:
    def __init__(self, path: str):
        from transformers import AutoTokenizer
        self.tok = AutoTokenizer.from_pretrained(path, local_files_only=True)
        self.eos_id = self.tok.eos_token_id
        self.stop_ids = sorted(set(([self.eos_id] if self.eos_id is not None else []) + _generation_eos(path)))
        self.vocab_size = len(self.tok)

    def encode(self, text: str, add_bos: bool = False) -> List[int]:
        return self.tok.encode(text, add_special_tokens=add_bos)

    def decode(self, ids: Sequence[int]) -> str:
        return self.tok.decode(list(ids), skip_special_tokens=True)

    def apply_chat_template(self, messages: List[dict]) -> str:
        return self.tok.apply_chat_template(messages, tokenize=False, add_generation_prompt=True)


def _generation_eos(path: str) -> List[int]:
    """End-of-turn ids a chat checkpoint lists in generation_config.json (an int or a list)."""
    import json
    import os
    f = os.path.join(path, "generation_config.json")
    try:
        with open(f) as fh:
            v = json.load(fh).get("eos_token_id")
    except (OSError, ValueError):
        return []
    return [int(x) for x in (v if isinstance(v, list) else [v]) if isinstance(x, int)]


def has_tokenizer(path: Optional[str]) -> bool:
    import os
    return bool(path) and any(os.path.exists(os.path.join(path, f))
                              for f in ("tokenizer.json", "tokenizer.model", "tokenizer_config.json"))


def load_tokenizer(path: Optional[str] = None):
    return HFTokenizer(path) if path else ByteTokenizer()
