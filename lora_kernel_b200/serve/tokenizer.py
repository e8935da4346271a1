"""Byte-level tokenizer: token id = byte value.

Same behaviour as the reference's TiktokenTokenizer (include/data/tokenizers.hpp:
10-35: encode maps each byte to its value, decode clamps ids to a byte); ids
outside [0, 256) decode to nothing.  The benchmarks feed synthetic token ids,
so the tokenizer is only used by the HTTP server for text prompts.
"""
from __future__ import annotations

from typing import Iterable, List


class ByteTokenizer:
    eos_token_id = 0

    def __init__(self, vocab_size: int = 256):
        self.vocab_size = vocab_size

    def encode(self, text: str) -> List[int]:
        return [b % self.vocab_size for b in text.encode("utf-8")]

    def decode(self, ids: Iterable[int]) -> str:
        return bytes(i for i in ids if 0 <= i < 256).decode("utf-8", errors="replace")

    def apply_chat_template(self, messages) -> List[int]:
        text = "".join(f"{m.get('role', 'user')}: {m.get('content', '')}\n" for m in messages)
        return self.encode(text + "assistant: ")
