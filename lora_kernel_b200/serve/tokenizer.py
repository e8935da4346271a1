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


class HFTokenizer:
    """A Hugging Face `tokenizer.json` (BPE / unigram / word-level, through the
    `tokenizers` library) with the interface of ByteTokenizer, for serving
    models that come with their own vocabulary (e.g. an imported GPTQ / AWQ
    Llama).  `apply_chat_template` renders the `chat_template` of a
    tokenizer_config.json next to the file when there is one (Jinja), else the
    plain "role: content" lines of ByteTokenizer."""

    def __init__(self, path: str):
        import json
        import os

        from tokenizers import Tokenizer
        self.tok = Tokenizer.from_file(path)
        self.vocab_size = self.tok.get_vocab_size()
        self.template = None
        self.bos = self.eos = ""
        conf = os.path.join(os.path.dirname(os.path.abspath(path)), "tokenizer_config.json")
        if os.path.exists(conf):
            with open(conf) as f:
                c = json.load(f)
            self.template = c.get("chat_template")
            tok_str = (lambda v: v.get("content", "") if isinstance(v, dict) else (v or ""))
            self.bos, self.eos = tok_str(c.get("bos_token")), tok_str(c.get("eos_token"))
        eid = self.tok.token_to_id(self.eos) if self.eos else None
        self.eos_token_id = eid if eid is not None else 0
        self.stop_ids = (eid,) if eid is not None else ()   # generation ends at the end-of-sequence token

    def encode(self, text: str) -> List[int]:
        return list(self.tok.encode(text, add_special_tokens=False).ids)

    def decode(self, ids: Iterable[int]) -> str:
        return self.tok.decode([int(i) for i in ids], skip_special_tokens=True)

    def apply_chat_template(self, messages) -> List[int]:
        if self.template:
            from jinja2.sandbox import ImmutableSandboxedEnvironment
            env = ImmutableSandboxedEnvironment(trim_blocks=True, lstrip_blocks=True)
            text = env.from_string(self.template).render(messages=messages, add_generation_prompt=True,
                                                         bos_token=self.bos, eos_token=self.eos)
            return self.encode(text)
        text = "".join(f"{m.get('role', 'user')}: {m.get('content', '')}\n" for m in messages)
        return self.encode(text + "assistant: ")

