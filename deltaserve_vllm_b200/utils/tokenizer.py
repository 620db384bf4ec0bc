"""Tokenizers: an HF tokenizer from a local directory when one is configured,
otherwise a byte-level fallback (UTF-8 bytes shifted past the special ids)
so random-initialised models can still serve text prompts offline."""

from __future__ import annotations

import os


class ByteTokenizer:
    """Byte-level tokenizer over any vocabulary of at least 259 ids: 0=pad,
    1=bos, 2=eos, 3+b for byte b. Ids beyond the byte range decode to ''."""

    pad_token_id, bos_token_id, eos_token_id = 0, 1, 2

    def __init__(self, vocab_size: int):
        if vocab_size < 259:
            raise ValueError("byte tokenizer needs a vocabulary of at least 259 ids")
        self.vocab_size = vocab_size

    def encode(self, text: str, add_special_tokens: bool = False) -> list[int]:
        ids = [3 + b for b in text.encode("utf-8")]
        return ([self.bos_token_id] + ids) if add_special_tokens else ids

    def decode(self, ids, skip_special_tokens: bool = True) -> str:
        bs = bytes(i - 3 for i in ids if 3 <= i < 259)
        return bs.decode("utf-8", errors="replace")


def load_tokenizer(path: str | None, vocab_size: int):
    if path and os.path.isdir(path):
        try:
            from transformers import AutoTokenizer
            return AutoTokenizer.from_pretrained(path, local_files_only=True)
        except Exception:
            pass
    return ByteTokenizer(vocab_size)
