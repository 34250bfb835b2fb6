"""Byte-level tokenizer (reference text.py:9-20): UTF-8 bytes <-> token ids, vocab 256."""

from __future__ import annotations

from dataclasses import dataclass

from underhfs_b200.tensor import Tensor, tensor


@dataclass(frozen=True)
class ByteTokenizer:
    vocab_size: int = 256

    def encode(self, text: str) -> Tensor:
        return tensor(list(text.encode("utf-8")))

    def decode(self, tokens: Tensor) -> str:
        values = tokens._storage if isinstance(tokens, Tensor) else list(tokens)
        return bytes(max(0, min(255, int(v))) for v in values).decode("utf-8", errors="ignore")
