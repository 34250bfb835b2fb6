"""Datasets and loaders (reference data.py:10-39) plus the token pipeline
used for training on GPUs.

``DataLoader`` keeps the reference behaviour (lists of items, seeded
shuffle).  ``SyntheticTokens`` produces uniform token ids of a fixed
[batch, seq] shape from a seed, and ``PinnedBatchLoader`` stages each batch in
pinned host memory and copies it to the GPU with a non-blocking copy on a
dedicated stream, so host-to-device traffic overlaps compute.
"""

from __future__ import annotations

from dataclasses import dataclass
from random import Random
from typing import Generic, Iterator, Protocol, Sequence, TypeVar

import torch

T = TypeVar("T")


class Dataset(Protocol[T]):
    def __len__(self) -> int: ...

    def __getitem__(self, index: int) -> T: ...


@dataclass
class TensorDataset(Generic[T]):
    tensors: Sequence[T]

    def __len__(self) -> int:
        return len(self.tensors)

    def __getitem__(self, index: int) -> T:
        return self.tensors[index]


class DataLoader(Generic[T]):
    def __init__(self, dataset: Dataset[T], batch_size: int = 1, shuffle: bool = False, seed: int = 0) -> None:
        if batch_size <= 0:
            raise ValueError("batch_size must be positive")
        self.dataset = dataset
        self.batch_size = batch_size
        self.shuffle = shuffle
        self.seed = seed

    def __iter__(self) -> Iterator[list[T]]:
        order = list(range(len(self.dataset)))
        if self.shuffle:
            Random(self.seed).shuffle(order)
        for start in range(0, len(order), self.batch_size):
            yield [self.dataset[i] for i in order[start : start + self.batch_size]]


class SyntheticTokens:
    """Endless (ids, next-token targets) batches of uniform token ids in
    [0, vocab); deterministic for a (seed, rank) pair."""

    def __init__(self, vocab_size: int, batch: int, seq_len: int, *, seed: int = 0, rank: int = 0) -> None:
        self.vocab_size = vocab_size
        self.batch = batch
        self.seq_len = seq_len
        self.gen = torch.Generator().manual_seed(seed * 1000003 + rank)

    def next_host(self, out: torch.Tensor | None = None) -> torch.Tensor:
        """A [2, batch, seq_len] int64 host tensor: ids and targets."""
        seq = torch.randint(0, self.vocab_size, (self.batch, self.seq_len + 1), generator=self.gen)
        pair = torch.stack([seq[:, :-1], seq[:, 1:]])
        if out is None:
            return pair
        out.copy_(pair)
        return out

    def __iter__(self):
        while True:
            yield self.next_host()


class PinnedBatchLoader:
    """Double-buffered pinned host staging + async H2D on a copy stream."""

    def __init__(self, source: SyntheticTokens, device: torch.device | str = "cuda", depth: int = 2) -> None:
        self.source = source
        self.device = torch.device(device)
        shape = (2, source.batch, source.seq_len)
        self.host = [torch.empty(shape, dtype=torch.int64, pin_memory=True) for _ in range(depth)]
        self.dev = [torch.empty(shape, dtype=torch.int64, device=self.device) for _ in range(depth)]
        self.stream = torch.cuda.Stream(device=self.device)
        self.events = [None] * depth
        self.i = 0
        for k in range(depth):
            self.source.next_host(self.host[k])

    @property
    def bytes_per_batch(self) -> int:
        return self.host[0].numel() * self.host[0].element_size()

    def next(self) -> tuple[torch.Tensor, torch.Tensor]:
        k = self.i % len(self.host)
        self.i += 1
        with torch.cuda.stream(self.stream):
            self.stream.wait_stream(torch.cuda.current_stream(self.device))
            self.dev[k].copy_(self.host[k], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(self.stream)
        torch.cuda.current_stream(self.device).wait_event(ev)
        return self.dev[k][0], self.dev[k][1]
