"""NVTX ranges for timeline profilers (Nsight Systems and the like).

Set ``UNDERHFS_NVTX=1`` to emit them; otherwise every call is a no-op, so the
ranges cost nothing in normal runs and inside CUDA-graph capture.  The engine
marks each forward / backward block, each DDP bucket reduction and each
ZeRO-3 gather / reduce, which is what an overlap timeline needs.
"""

from __future__ import annotations

import contextlib
import os

import torch

ENABLED = os.environ.get("UNDERHFS_NVTX", "0") == "1"


def push(name: str) -> None:
    if ENABLED:
        torch.cuda.nvtx.range_push(name)


def pop() -> None:
    if ENABLED:
        torch.cuda.nvtx.range_pop()


@contextlib.contextmanager
def nvtx_range(name: str):
    push(name)
    try:
        yield
    finally:
        pop()
