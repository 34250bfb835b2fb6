"""Context-parallel causal attention on CPU ranks (gloo): the zigzag-sharded
forward, log-sum-exp merge and backward against full-sequence attention."""

from __future__ import annotations

import math
import multiprocessing as mp
import socket
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _full_attention(qkv, B, T, H, D):
    q, k, v = qkv.view(B, T, 3, H, D).unbind(2)
    s = torch.einsum("bthd,bshd->bhts", q, k) / math.sqrt(D)
    s = s.masked_fill(torch.ones(T, T, dtype=torch.bool).triu(1), float("-inf"))
    lse2 = torch.logsumexp(s, -1) / math.log(2.0)
    o = torch.einsum("bhts,bshd->bthd", torch.softmax(s, -1), v).reshape(B, T, H * D)
    return o, lse2


def _worker(rank, world, port, q):
    sys.path.insert(0, str(ROOT))
    import torch.distributed as dist

    from underhfs_b200.parallel.context import (ContextParallelAttention, ContextParallelFunction, shard_sequence,
                                                unshard_sequence, zigzag_positions)

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        torch.manual_seed(0)
        B, H, D = 2, 2, 8
        T = 4 * world * 3
        F = H * D
        qkv = torch.randn(B, T, 3 * F, dtype=torch.float64).requires_grad_(True)
        do = torch.randn(B, T, F, dtype=torch.float64)
        o_ref, lse_ref = _full_attention(qkv, B, T, H, D)
        (dqkv_ref,) = torch.autograd.grad(o_ref, qkv, do)

        Tl = T // world
        local = shard_sequence(qkv.detach(), rank, world).contiguous()
        cp = ContextParallelAttention()
        o, lse = cp.forward(local.view(B * Tl, 3 * F), B, Tl, H, D)
        pos = zigzag_positions(rank, world, T)
        err_o = (o.view(B, Tl, F) - o_ref.detach()[:, pos]).abs().max().item()
        err_l = (lse - lse_ref.detach()[:, :, pos]).abs().max().item()
        d = cp.backward(local.view(B * Tl, 3 * F), o, lse, shard_sequence(do, rank, world).reshape(B * Tl, F),
                        B, Tl, H, D)
        err_d = (d.view(B, Tl, 3 * F) - dqkv_ref[:, pos]).abs().max().item()

        # autograd path, and the layout helpers round-trip
        x = local.view(B * Tl, 3 * F).clone().requires_grad_(True)
        y = ContextParallelFunction.apply(x, cp, B, Tl, H, D)
        (g,) = torch.autograd.grad(y, x, shard_sequence(do, rank, world).reshape(B * Tl, F))
        err_g = (g.view(B, Tl, 3 * F) - dqkv_ref[:, pos]).abs().max().item()
        parts = [shard_sequence(do, r, world) for r in range(world)]
        roundtrip = torch.equal(unshard_sequence(parts, world), do)
        q.put((rank, err_o, err_l, err_d, err_g, roundtrip))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [1, 2, 3])
def test_context_parallel_matches_full_attention(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    hung = [p for p in procs if p.is_alive()]
    for p in hung:
        p.kill()  # these exact child processes only
    assert not hung
    results = []
    while not q.empty():
        results.append(q.get())
    assert len(results) == world, results
    for rank, err_o, err_l, err_d, err_g, roundtrip in results:
        assert err_o < 1e-10 and err_l < 1e-10 and err_d < 1e-9 and err_g < 1e-9, results
        assert roundtrip


def test_zigzag_layout_balances_pairs():
    from underhfs_b200.parallel.context import chunk_owner, zigzag_chunks

    for size in (1, 2, 4, 8):
        owned = sorted(c for r in range(size) for c in zigzag_chunks(r, size))
        assert owned == list(range(2 * size))
        for r in range(size):
            a, b = zigzag_chunks(r, size)
            assert (a + 1) + (b + 1) == 2 * size + 1  # equal causal work on every rank
            assert chunk_owner(a, size) == (r, 0) and chunk_owner(b, size) == (r, 1)
