"""Context (sequence) parallelism for causal attention.

The reference has no sequence parallelism: its sequence length is bounded by
learned positions and one GPU (nn.py:300, 311-312; attention materialises
T x T scores, nn.py:263-271).  Here a group of C ranks shares each sequence.

Layout ("zigzag"): a sequence of T tokens is cut into 2C chunks of T / (2C);
rank r holds chunks r and 2C-1-r, in that order.  Under a causal mask chunk
a attends chunks b <= a, so every rank computes the same number (2C + 1) of
chunk pairs and the work is balanced.

Forward: each rank all-gathers the K/V of the group (NVSwitch gives every
rank full bandwidth to every peer, so one all-gather beats a ring of C-1
steps), computes its two chunks against their diagonal and local key chunks
while the all-gather is in flight, then against the remote chunks, and merges
the partial results with their log-sum-exps (log2 domain, as the attention
kernels store them):  lse = log2 sum_b 2^lse_b,  O = sum_b 2^(lse_b - lse) O_b.

Backward: the flash backward of every pair uses the merged O and lse, which
makes each pair's dQ / dK / dV the exact restriction of the full gradient.
dQ stays local; dK / dV of remote chunks are summed over the group with one
reduce-scatter, launched as soon as the remote pairs are done and overlapped
with the local pairs.

Weight gradients of a context-parallel model are averaged over the group like
data-parallel gradients (each rank's loss is the mean over its own tokens).
"""

from __future__ import annotations

import math

import torch
import torch.distributed as dist


# ------------------------------------------------------------ layout helpers
def zigzag_chunks(rank: int, size: int) -> tuple[int, int]:
    """The two sequence chunks (of 2 * size) that `rank` holds."""
    return rank, 2 * size - 1 - rank


def chunk_owner(chunk: int, size: int) -> tuple[int, int]:
    """(rank, slot) holding `chunk`: slot 0 is the first half of the rank's tokens."""
    return (chunk, 0) if chunk < size else (2 * size - 1 - chunk, 1)


def zigzag_positions(rank: int, size: int, seq_len: int, device=None) -> torch.Tensor:
    """Global positions of this rank's tokens, in local order."""
    if seq_len % (2 * size):
        raise ValueError(f"sequence length {seq_len} must be a multiple of 2 x context size {2 * size}")
    tc = seq_len // (2 * size)
    a, b = zigzag_chunks(rank, size)
    return torch.cat([torch.arange(a * tc, (a + 1) * tc), torch.arange(b * tc, (b + 1) * tc)]).to(device)


def shard_sequence(x: torch.Tensor, rank: int, size: int, dim: int = 1) -> torch.Tensor:
    """This rank's tokens of a full-sequence tensor ([B, T, ...] by default)."""
    pos = zigzag_positions(rank, size, x.shape[dim], device=x.device)
    return x.index_select(dim, pos)


def unshard_sequence(parts: list[torch.Tensor], size: int, dim: int = 1) -> torch.Tensor:
    """Inverse of shard_sequence given every rank's part (in rank order)."""
    tl = parts[0].shape[dim]
    seq = tl * size
    out = torch.empty(*parts[0].shape[:dim], seq, *parts[0].shape[dim + 1:], dtype=parts[0].dtype,
                      device=parts[0].device)
    for r, p in enumerate(parts):
        out.index_copy_(dim, zigzag_positions(r, size, seq, device=p.device), p)
    return out


def _acc(t: torch.Tensor) -> torch.dtype:
    """Accumulation dtype: fp32, or fp64 for fp64 inputs (oracle runs)."""
    return torch.float64 if t.dtype == torch.float64 else torch.float32


# ------------------------------------------------------------ block kernels
class _KernelBlocks:
    """One chunk pair on the fused tcgen05 attention kernels ([B*Tc, 3F] in)."""

    @staticmethod
    def fwd(fb, B, Tc, H, D, causal, scale):
        from underhfs_b200.ops import kernels as K

        return K.flash_attn_qkv(fb, B, Tc, H, D, causal, scale)

    @staticmethod
    def bwd(fb, o, lse, do, B, Tc, H, D, causal, scale):
        from underhfs_b200.ops import kernels as K

        return K.flash_attn_qkv_backward(fb, o, lse, do, B, Tc, H, D, causal, scale)


class _ReferenceBlocks:
    """The same contract in plain fp32 PyTorch (CPU ranks, oracle)."""

    @staticmethod
    def _split(fb, B, Tc, H, D):
        q, k, v = fb.to(_acc(fb)).view(B, Tc, 3, H, D).unbind(2)
        return q, k, v

    @staticmethod
    def fwd(fb, B, Tc, H, D, causal, scale):
        q, k, v = _ReferenceBlocks._split(fb, B, Tc, H, D)
        s = torch.einsum("bthd,bshd->bhts", q, k) * scale
        if causal:
            s = s.masked_fill(torch.ones(Tc, Tc, dtype=torch.bool, device=s.device).triu(1), float("-inf"))
        m = s.amax(-1, keepdim=True)
        p = torch.exp(s - m)
        l = p.sum(-1, keepdim=True)
        o = torch.einsum("bhts,bshd->bthd", p / l, v).reshape(B * Tc, H * D).to(fb.dtype)
        lse2 = ((m + torch.log(l)).squeeze(-1) / math.log(2.0)).contiguous()
        return o, lse2

    @staticmethod
    def bwd(fb, o, lse, do, B, Tc, H, D, causal, scale):
        q, k, v = _ReferenceBlocks._split(fb, B, Tc, H, D)
        of = o.to(q.dtype).view(B, Tc, H, D)
        dof = do.to(q.dtype).view(B, Tc, H, D)
        s = torch.einsum("bthd,bshd->bhts", q, k) * scale
        p = torch.exp(s - lse.unsqueeze(-1) * math.log(2.0))
        if causal:
            p = p.masked_fill(torch.ones(Tc, Tc, dtype=torch.bool, device=p.device).triu(1), 0.0)
        delta = (dof * of).sum(-1).permute(0, 2, 1)  # [B, H, Tc]
        dv = torch.einsum("bhts,bthd->bshd", p, dof)
        dp = torch.einsum("bthd,bshd->bhts", dof, v)
        ds = p * (dp - delta.unsqueeze(-1))
        dq = torch.einsum("bhts,bshd->bthd", ds, k) * scale
        dk = torch.einsum("bhts,bthd->bshd", ds, q) * scale
        return torch.stack([dq, dk, dv], dim=2).reshape(B * Tc, 3 * H * D).to(fb.dtype)


# ------------------------------------------------------------ the attention
class ContextParallelAttention:
    """Causal attention over a sequence sharded by `zigzag_positions`.

    ``forward(qkv, B, Tl, H, D)`` takes this rank's fused projection
    [B*Tl, 3F] (Tl = T / C local tokens per sequence, local order) and returns
    (o [B*Tl, F], lse [B, H, Tl]) like the single-GPU kernel; ``backward``
    returns dqkv [B*Tl, 3F].  `group` is the context-parallel process group
    (None = the default group).
    """

    def __init__(self, group=None, *, blocks=None, scale: float | None = None) -> None:
        self.group = group
        self.size = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.blocks = blocks
        self.scale = scale
        self.backend = dist.get_backend(group)

    def _blocks(self, t: torch.Tensor):
        if self.blocks is not None:
            return self.blocks
        return _KernelBlocks if t.is_cuda else _ReferenceBlocks

    # ------------------------------------------------------------ helpers
    def _pairs(self):
        a0, a1 = zigzag_chunks(self.rank, self.size)
        pairs = [(a, b) for a in (a0, a1) for b in range(a + 1)]
        local = [(a, b) for a, b in pairs if chunk_owner(b, self.size)[0] == self.rank]
        remote = [(a, b) for a, b in pairs if chunk_owner(b, self.size)[0] != self.rank]
        return local, remote

    def _slot(self, chunk: int) -> int:
        return chunk_owner(chunk, self.size)[1]

    def _fused(self, qkv3, kv_src, a, b, B, Tc, F):
        """[B*Tc, 3F]: q of local chunk a next to k / v of chunk b."""
        fb = torch.empty(B, Tc, 3 * F, dtype=qkv3.dtype, device=qkv3.device)
        sa = self._slot(a)
        fb[:, :, :F] = qkv3[:, sa * Tc:(sa + 1) * Tc, :F]
        sb = self._slot(b)
        fb[:, :, F:] = kv_src[:, sb * Tc:(sb + 1) * Tc]
        return fb.view(B * Tc, 3 * F)

    def _all_gather(self, kv: torch.Tensor, async_op: bool):
        out = torch.empty((self.size,) + tuple(kv.shape), dtype=kv.dtype, device=kv.device)
        if self.backend == "gloo":
            work = dist.all_gather(list(out.unbind(0)), kv, group=self.group, async_op=async_op)
        else:
            work = dist.all_gather_into_tensor(out, kv, group=self.group, async_op=async_op)
        return out, work

    def _kv_of(self, gathered, chunk, qkv3, F):
        owner, _ = chunk_owner(chunk, self.size)
        if owner == self.rank:
            return qkv3[:, :, F:]
        return gathered[owner]

    # ------------------------------------------------------------ forward
    def forward(self, qkv: torch.Tensor, B: int, Tl: int, H: int, D: int):
        F = H * D
        if Tl % 2:
            raise ValueError("context-parallel local length must be even (two chunks)")
        Tc = Tl // 2
        scale = (1.0 / math.sqrt(D)) if self.scale is None else self.scale
        blocks = self._blocks(qkv)
        qkv3 = qkv.view(B, Tl, 3 * F)
        kv_local = qkv3[:, :, F:].contiguous()
        gathered, work = self._all_gather(kv_local, async_op=True)
        local, remote = self._pairs()
        parts: dict[int, list] = {a: [] for a in zigzag_chunks(self.rank, self.size)}
        for a, b in local:  # overlaps the all-gather
            o_ab, lse_ab = blocks.fwd(self._fused(qkv3, kv_local, a, b, B, Tc, F), B, Tc, H, D, a == b, scale)
            parts[a].append((o_ab, lse_ab))
        if work is not None:
            work.wait()
        for a, b in remote:
            kv_b = self._kv_of(gathered, b, qkv3, F)
            o_ab, lse_ab = blocks.fwd(self._fused(qkv3, kv_b, a, b, B, Tc, F), B, Tc, H, D, False, scale)
            parts[a].append((o_ab, lse_ab))
        o = torch.empty(B, Tl, F, dtype=qkv.dtype, device=qkv.device)
        lse = torch.empty(B, H, Tl, dtype=_acc(qkv), device=qkv.device)
        for a, lst in parts.items():
            sa = self._slot(a)
            oa, la = self._merge(lst, B, Tc, H, D)
            o[:, sa * Tc:(sa + 1) * Tc] = oa
            lse[:, :, sa * Tc:(sa + 1) * Tc] = la
        return o.view(B * Tl, F), lse

    @staticmethod
    def _merge(parts, B, Tc, H, D):
        lses = torch.stack([p[1] for p in parts])  # [n, B, H, Tc]
        m = lses.amax(0)
        lse = m + torch.log2(torch.exp2(lses - m).sum(0))
        acc = torch.zeros(B, Tc, H, D, dtype=_acc(parts[0][0]), device=lses.device)
        for o_ab, lse_ab in parts:
            w = torch.exp2(lse_ab - lse).permute(0, 2, 1).unsqueeze(-1)  # [B, Tc, H, 1]
            acc += w * o_ab.to(acc.dtype).view(B, Tc, H, D)
        return acc.view(B, Tc, H * D).to(parts[0][0].dtype), lse

    # ------------------------------------------------------------ backward
    def backward(self, qkv, o, lse, do, B: int, Tl: int, H: int, D: int, gathered=None):
        F = H * D
        Tc = Tl // 2
        scale = (1.0 / math.sqrt(D)) if self.scale is None else self.scale
        blocks = self._blocks(qkv)
        qkv3 = qkv.view(B, Tl, 3 * F)
        kv_local = qkv3[:, :, F:].contiguous()
        if gathered is None:
            gathered, work = self._all_gather(kv_local, async_op=False)
        o3 = o.view(B, Tl, F)
        do3 = do.reshape(B, Tl, F)
        local, remote = self._pairs()
        acc = _acc(qkv)
        dq = torch.zeros(B, Tl, F, dtype=acc, device=qkv.device)
        # dK / dV of every rank's tokens, summed over the group by reduce-scatter
        dkv = torch.zeros(self.size, B, Tl, 2 * F, dtype=acc, device=qkv.device)

        def run(a, b, kv_b, causal):
            sa, sb = self._slot(a), self._slot(b)
            oa = o3[:, sa * Tc:(sa + 1) * Tc].reshape(B * Tc, F).contiguous()
            la = lse[:, :, sa * Tc:(sa + 1) * Tc].contiguous()
            da = do3[:, sa * Tc:(sa + 1) * Tc].reshape(B * Tc, F).contiguous()
            d = blocks.bwd(self._fused(qkv3, kv_b, a, b, B, Tc, F), oa, la, da, B, Tc, H, D, causal, scale)
            d = d.view(B, Tc, 3 * F).to(acc)
            dq[:, sa * Tc:(sa + 1) * Tc] += d[:, :, :F]
            owner = chunk_owner(b, self.size)[0]
            dkv[owner, :, sb * Tc:(sb + 1) * Tc] += d[:, :, F:]

        for a, b in remote:
            run(a, b, self._kv_of(gathered, b, qkv3, F), False)
        mine = torch.empty(B, Tl, 2 * F, dtype=acc, device=qkv.device)
        if self.backend == "gloo":  # gloo has no reduce-scatter
            work = dist.all_reduce(dkv, group=self.group, async_op=True)
        else:
            work = dist.reduce_scatter_tensor(mine, dkv, group=self.group, async_op=True)
        own = torch.zeros(B, Tl, 2 * F, dtype=acc, device=qkv.device)
        for a, b in local:
            sa, sb = self._slot(a), self._slot(b)
            oa = o3[:, sa * Tc:(sa + 1) * Tc].reshape(B * Tc, F).contiguous()
            la = lse[:, :, sa * Tc:(sa + 1) * Tc].contiguous()
            da = do3[:, sa * Tc:(sa + 1) * Tc].reshape(B * Tc, F).contiguous()
            d = blocks.bwd(self._fused(qkv3, kv_local, a, b, B, Tc, F), oa, la, da, B, Tc, H, D, a == b, scale)
            d = d.view(B, Tc, 3 * F).to(acc)
            dq[:, sa * Tc:(sa + 1) * Tc] += d[:, :, :F]
            own[:, sb * Tc:(sb + 1) * Tc] += d[:, :, F:]
        work.wait()
        if self.backend == "gloo":
            mine = dkv[self.rank]
        mine += own
        return torch.cat([dq, mine], dim=2).to(qkv.dtype).view(B * Tl, 3 * F)


class ContextParallelFunction(torch.autograd.Function):
    """Autograd wrapper: qkv [B*Tl, 3F] -> o [B*Tl, F]."""

    @staticmethod
    def forward(ctx, qkv, cp: ContextParallelAttention, B: int, Tl: int, H: int, D: int):
        o, lse = cp.forward(qkv, B, Tl, H, D)
        ctx.save_for_backward(qkv, o, lse)
        ctx.cp, ctx.shape = cp, (B, Tl, H, D)
        return o

    @staticmethod
    def backward(ctx, do):
        qkv, o, lse = ctx.saved_tensors
        return ctx.cp.backward(qkv, o, lse, do.contiguous(), *ctx.shape), None, None, None, None, None


def enable_context_parallel(engine, seq_len: int, group=None) -> ContextParallelAttention:
    """Run `engine` (an LMEngine) on this rank's zigzag shard of `seq_len`-token
    sequences: attention spans the whole group, position embeddings use the
    tokens' global positions.  Feed it ``shard_sequence(ids / targets)`` and
    average its gradients over the group (e.g. with the data-parallel
    all-reduce, whose group then contains the context group)."""
    if not engine.causal:
        raise ValueError("context parallelism is implemented for causal attention")
    if seq_len > engine.spec.max_seq_len:
        raise ValueError(f"sequence length {seq_len} exceeds max_seq_len {engine.spec.max_seq_len}")
    cp = ContextParallelAttention(group)
    engine.context_attention = cp
    engine.positions = zigzag_positions(cp.rank, cp.size, seq_len, device=engine.E.device)
    return cp
