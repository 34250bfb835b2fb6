"""torch.autograd Functions whose forward and backward are native kernels.

These back the generic Tensor / nn API on CUDA tensors (the TransformerLM
training path uses the fused engine in models/transformer.py instead).
Each Function launches only kernels from ``underhfs_b200._core``.
"""

from __future__ import annotations

import math

import torch

from underhfs_b200.ops import kernels as K

_OPS = {"add": K.OP_ADD, "mul": K.OP_MUL, "sub": K.OP_SUB, "div": K.OP_DIV}


class _Ew(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a, b, op):
        ctx.op = op
        if op == "mul":
            ctx.save_for_backward(a, b)
        return K.ew_binary(_OPS[op], a.contiguous(), b.contiguous())

    @staticmethod
    def backward(ctx, g):
        g = g.contiguous()
        if ctx.op == "add":
            return g, g, None
        a, b = ctx.saved_tensors
        ga = K.ew_binary(K.OP_MUL, g, b) if ctx.needs_input_grad[0] else None
        gb = K.ew_binary(K.OP_MUL, g, a) if ctx.needs_input_grad[1] else None
        return ga, gb, None


def ew(op: str, a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    return _Ew.apply(a, b, op)


def _mm(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """a[M,K] @ b[K,N] with native kernels: tcgen05 for bf16 (aligned shapes),
    exact-fp32 SIMT otherwise (fp16 is computed in fp32 and rounded)."""
    if a.dtype == torch.bfloat16 and a.shape[1] % 8 == 0 and b.shape[1] % 8 == 0:
        return K.matmul_bf16(a.contiguous(), b.contiguous())
    if a.dtype == torch.float32:
        return K.matmul_f32(a, b)
    out = K.matmul_f32(K.cast(a.contiguous(), torch.float32), K.cast(b.contiguous(), torch.float32))
    return K.cast(out, a.dtype)


class _Matmul(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a, b):
        ctx.save_for_backward(a, b)
        return _mm(a, b)

    @staticmethod
    def backward(ctx, g):
        a, b = ctx.saved_tensors
        ga = _mm(g.contiguous(), b.t().contiguous()) if ctx.needs_input_grad[0] else None
        gb = _mm(a.t().contiguous(), g.contiguous()) if ctx.needs_input_grad[1] else None
        return ga, gb


def matmul(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    return _Matmul.apply(a, b)


class _SumAll(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x):
        ctx.shape = x.shape
        ctx.dtype = x.dtype
        return K.reduce_sum(x.contiguous()).to(x.dtype)

    @staticmethod
    def backward(ctx, g):
        return g.expand(ctx.shape).contiguous()


def sum_all(x: torch.Tensor) -> torch.Tensor:
    return _SumAll.apply(x)


class _Softmax(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x):
        y = K.softmax_rows(x.contiguous())
        ctx.save_for_backward(y)
        return y

    @staticmethod
    def backward(ctx, g):
        (y,) = ctx.saved_tensors
        return K.softmax_rows_backward(y, g)


def softmax(x: torch.Tensor) -> torch.Tensor:
    return _Softmax.apply(x)


# --------------------------------------------------------------- nn layers
class _Linear(torch.autograd.Function):
    """y = x W^T + b for bf16 2-D x (tcgen05 GEMMs in both directions)."""

    @staticmethod
    def forward(ctx, x, w, b):
        ctx.save_for_backward(x, w)
        ctx.has_bias = b is not None
        return K.linear_fwd(x, w, b)

    @staticmethod
    def backward(ctx, g):
        x, w = ctx.saved_tensors
        g = g.contiguous()
        gx = K.linear_dgrad(g, w) if ctx.needs_input_grad[0] else None
        gw = gb = None
        if ctx.needs_input_grad[1]:
            acc = torch.zeros(w.shape, dtype=torch.float32, device=w.device)
            K.linear_wgrad_accum(g, x, acc)
            gw = acc.to(w.dtype)
        if ctx.has_bias and ctx.needs_input_grad[2]:
            acc = torch.zeros(w.shape[0], dtype=torch.float32, device=w.device)
            K.colsum_accum(g, acc)
            gb = acc.to(w.dtype)
        return gx, gw, gb


class _LinearF32(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, b):
        ctx.save_for_backward(x, w)
        ctx.has_bias = b is not None
        y = _mm(x, w.t().contiguous())
        if b is not None:
            y = K.ew_binary(K.OP_ADD, y, b.expand_as(y).contiguous())
        return y

    @staticmethod
    def backward(ctx, g):
        x, w = ctx.saved_tensors
        g = g.contiguous()
        gx = _mm(g, w) if ctx.needs_input_grad[0] else None
        gw = _mm(g.t().contiguous(), x) if ctx.needs_input_grad[1] else None
        gb = None
        if ctx.has_bias and ctx.needs_input_grad[2]:
            gb = K.reduce_sum(g) if g.shape[1] == 1 else g.sum(0)
            gb = gb.reshape(w.shape[0])
        return gx, gw, gb


def linear(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None) -> torch.Tensor:
    shape = x.shape
    x2 = x.reshape(-1, shape[-1]).contiguous()
    if x.dtype == torch.bfloat16 and shape[-1] % 8 == 0 and w.shape[0] % 8 == 0:
        y = _Linear.apply(x2, w.contiguous(), b)
    else:
        y = _LinearF32.apply(x2, w.contiguous(), b)
    return y.reshape(*shape[:-1], w.shape[0])


class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps):
        y, rstd = K.rmsnorm(x, w, eps)
        ctx.save_for_backward(x, w, rstd)
        return y

    @staticmethod
    def backward(ctx, g):
        x, w, rstd = ctx.saved_tensors
        dw = torch.zeros(w.shape, dtype=torch.float32, device=w.device)
        dx = K.rmsnorm_backward(g.contiguous(), x, w, rstd, None, dw)
        return dx, dw.to(w.dtype), None


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    shape = x.shape
    y = _RMSNorm.apply(x.reshape(-1, shape[-1]).contiguous(), w.contiguous(), eps)
    return y.reshape(shape)


class _Gelu(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x):
        ctx.save_for_backward(x)
        return K.gelu(x)

    @staticmethod
    def backward(ctx, g):
        (x,) = ctx.saved_tensors
        return K.gelu_backward(x, g.contiguous())


def gelu(x: torch.Tensor) -> torch.Tensor:
    return _Gelu.apply(x.contiguous())


class _Embedding(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ids, w):
        ctx.save_for_backward(ids)
        ctx.wshape = w.shape
        ctx.wdtype = w.dtype
        return K.embedding(ids, w.contiguous(), None, 1)

    @staticmethod
    def backward(ctx, g):
        (ids,) = ctx.saved_tensors
        acc = torch.zeros(ctx.wshape, dtype=torch.float32, device=g.device)
        K.embedding_backward(ids, g.contiguous(), acc, None, 1)
        return None, acc.to(ctx.wdtype)


def embedding(ids: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    flat = ids.reshape(-1).to(torch.int64).contiguous()
    out = _Embedding.apply(flat, w)
    return out.reshape(*ids.shape, w.shape[1])


class _CrossEntropy(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, targets, reduction):
        rows = logits.shape[0]
        loss_rows = K.softmax_cross_entropy(logits, targets, None, 1.0)
        ctx.save_for_backward(logits, targets)
        ctx.reduction = reduction
        if reduction == "none":
            return loss_rows.to(logits.dtype)
        total = K.reduce_sum(loss_rows)
        if reduction == "mean":
            total = K.ew_scalar(K.OP_MUL, total.reshape(1), 1.0 / max(1, rows)).reshape(())
        return total.to(logits.dtype)

    @staticmethod
    def backward(ctx, g):
        logits, targets = ctx.saved_tensors
        rows = logits.shape[0]
        dl = torch.empty_like(logits)
        if ctx.reduction == "none":
            # per-row scales: (p - onehot) * g[r]
            K.softmax_cross_entropy(logits, targets, dl, 1.0)
            dl = dl * g.reshape(rows, 1).to(dl.dtype)
        else:
            scale = 1.0 / max(1, rows) if ctx.reduction == "mean" else 1.0
            K.softmax_cross_entropy(logits, targets, dl, scale, g.reshape(()).float().contiguous())
        return dl, None, None


def cross_entropy(logits: torch.Tensor, targets: torch.Tensor, reduction: str = "mean") -> torch.Tensor:
    return _CrossEntropy.apply(logits.contiguous(), targets.reshape(-1).to(torch.int64).contiguous(), reduction)


class _FlashAttention(torch.autograd.Function):
    """Causal/full multi-head attention over a fused qkv [B*T, 3*H*D] bf16 tensor."""

    @staticmethod
    def forward(ctx, qkv, B, T, H, D, causal):
        o, lse = K.flash_attn_qkv(qkv, B, T, H, D, causal)
        ctx.save_for_backward(qkv, o, lse)
        ctx.dims = (B, T, H, D, causal)
        return o

    @staticmethod
    def backward(ctx, do):
        qkv, o, lse = ctx.saved_tensors
        B, T, H, D, causal = ctx.dims
        return K.flash_attn_qkv_backward(qkv, o, lse, do.contiguous(), B, T, H, D, causal), None, None, None, None, None


def flash_attention(qkv: torch.Tensor, B: int, T: int, H: int, D: int, causal: bool) -> torch.Tensor:
    return _FlashAttention.apply(qkv.contiguous(), B, T, H, D, causal)


class _AttentionF32(torch.autograd.Function):
    """Reference-contract single-head fp32 attention (inference kernel; the
    backward recomputes with the row-softmax kernels)."""

    @staticmethod
    def forward(ctx, q, k, v, scale, causal):
        ctx.save_for_backward(q, k, v)
        ctx.scale, ctx.causal = scale, causal
        return K.attention_f32(q, k, v, scale, causal)

    @staticmethod
    def backward(ctx, g):
        q, k, v = ctx.saved_tensors
        s = K.matmul_f32(q, k.t().contiguous()) * ctx.scale
        if ctx.causal:
            T = q.shape[0]
            s = s.masked_fill(torch.triu(torch.ones(T, T, dtype=torch.bool, device=q.device), 1), float("-inf"))
        p = K.softmax_rows(s)
        g = g.contiguous()
        dv = K.matmul_f32(p.t().contiguous(), g)
        dp = K.matmul_f32(g, v.t().contiguous())
        ds = K.softmax_rows_backward(p, dp) * ctx.scale
        dq = K.matmul_f32(ds, k)
        dk = K.matmul_f32(ds.t().contiguous(), q)
        return dq, dk, dv, None, None


def attention_f32(q, k, v, scale: float, causal: bool) -> torch.Tensor:
    return _AttentionF32.apply(q.contiguous(), k.contiguous(), v.contiguous(), scale, causal)


class _Conv2d(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, b, stride, padding):
        ctx.save_for_backward(x, w)
        ctx.cfg = (stride, padding, b is not None)
        return K.conv2d_fwd(x.contiguous(), w.contiguous(), b, stride, padding)

    @staticmethod
    def backward(ctx, g):
        x, w = ctx.saved_tensors
        stride, padding, has_b = ctx.cfg
        dx, dw, db = K.conv2d_bwd(g, x.contiguous(), w.contiguous(), stride, padding, has_b)
        return dx, dw, db, None, None


def conv2d(x, w, b, stride, padding):
    return _Conv2d.apply(x, w, b, stride, padding)


def _unused() -> None:  # keeps math imported for type checkers of callers
    math.sqrt(1.0)
