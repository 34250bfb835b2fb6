"""Thin, allocation-explicit wrappers around the sm_100a kernels.

Each function takes torch tensors that already live on the current CUDA
device, allocates its outputs with the PyTorch caching allocator (so the calls
are CUDA-graph capturable) and launches exactly the native kernel(s) named in
its docstring on the current stream.
"""

from __future__ import annotations

import math
import os

import torch

from underhfs_b200.ops._lib import DT_BF16, DT_F32, core, dt, ptr, stream

# GEMM epilogues (csrc/kernels/gemm.h)
EPI_BF16, EPI_BIAS_GELU, EPI_RESID, EPI_DGELU, EPI_F32_ACCUM, EPI_F32_STORE = range(6)
NUM_SMS = 148

OP_ADD, OP_MUL, OP_SUB, OP_DIV = range(4)


def _check_cuda(*ts: torch.Tensor | None) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("native kernel requires CUDA tensors")


# --------------------------------------------------------------------- GEMM
def gemm_raw(
    M: int,
    N: int,
    K: int,
    a: torch.Tensor,
    lda: int,
    a_mn: bool,
    b: torch.Tensor,
    ldb: int,
    b_mn: bool,
    c: torch.Tensor,
    ldc: int,
    epi: int = EPI_BF16,
    bias: torch.Tensor | None = None,
    aux: torch.Tensor | None = None,
    ld_aux: int = 0,
    aux_out: torch.Tensor | None = None,
    ld_aux_out: int = 0,
    splits: int = 1,
    block_n: int = 0,
    cta_pair: int = -1,
) -> None:
    """tcgen05 GEMM: C[M,N] (op)= sum_k A(m,k) B(n,k) with a fused epilogue.

    ``cta_pair``: -1 lets the launcher choose between 128 x N tiles on one SM
    and 256 x 256 tiles on a CTA pair (two SMs of a TPC); 0 / 1 force it
    (1 only takes effect where the pair kernel supports the problem).

    When a B-gather resolver is installed (ZeRO-3 with fused gathers) and B
    lives in a gather slot, the launch carries the all-gather of B's rows.
    """
    ag = _b_gather(b, b_mn) if _b_gather is not None else None
    if ag is not None:
        core().gemm_ag(
            M, N, K, ptr(a), lda, a_mn, ptr(b), ldb, b_mn, ptr(c), ldc, epi, ptr(bias), ptr(aux), ld_aux,
            ptr(aux_out), ld_aux_out, splits, *ag, stream(),
        )
        return
    core().gemm(
        M, N, K, ptr(a), lda, a_mn, ptr(b), ldb, b_mn, ptr(c), ldc, epi, ptr(bias), ptr(aux), ld_aux,
        ptr(aux_out), ld_aux_out, splits, block_n, cta_pair, stream(),
    )


# ZeRO-3 hook: callable (b_tensor, b_mn) -> gather arguments for gemm_ag or None
_b_gather = None


def set_b_gather(resolver) -> None:
    """Install (or clear with None) the resolver that attaches a fused
    all-gather to GEMMs whose B operand is a gathered weight."""
    global _b_gather
    _b_gather = resolver


def _splits_for(tiles: int, k: int) -> int:
    kb = max(1, math.ceil(k / 64))
    want = max(1, math.ceil(2 * NUM_SMS / max(1, tiles)))
    return max(1, min(want, kb // 4 if kb >= 8 else 1))


def linear_fwd(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    """y[M,N] = x[M,K] w[N,K]^T (+ bias)  -- one tcgen05 GEMM (both K-major)."""
    M, K = x.shape
    N = w.shape[0]
    y = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    gemm_raw(M, N, K, x, x.stride(0), False, w, w.stride(0), False, y, N, EPI_BF16, bias=bias)
    return y


def linear_fwd_resid(x, w, bias, resid, out=None):
    """out = resid + x w^T + bias (residual add fused into the epilogue)."""
    M, K = x.shape
    N = w.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    gemm_raw(M, N, K, x, x.stride(0), False, w, w.stride(0), False, out, N, EPI_RESID, bias=bias, aux=resid,
             ld_aux=resid.stride(0))
    return out


def linear_fwd_gelu(x, w, bias):
    """(u, g): u = x w^T + bias (kept for backward), g = gelu_tanh(u) -- one GEMM."""
    M, K = x.shape
    N = w.shape[0]
    g = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    u = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    gemm_raw(M, N, K, x, x.stride(0), False, w, w.stride(0), False, g, N, EPI_BIAS_GELU, bias=bias,
             aux_out=u, ld_aux_out=N)
    return u, g


def linear_dgrad(dy: torch.Tensor, w: torch.Tensor, gelu_in: torch.Tensor | None = None) -> torch.Tensor:
    """dx[M,K] = dy[M,N] w[N,K]; with `gelu_in`: dx *= gelu'(gelu_in) in the epilogue."""
    M, N = dy.shape
    K = w.shape[1]
    dx = torch.empty((M, K), dtype=torch.bfloat16, device=dy.device)
    if gelu_in is None:
        gemm_raw(M, K, N, dy, dy.stride(0), False, w, w.stride(0), True, dx, K, EPI_BF16)
    else:
        gemm_raw(M, K, N, dy, dy.stride(0), False, w, w.stride(0), True, dx, K, EPI_DGELU, aux=gelu_in,
                 ld_aux=gelu_in.stride(0))
    return dx


# UHFS_WGRAD_SPLITS=<n>: weight gradients as classic split-K with n splits
# (split-major unit order) instead of stream-K, for comparisons
_WGRAD_SPLITS = int(os.environ.get("UHFS_WGRAD_SPLITS", "0") or 0)


def linear_wgrad_accum(dy: torch.Tensor, x: torch.Tensor, dw32: torch.Tensor, splits: int = 0) -> None:
    """dw32[N,K] += dy[M,N]^T x[M,K]  (fp32, atomic accumulation).

    splits=0 runs stream-K: every CTA takes an equal share of the
    (tile, k-block) work and accumulates partial tiles, so the grid stays full
    whatever the tile count; splits>=1 is classic split-K.
    """
    M, N = dy.shape
    K = x.shape[1]
    if splits == 0 and _WGRAD_SPLITS:
        splits = _WGRAD_SPLITS
    if splits == 0 and math.ceil(N / 128) * math.ceil(K / 256) >= 4 * NUM_SMS:
        splits = 1  # enough tiles for >= 4 full waves: plain tiles keep better L2 reuse
    gemm_raw(N, K, M, dy, dy.stride(0), True, x, x.stride(0), True, dw32, dw32.stride(0), EPI_F32_ACCUM,
             splits=splits)


def matmul_bf16(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """c[M,N] = a[M,K] b[K,N] for bf16 row-major operands (B read MN-major)."""
    M, K = a.shape
    N = b.shape[1]
    c = torch.empty((M, N), dtype=torch.bfloat16, device=a.device)
    gemm_raw(M, N, K, a, a.stride(0), False, b, b.stride(0), True, c, N, EPI_BF16)
    return c


# fp32 products at least this large (M, N and K) run as 3xTF32 on the
# tensor cores; smaller ones (and UHFS_F32_GEMM=simt) on the SIMT kernel
_F32_TC_MIN = 256
_F32_GEMM = os.environ.get("UHFS_F32_GEMM", "auto")


def matmul_f32(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """fp32 c = a @ b.  Large products: three tf32 tensor-core products per
    term (hi*hi + hi*lo + lo*hi of a tf32 split, fp32 accumulation), within a
    few fp32 ulps of the exact dot product; small ones: exact SIMT FMA."""
    a = a.contiguous()
    b = b.contiguous()
    M, K = a.shape
    N = b.shape[1]
    c = torch.empty((M, N), dtype=torch.float32, device=a.device)
    if _F32_GEMM != "simt" and min(M, N, K) >= _F32_TC_MIN and N % 4 == 0:
        kp = (K + 31) // 32 * 32
        ws_a = torch.empty((M, 3 * kp), dtype=torch.float32, device=a.device)
        ws_b = torch.empty((N, 3 * kp), dtype=torch.float32, device=a.device)
        core().gemm_f32_3xtf32(ptr(a), ptr(b), ptr(c), M, N, K, False, ptr(ws_a), ptr(ws_b), stream())
        return c
    core().gemm_f32(ptr(a), ptr(b), ptr(c), M, N, K, False, stream())
    return c


# -------------------------------------------------------------- elementwise
def ew_binary(op: int, a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    out = torch.empty_like(a)
    core().ew_binary(op, dt(a), ptr(a), ptr(b), ptr(out), a.numel(), stream())
    return out


def ew_scalar(op: int, a: torch.Tensor, s: float) -> torch.Tensor:
    out = torch.empty_like(a)
    core().ew_scalar(op, dt(a), ptr(a), float(s), ptr(out), a.numel(), stream())
    return out


def cast(src: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    out = torch.empty(src.shape, dtype=dtype, device=src.device)
    core().cast(dt(src), dt(out), ptr(src), ptr(out), src.numel(), stream())
    return out


def reduce_sum(x: torch.Tensor) -> torch.Tensor:
    """fp32 scalar sum in one deterministic launch."""
    c = core()
    nparts = c.reduce_sum_partials()
    scratch = torch.zeros(nparts + 2, dtype=torch.float32, device=x.device)
    out = torch.empty((), dtype=torch.float32, device=x.device)
    counter = scratch[nparts:]
    c.reduce_sum(dt(x), ptr(x), x.numel(), ptr(out), ptr(scratch), ptr(counter), stream())
    return out


def gelu(x: torch.Tensor) -> torch.Tensor:
    y = torch.empty_like(x)
    core().gelu_fwd(dt(x), ptr(x), ptr(y), x.numel(), stream())
    return y


def gelu_backward(x: torch.Tensor, dy: torch.Tensor) -> torch.Tensor:
    dx = torch.empty_like(x)
    core().gelu_bwd(dt(x), ptr(x), ptr(dy), ptr(dx), x.numel(), stream())
    return dx


def colsum_accum(x: torch.Tensor, out32: torch.Tensor) -> None:
    """out32[N] += sum over rows of bf16 x[M,N]."""
    M, N = x.shape
    core().colsum_accum(ptr(x), x.stride(0), ptr(out32), M, N, stream())


# --------------------------------------------------------------------- rows
def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    rows, cols = x.shape
    y = torch.empty_like(x)
    rstd = torch.empty((rows,), dtype=torch.float32, device=x.device)
    core().rmsnorm_fwd(dt(x), ptr(x), ptr(w), ptr(y), ptr(rstd), rows, cols, float(eps), stream())
    return y, rstd


def rmsnorm_backward(dy, x, w, rstd, dres=None, dw32=None):
    rows, cols = x.shape
    dx = torch.empty_like(x)
    core().rmsnorm_bwd(dt(x), ptr(dy), ptr(x), ptr(w), ptr(rstd), ptr(dres), ptr(dx), ptr(dw32), rows, cols,
                       stream())
    return dx


def embedding(ids: torch.Tensor, tok: torch.Tensor, pos: torch.Tensor | None, seq_len: int) -> torch.Tensor:
    rows = ids.numel()
    dim = tok.shape[1]
    out = torch.empty((rows, dim), dtype=tok.dtype, device=tok.device)
    core().embedding_fwd(dt(tok), ptr(ids), ptr(tok), ptr(pos), ptr(out), rows, dim, seq_len, stream(),
                         tok.shape[0])
    return out


def embedding_backward(ids, dout, dtok32, dpos32, seq_len):
    rows, dim = dout.shape
    vocab = dtok32.shape[0] if dtok32 is not None else 0
    core().embedding_bwd(dt(dout), ptr(ids), ptr(dout), ptr(dtok32), ptr(dpos32), rows, dim, seq_len, stream(),
                         vocab)


def softmax_cross_entropy(logits: torch.Tensor, targets: torch.Tensor, dlogits: torch.Tensor | None,
                          grad_scale: float, grad_scale_t: torch.Tensor | None = None) -> torch.Tensor:
    """Per-row NLL (fp32); when `dlogits` is given it receives
    (p - onehot) * grad_scale (* grad_scale_t, a device fp32 scalar, when given)."""
    rows, cols = logits.shape
    loss_rows = torch.empty((rows,), dtype=torch.float32, device=logits.device)
    if grad_scale_t is not None and grad_scale_t.dtype != torch.float32:
        grad_scale_t = grad_scale_t.float()
    core().softmax_ce(dt(logits), ptr(logits), logits.stride(0), ptr(targets), ptr(loss_rows), ptr(dlogits), rows,
                      cols, float(grad_scale), ptr(grad_scale_t), stream())
    return loss_rows


def softmax_rows(x: torch.Tensor) -> torch.Tensor:
    x = x.contiguous()
    rows, cols = x.reshape(-1, x.shape[-1]).shape
    y = torch.empty_like(x)
    core().softmax_rows(dt(x), ptr(x), ptr(y), rows, cols, stream())
    return y


def softmax_rows_backward(y: torch.Tensor, dy: torch.Tensor) -> torch.Tensor:
    rows, cols = y.reshape(-1, y.shape[-1]).shape
    dx = torch.empty_like(y)
    core().softmax_rows_bwd(dt(y), ptr(y), ptr(dy.contiguous()), ptr(dx), rows, cols, stream())
    return dx


# ---------------------------------------------------------------- attention
def flash_attn_qkv(qkv: torch.Tensor, B: int, T: int, H: int, D: int, causal: bool, scale: float | None = None):
    """Attention over a fused [B*T, 3*H*D] projection; returns (o [B*T, H*D], lse [B,H,T])."""
    F = H * D
    scale = (1.0 / math.sqrt(D)) if scale is None else scale
    o = torch.empty((B * T, F), dtype=torch.bfloat16, device=qkv.device)
    lse = torch.empty((B, H, T), dtype=torch.float32, device=qkv.device)
    base = qkv.data_ptr()
    st = qkv.stride(0)
    core().flash_attn_fwd(base, base + 2 * F, base + 4 * F, ptr(o), ptr(lse), T * st, st, T * st, st, T * st, st,
                          T * F, F, B, H, T, D, float(scale), bool(causal), stream())
    return o, lse


def flash_attn_qkv_backward(qkv, o, lse, do, B, T, H, D, causal, scale=None):
    F = H * D
    scale = (1.0 / math.sqrt(D)) if scale is None else scale
    dqkv = torch.empty((B * T, 3 * F), dtype=torch.bfloat16, device=qkv.device)
    delta = torch.empty((B, H, T), dtype=torch.float32, device=qkv.device)
    dq_acc = torch.empty((B * T, F), dtype=torch.float32, device=qkv.device)
    base = qkv.data_ptr()
    dbase = dqkv.data_ptr()
    st = qkv.stride(0)
    do = do.contiguous()
    core().flash_attn_bwd(
        base, base + 2 * F, base + 4 * F, ptr(o), ptr(lse), ptr(do), dbase, dbase + 2 * F, dbase + 4 * F,
        ptr(delta), ptr(dq_acc),
        T * st, st, T * st, st, T * st, st, T * F, F, T * F, F,
        T * 3 * F, 3 * F, T * 3 * F, 3 * F, T * 3 * F, 3 * F,
        B, H, T, D, float(scale), bool(causal), stream(),
    )
    return dqkv


def attention_f32(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float, causal: bool) -> torch.Tensor:
    """Reference-contract single-head fp32 attention, q/k/v [T, F]."""
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    T, F = q.shape
    out = torch.empty_like(q)
    core().attention_f32(ptr(q), ptr(k), ptr(v), ptr(out), T, F, float(scale), bool(causal), stream())
    return out


# -------------------------------------------------------------------- AdamW
def adamw_(p32, g, m, v, p16, *, lr, beta1, beta2, eps, weight_decay, decoupled, grad_scale=1.0, step=1,
           step_t=None, lr_t=None):
    """In-place fused AdamW over flat fp32 state (g fp32 or bf16); writes bf16 copy if p16."""
    core().adamw(ptr(p32), ptr(g), ptr(m), ptr(v), ptr(p16), p32.numel(), float(lr), float(beta1), float(beta2),
                 float(eps), float(weight_decay), bool(decoupled), float(grad_scale), int(step), ptr(step_t),
                 ptr(lr_t), g.dtype == torch.bfloat16, stream())


def increment_(counter: torch.Tensor) -> None:
    core().increment_counter(ptr(counter), stream())


# ------------------------------------------------------------------- conv2d
def conv2d_fwd(x, w, b, stride, padding):
    """fp32 NCHW conv2d as an implicit GEMM (csrc/kernels/conv_igemm.cu)."""
    x, w = x.contiguous(), w.contiguous()
    b = b.contiguous() if b is not None else None
    N, C, H, W = x.shape
    K, _, R, S = w.shape
    sh, sw = stride
    ph, pw = padding
    P = (H + 2 * ph - R) // sh + 1
    Q = (W + 2 * pw - S) // sw + 1
    y = torch.empty((N, K, P, Q), dtype=torch.float32, device=x.device)
    core().conv2d_fwd(ptr(x), ptr(w), ptr(b), ptr(y), N, C, H, W, K, R, S, sh, sw, ph, pw, P, Q, stream())
    return y


def conv2d_bwd(dy, x, w, stride, padding, need_bias):
    N, C, H, W = x.shape
    K, _, R, S = w.shape
    sh, sw = stride
    ph, pw = padding
    P, Q = dy.shape[2], dy.shape[3]
    dy, x, w = dy.contiguous(), x.contiguous(), w.contiguous()
    dx = torch.empty_like(x)
    dw = torch.empty_like(w)
    db = torch.empty((K,), dtype=torch.float32, device=x.device) if need_bias else None
    c = core()
    c.conv2d_dgrad(ptr(dy), ptr(w), ptr(dx), N, C, H, W, K, R, S, sh, sw, ph, pw, P, Q, stream())
    c.conv2d_wgrad(ptr(dy), ptr(x), ptr(dw), ptr(db), N, C, H, W, K, R, S, sh, sw, ph, pw, P, Q, stream())
    return dx, dw, db


__all__ = [name for name in dir() if not name.startswith("_")] + ["DT_BF16", "DT_F32"]
