"""B200 training engine for the TransformerLM family.

Same architecture as the reference TransformerLM (nn.py:274-334: token +
learned position embedding, pre-norm blocks ``x += attn(rms(x)); x +=
mlp(rms(x))``, final RMSNorm, linear head), generalised to a batch dimension,
multi-head causal attention and optionally tied embeddings, and executed as a
fixed sequence of sm_100a kernels on flat bf16 parameters:

forward, per block (7 launches + attention):
    rmsnorm -> QKV GEMM(+bias) -> flash attention -> out-proj GEMM(+bias+residual)
    -> rmsnorm -> FC1 GEMM(+bias, GELU, pre-activation kept) -> FC2 GEMM(+bias+residual)
backward, per block:
    FC2 dgrad GEMM with the GELU derivative fused into its epilogue, weight
    gradients as split-K GEMMs accumulating in fp32 straight into the flat
    gradient buffer, bias gradients as column sums, RMSNorm backward with the
    residual gradient added in the same pass, flash-attention backward.
The loss is a fused softmax-cross-entropy over the vocabulary that also emits
the logits gradient.

After each block's gradients are complete the engine calls
``grad_ready(lo, hi)`` with the flat-buffer range that just became final, so
a data-parallel wrapper can start reducing that bucket while the remaining
blocks run backward.
"""

from __future__ import annotations

import math
import os
from dataclasses import dataclass
from typing import Callable

import torch

from underhfs_b200.ops import kernels as K
from underhfs_b200.parallel.flat import FlatBuffers, FlatLayout
from underhfs_b200.utils import nvtx


@dataclass(frozen=True)
class LMSpec:
    vocab_size: int
    max_seq_len: int
    features: int
    hidden_features: int
    layers: int
    heads: int = 1
    tied: bool = False
    eps: float = 1e-8
    bias: bool = True

    @property
    def head_dim(self) -> int:
        return self.features // self.heads

    def num_params(self) -> int:
        F, Hd, V = self.features, self.hidden_features, self.vocab_size
        per_block = 2 * F + 4 * F * F + (4 * F if self.bias else 0) + 2 * F * Hd + (Hd + F if self.bias else 0)
        n = V * F + self.max_seq_len * F + self.layers * per_block + F
        if not self.tied:
            n += V * F
        return n

    def activation_bytes(self, batch: int, seq_len: int) -> int:
        """Device bytes the engine keeps for one training step's backward:
        per token and block the bf16 tensors saved by the forward (x, rmsnorm
        out, qkv, attention out, x1, rmsnorm out: 8F; fc1 pre- and
        post-activation: 2 x hidden) plus the bf16 logits / logits gradient and
        a transient of two blocks' worth of gradients of the activations."""
        tokens = batch * seq_len
        per_block = 2 * (8 * self.features + 2 * self.hidden_features)
        transient = 2 * 2 * (4 * self.features + self.hidden_features)
        return int(tokens * (self.layers * per_block + 2 * self.vocab_size + transient))

    def train_flops_per_token(self, seq_len: int) -> float:
        """6N for the dense weights + causal attention (fwd 2 matmuls, bwd 4)."""
        dense = 6.0 * (self.num_params() - self.vocab_size * self.features - self.max_seq_len * self.features)
        dense += 6.0 * self.vocab_size * self.features  # head (tied or not)
        attn = self.layers * 3 * 2 * 2 * seq_len * self.features / 2  # causal half
        return dense + attn


def param_names(spec: LMSpec) -> list[tuple[str, tuple[int, ...]]]:
    """Reference-compatible parameter names (TransformerLM named_parameters)."""
    F, Hd, V = spec.features, spec.hidden_features, spec.vocab_size
    out: list[tuple[str, tuple[int, ...]]] = [
        ("token_embedding.weight", (V, F)),
        ("position_embedding.weight", (spec.max_seq_len, F)),
    ]
    for i in range(spec.layers):
        p = f"blocks.{i}."
        out.append((p + "attn_norm.weight", (F,)))
        for proj in ("q_proj", "k_proj", "v_proj", "out_proj"):
            out.append((p + f"attn.{proj}.weight", (F, F)))
            if spec.bias:
                out.append((p + f"attn.{proj}.bias", (F,)))
        out.append((p + "mlp_norm.weight", (F,)))
        out.append((p + "mlp.net.0.weight", (Hd, F)))
        if spec.bias:
            out.append((p + "mlp.net.0.bias", (Hd,)))
        out.append((p + "mlp.net.2.weight", (F, Hd)))
        if spec.bias:
            out.append((p + "mlp.net.2.bias", (F,)))
    out.append(("norm.weight", (F,)))
    if not spec.tied:
        out.append(("head.weight", (V, F)))
    return out


def build_layout(spec: LMSpec) -> FlatLayout:
    """Flat layout in forward order; q/k/v weights (and biases) are adjacent so
    the fused QKV GEMM reads them as one [3F, F] matrix."""
    F, Hd, V = spec.features, spec.hidden_features, spec.vocab_size
    lay = FlatLayout()
    lay.add("token_embedding.weight", (V, F))
    lay.add("position_embedding.weight", (spec.max_seq_len, F))
    for i in range(spec.layers):
        p = f"blocks.{i}."
        lay.add(p + "attn_norm.weight", (F,))
        lay.add_group([(p + f"attn.{x}_proj.weight", (F, F)) for x in "qkv"])
        if spec.bias:
            lay.add_group([(p + f"attn.{x}_proj.bias", (F,)) for x in "qkv"])
        lay.add(p + "attn.out_proj.weight", (F, F))
        if spec.bias:
            lay.add(p + "attn.out_proj.bias", (F,))
        lay.add(p + "mlp_norm.weight", (F,))
        lay.add(p + "mlp.net.0.weight", (Hd, F))
        if spec.bias:
            lay.add(p + "mlp.net.0.bias", (Hd,))
        lay.add(p + "mlp.net.2.weight", (F, Hd))
        if spec.bias:
            lay.add(p + "mlp.net.2.bias", (F,))
    lay.add("norm.weight", (F,))
    if not spec.tied:
        lay.add("head.weight", (V, F))
    return lay


def init_reference_lcg(shape: tuple[int, ...], bound: float) -> torch.Tensor:
    """The reference's deterministic initializer (tensor.py:1076-1088):
    value_i = (((i*1103515245 + 12345) % 10000) / 5000 - 1) * bound, vectorised."""
    n = 1
    for d in shape:
        n *= d
    i = torch.arange(n, dtype=torch.int64)
    v = ((i * 1103515245 + 12345) % 10000).to(torch.float64) / 5000.0 - 1.0
    return (v * bound).to(torch.float32).reshape(shape)


def initial_value(spec: LMSpec, name: str, shape: tuple[int, ...], init: str, gen: torch.Generator) -> torch.Tensor:
    if name.endswith("norm.weight"):
        return torch.ones(shape)
    if name.endswith(".bias"):
        return torch.zeros(shape)
    if init == "reference":
        rows, cols = shape
        return init_reference_lcg(shape, math.sqrt(6.0 / max(1, rows + cols)))
    std = 0.02
    if name.endswith("out_proj.weight") or name.endswith("mlp.net.2.weight"):
        std = 0.02 / math.sqrt(2 * spec.layers)
    return torch.randn(shape, generator=gen) * std


_SIDE_STREAMS: dict = {}


# UNDERHFS_WGRAD_SIDE=0 keeps the weight-gradient GEMMs on the compute stream
_WGRAD_SIDE = os.environ.get("UNDERHFS_WGRAD_SIDE", "1") != "0"


def _side_stream(device) -> torch.cuda.Stream:
    """One side stream per device for work that runs beside the backward."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    key = dev.index if dev.index is not None else torch.cuda.current_device()
    st = _SIDE_STREAMS.get(key)
    if st is None:
        st = _SIDE_STREAMS[key] = torch.cuda.Stream(device=torch.device("cuda", key))
    return st


class LMEngine:
    """Forward/backward of one TransformerLM over flat buffers, on the current stream."""

    # context parallelism (parallel/context.py): attention over the group's
    # sequence shards and the global positions of this rank's tokens; class
    # defaults so engines that build their own state (ZeRO-3) inherit them
    context_attention = None
    positions: torch.Tensor | None = None

    def __init__(self, spec: LMSpec, flat: FlatBuffers, *, causal: bool = True) -> None:
        if spec.features % spec.heads != 0:
            raise ValueError("features must be divisible by heads")
        if spec.head_dim not in (64, 128):
            raise ValueError("the flash-attention kernels support head_dim 64 or 128")
        self.spec = spec
        self.flat = flat
        self.causal = causal
        self.grad_ready: Callable[[int, int], None] | None = None
        self._saved: dict | None = None
        F = spec.features
        self.blocks = []
        for i in range(spec.layers):
            p = f"blocks.{i}."
            lo, _ = flat.span(p + "attn_norm.weight", p + "attn_norm.weight")
            _, hi = flat.span(p + "mlp_norm.weight", p + ("mlp.net.2.bias" if spec.bias else "mlp.net.2.weight"))
            qkv_off = flat.by_name[p + "attn.q_proj.weight"].offset
            blk = {
                "ln1": flat.param(p + "attn_norm.weight"),
                "g_ln1": flat.grad(p + "attn_norm.weight"),
                "Wqkv": flat.params[qkv_off : qkv_off + 3 * F * F].view(3 * F, F),
                "gWqkv": flat.grads[qkv_off : qkv_off + 3 * F * F].view(3 * F, F),
                "Wo": flat.param(p + "attn.out_proj.weight"),
                "gWo": flat.grad(p + "attn.out_proj.weight"),
                "ln2": flat.param(p + "mlp_norm.weight"),
                "g_ln2": flat.grad(p + "mlp_norm.weight"),
                "W1": flat.param(p + "mlp.net.0.weight"),
                "gW1": flat.grad(p + "mlp.net.0.weight"),
                "W2": flat.param(p + "mlp.net.2.weight"),
                "gW2": flat.grad(p + "mlp.net.2.weight"),
                "range": (lo, hi),
            }
            if spec.bias:
                qb = flat.by_name[p + "attn.q_proj.bias"].offset
                blk.update(
                    bqkv=flat.params[qb : qb + 3 * F],
                    gbqkv=flat.grads[qb : qb + 3 * F],
                    bo=flat.param(p + "attn.out_proj.bias"),
                    gbo=flat.grad(p + "attn.out_proj.bias"),
                    b1=flat.param(p + "mlp.net.0.bias"),
                    gb1=flat.grad(p + "mlp.net.0.bias"),
                    b2=flat.param(p + "mlp.net.2.bias"),
                    gb2=flat.grad(p + "mlp.net.2.bias"),
                )
            else:
                blk.update(bqkv=None, gbqkv=None, bo=None, gbo=None, b1=None, gb1=None, b2=None, gb2=None)
            self.blocks.append(blk)
        self.E = flat.param("token_embedding.weight")
        self.gE = flat.grad("token_embedding.weight")
        self.P = flat.param("position_embedding.weight")
        self.gP = flat.grad("position_embedding.weight")
        self.lnf = flat.param("norm.weight")
        self.g_lnf = flat.grad("norm.weight")
        self.Wh = self.E if spec.tied else flat.param("head.weight")
        self.gWh = self.gE if spec.tied else flat.grad("head.weight")
        self.tail_range = (flat.by_name["norm.weight"].offset, flat.numel)
        self.embed_range = (0, self.blocks[0]["range"][0] if self.blocks else flat.by_name["norm.weight"].offset)

    # Unit hooks: a unit is "embed", a block index, or "tail".  Sharded-parameter
    # engines (ZeRO-3) gather a unit's weights before it runs and reduce its
    # gradients after its backward; the flat-buffer engine needs neither.
    def unit_forward(self, unit) -> None:
        pass

    def unit_backward_begin(self, unit) -> None:
        pass

    def unit_backward_end(self, unit) -> None:
        pass

    # ------------------------------------------------------------ forward
    def forward(self, ids: torch.Tensor, targets: torch.Tensor | None, *, fuse_loss_grad: bool,
                keep_logits: bool = False):
        """ids/targets int64 [B, T] on the device.  Returns (loss or None, logits or None)."""
        s = self.spec
        B, T = ids.shape
        if T > s.max_seq_len:
            raise ValueError(f"sequence length {T} exceeds max_seq_len {s.max_seq_len}")
        M = B * T
        H, D = s.heads, s.head_dim
        ids = ids.reshape(-1)
        self.unit_forward("embed")
        # context parallelism: this rank's tokens sit at `positions` of the sequence
        P = self.P if self.positions is None else self.P.index_select(0, self.positions)
        x = K.embedding(ids, self.E, P, T)
        saved_blocks = []
        for bi, blk in enumerate(self.blocks):
            nvtx.push(f"fwd/block{bi}")
            self.unit_forward(bi)
            h1, r1 = K.rmsnorm(x, blk["ln1"], s.eps)
            qkv = K.linear_fwd(h1, blk["Wqkv"], blk["bqkv"])
            if self.context_attention is not None:
                o, lse = self.context_attention.forward(qkv, B, T, H, D)
            else:
                o, lse = K.flash_attn_qkv(qkv, B, T, H, D, self.causal)
            x1 = K.linear_fwd_resid(o, blk["Wo"], blk["bo"], x)
            h2, r2 = K.rmsnorm(x1, blk["ln2"], s.eps)
            u, g = K.linear_fwd_gelu(h2, blk["W1"], blk["b1"])
            x2 = K.linear_fwd_resid(g, blk["W2"], blk["b2"], x1)
            saved_blocks.append((x, h1, r1, qkv, o, lse, x1, h2, r2, u, g))
            x = x2
            nvtx.pop()
        self.unit_forward("tail")
        hf, rf = K.rmsnorm(x, self.lnf, s.eps)
        logits = K.linear_fwd(hf, self.Wh, None)
        loss = None
        dlogits_ready = False
        if targets is not None:
            tg = targets.reshape(-1)
            if fuse_loss_grad and not keep_logits:
                loss_rows = K.softmax_cross_entropy(logits, tg, logits, 1.0 / M)  # dlogits in place
                dlogits_ready = True
            else:
                loss_rows = K.softmax_cross_entropy(logits, tg, None, 1.0)
            loss = K.ew_scalar(K.OP_MUL, K.reduce_sum(loss_rows).reshape(1), 1.0 / M).reshape(())
        self._saved = {
            "ids": ids, "targets": None if targets is None else targets.reshape(-1), "B": B, "T": T,
            "blocks": saved_blocks, "xL": x, "hf": hf, "rf": rf, "logits": logits,
            "dlogits_ready": dlogits_ready,
        }
        return loss, (None if dlogits_ready else logits)

    # ----------------------------------------------------------- backward
    def backward(self, dlogits: torch.Tensor | None = None, loss_grad: torch.Tensor | None = None) -> None:
        """Accumulate every parameter gradient into the flat fp32 buffer.

        Exactly one of: the forward fused the loss gradient (nothing to pass),
        `dlogits` (gradient w.r.t. returned logits), or `loss_grad` (device
        scalar dL/dloss; the logits gradient is recomputed from the kept logits).
        """
        sv = self._saved
        if sv is None:
            raise RuntimeError("backward() called without a saved forward")
        s = self.spec
        B, T = sv["B"], sv["T"]
        M = B * T
        H, D = s.heads, s.head_dim
        hook = self.grad_ready
        if sv["dlogits_ready"]:
            dl = sv["logits"]
        elif dlogits is not None:
            dl = dlogits.reshape(M, -1)
            if dl.dtype != torch.bfloat16 or not dl.is_contiguous():
                dl = dl.to(torch.bfloat16).contiguous()
        else:
            if sv["targets"] is None:
                raise RuntimeError("no loss gradient available")
            dl = sv["logits"]
            # (p - onehot) / M * dL/dloss, computed in place over the kept logits
            K.softmax_cross_entropy(dl, sv["targets"], dl, 1.0 / M, loss_grad)
        # Side stream: bias-gradient column sums (HBM-bound reductions) and,
        # with _WGRAD_SIDE, the weight-gradient GEMMs, launched as soon as
        # their inputs exist.  Nothing on the compute stream's critical path
        # (dgrad -> attention -> dgrad) reads their outputs, so they fill the
        # SMs the critical-path kernels leave idle (fill, tail, latency-bound
        # phases); the compute stream joins the side stream at the end of each
        # unit, before the unit's gradients are handed to the reduction hooks.
        flat = getattr(self, "flat", None)
        side = _side_stream(flat.device if flat is not None else None)
        pending: list = []

        def on_side(fn, *keep):
            ready = torch.cuda.Event()
            ready.record()
            side.wait_event(ready)
            with torch.cuda.stream(side):
                fn()
            pending.extend(keep)  # inputs kept alive until the join

        def wgrad(dy, x, dw):
            if _WGRAD_SIDE:
                on_side(lambda: K.linear_wgrad_accum(dy, x, dw), dy, x)
            else:
                K.linear_wgrad_accum(dy, x, dw)

        def colsum_async(x, out):
            if out is not None:
                on_side(lambda: K.colsum_accum(x, out), x)

        def join():
            if pending:
                torch.cuda.current_stream().wait_stream(side)
                pending.clear()

        # head + final norm
        self.unit_backward_begin("tail")
        dhf = K.linear_dgrad(dl, self.Wh)
        wgrad(dl, sv["hf"], self.gWh)
        dx = K.rmsnorm_backward(dhf, sv["xL"], self.lnf, sv["rf"], None, self.g_lnf)
        join()
        self.unit_backward_end("tail")
        if hook is not None and not s.tied:
            hook(*self.tail_range)
        elif hook is not None:
            hook(self.flat.by_name["norm.weight"].offset, self.flat.numel)
        del dl, dhf
        for bi in range(len(self.blocks) - 1, -1, -1):
            blk, saved = self.blocks[bi], sv["blocks"][bi]
            nvtx.push(f"bwd/block{bi}")
            self.unit_backward_begin(bi)
            x, h1, r1, qkv, o, lse, x1, h2, r2, u, g = saved
            # MLP
            colsum_async(dx, blk["gb2"])
            du = K.linear_dgrad(dx, blk["W2"], gelu_in=u)
            wgrad(dx, g, blk["gW2"])
            colsum_async(du, blk["gb1"])
            dh2 = K.linear_dgrad(du, blk["W1"])
            wgrad(du, h2, blk["gW1"])
            del du
            dx1 = K.rmsnorm_backward(dh2, x1, blk["ln2"], r2, dx, blk["g_ln2"])
            del dh2
            # attention
            colsum_async(dx1, blk["gbo"])
            do = K.linear_dgrad(dx1, blk["Wo"])
            wgrad(dx1, o, blk["gWo"])
            if self.context_attention is not None:
                dqkv = self.context_attention.backward(qkv, o, lse, do, B, T, H, D)
            else:
                dqkv = K.flash_attn_qkv_backward(qkv, o, lse, do, B, T, H, D, self.causal)
            del do
            colsum_async(dqkv, blk["gbqkv"])
            dh1 = K.linear_dgrad(dqkv, blk["Wqkv"])
            wgrad(dqkv, h1, blk["gWqkv"])
            del dqkv
            dx = K.rmsnorm_backward(dh1, x, blk["ln1"], r1, dx1, blk["g_ln1"])
            del dh1, dx1
            join()
            self.unit_backward_end(bi)
            if hook is not None:
                hook(*blk["range"])
            nvtx.pop()
        self.unit_backward_begin("embed")
        if self.positions is None:
            K.embedding_backward(sv["ids"], dx, self.gE, self.gP, T)
        else:
            gP = torch.zeros((T, self.gP.shape[1]), dtype=self.gP.dtype, device=self.gP.device)
            K.embedding_backward(sv["ids"], dx, self.gE, gP, T)
            self.gP.index_add_(0, self.positions, gP)
        self.unit_backward_end("embed")
        if hook is not None:
            hook(*self.embed_range)
        self._saved = None
