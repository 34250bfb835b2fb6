"""Stateless ops: losses and activations (reference functional.py:8-89).

On CUDA tensors each op runs this package's kernels (fused softmax
cross-entropy, tanh-GELU, row softmax); on CPU they run PyTorch in float64,
matching the reference's Python-float semantics.
"""

from __future__ import annotations

import math

import torch

from underhfs_b200.tensor import Tensor


def _cuda_native(t: Tensor) -> bool:
    return t.device.kind == "cuda"


def mse_loss(input: Tensor, target: Tensor, reduction: str = "mean") -> Tensor:
    diff = input - target
    loss = diff * diff
    if reduction == "mean":
        return loss.mean()
    if reduction == "sum":
        return loss.sum()
    if reduction == "none":
        return loss
    raise ValueError(f"unsupported reduction: {reduction}")


def cross_entropy(logits: Tensor, target: Tensor, reduction: str = "mean") -> Tensor:
    """Mean/sum/none negative log-likelihood of integer targets.

    logits [batch, classes] (or [..., classes], flattened), target [batch].
    Matches the reference's clamp -log(max(p, 1e-30)).
    """
    if reduction not in ("mean", "sum", "none"):
        raise ValueError(f"unsupported reduction: {reduction}")
    if logits.ndim < 2:
        raise ValueError("cross_entropy expects logits with shape [batch, classes]")
    x = logits._data.reshape(-1, logits.shape[-1])
    tg = target._data.reshape(-1)
    if tg.shape[0] != x.shape[0]:
        raise ValueError(f"target batch {tg.shape[0]} does not match logits batch {x.shape[0]}")
    classes = x.shape[1]
    tgi = tg.to(torch.int64)
    bad = (tgi < 0) | (tgi >= classes)
    if bool(bad.any()):
        label = int(tgi[bad][0].item())
        raise ValueError(f"target class {label} is outside [0, {classes})")
    if _cuda_native(logits):
        from underhfs_b200.ops import functions as OF

        out = OF.cross_entropy(x, tgi, reduction)
        return Tensor._wrap(out, like=logits, backend="native_cuda")
    logp = torch.log_softmax(x, dim=-1)
    nll = -logp.gather(1, tgi.unsqueeze(1)).squeeze(1)
    nll = torch.clamp(nll, max=-math.log(1e-30))
    if reduction == "mean":
        nll = nll.sum() / max(1, x.shape[0])
    elif reduction == "sum":
        nll = nll.sum()
    return Tensor._wrap(nll, like=logits)


def relu(input: Tensor) -> Tensor:
    return input.relu()


def gelu(input: Tensor) -> Tensor:
    """tanh-approximation GELU: 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))."""
    if _cuda_native(input):
        from underhfs_b200.ops import functions as OF

        return Tensor._wrap(OF.gelu(input._data), like=input, backend="native_cuda")
    x = input._data
    c = math.sqrt(2.0 / math.pi)
    return Tensor._wrap(0.5 * x * (1.0 + torch.tanh(c * (x + 0.044715 * x * x * x))), like=input)


def softmax(input: Tensor) -> Tensor:
    return input.softmax()
