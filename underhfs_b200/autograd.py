"""Autograd utilities: grad mode, activation checkpointing, forward-mode JVP.

Reference: autograd.py:10-290.  Differences that matter for training on B200:

* ``no_grad()`` really disables graph recording (the reference's flag is
  never consulted by its Tensor);
* ``checkpoint()`` really recomputes: the function runs without saving
  activations and is re-run during backward (torch.utils.checkpoint), while
  keeping the reference's ``_underhfs_checkpoint`` tag on the outputs;
* ``jvp()`` keeps the reference's dual-number API over this package's Tensor.
"""

from __future__ import annotations

from contextlib import contextmanager
from dataclasses import dataclass
from typing import Any, Callable, Iterator

import torch
import torch.utils.checkpoint as _tckpt

from underhfs_b200.tensor import Tensor, tensor


@dataclass
class GradMode:
    enabled: bool = True


_grad_mode = GradMode()


def is_grad_enabled() -> bool:
    return _grad_mode.enabled and torch.is_grad_enabled()


@contextmanager
def no_grad() -> Iterator[None]:
    previous = _grad_mode.enabled
    _grad_mode.enabled = False
    try:
        with torch.no_grad():
            yield
    finally:
        _grad_mode.enabled = previous


def backward(value: Tensor, grad: Tensor | None = None) -> None:
    value.backward(grad)


def _to_torch(value: Any) -> Any:
    if isinstance(value, Tensor):
        return value._data
    if isinstance(value, (tuple, list)):
        return type(value)(_to_torch(v) for v in value)
    return value


def _from_torch(value: Any, like: Tensor | None) -> Any:
    if isinstance(value, torch.Tensor):
        return Tensor._wrap(value, like=like)
    if isinstance(value, (tuple, list)):
        return type(value)(_from_torch(v, like) for v in value)
    return value


def checkpoint(function: Callable[..., Any], *args: Any, preserve_rng_state: bool = True, **kwargs: Any) -> Any:
    """Activation checkpointing with real recomputation in backward."""
    like = next((a for a in args if isinstance(a, Tensor)), None)
    needs_grad = is_grad_enabled() and any(isinstance(a, Tensor) and a.requires_grad for a in args)
    if not needs_grad:
        result = function(*args, **kwargs)
    else:
        def run(*targs):
            wrapped = [Tensor._wrap(t, like=a) if isinstance(a, Tensor) else a for t, a in zip(targs, args)]
            return _to_torch(function(*wrapped, **kwargs))

        out = _tckpt.checkpoint(run, *[_to_torch(a) for a in args], use_reentrant=False,
                                preserve_rng_state=preserve_rng_state)
        result = _from_torch(out, like)
    _mark_checkpointed(result, function=getattr(function, "__name__", "anonymous"),
                       preserve_rng_state=preserve_rng_state)
    return result


def checkpoint_sequential(
    functions: tuple[Callable[[Any], Any], ...] | list[Callable[[Any], Any]],
    segments: int,
    input: Any,
    *,
    preserve_rng_state: bool = True,
) -> Any:
    if segments <= 0:
        raise ValueError("segments must be positive")
    if not functions:
        return input
    size = max(1, -(-len(functions) // segments))
    value = input
    for start in range(0, len(functions), size):
        chunk = list(functions[start : start + size])

        def run_chunk(current: Any, chunk=chunk) -> Any:
            for fn in chunk:
                current = fn(current)
            return current

        value = checkpoint(run_chunk, value, preserve_rng_state=preserve_rng_state)
    return value


def _mark_checkpointed(value: Any, *, function: str, preserve_rng_state: bool) -> None:
    if isinstance(value, Tensor):
        value._underhfs_checkpoint = {
            "function": function,
            "preserve_rng_state": preserve_rng_state,
            "mode": "eager-recompute-contract",
            "recompute": True,
        }
    elif isinstance(value, (tuple, list)):
        for item in value:
            _mark_checkpointed(item, function=function, preserve_rng_state=preserve_rng_state)
    elif isinstance(value, dict):
        for item in value.values():
            _mark_checkpointed(item, function=function, preserve_rng_state=preserve_rng_state)


# ------------------------------------------------------------ forward-mode AD
def jvp(function: Callable[..., Any], primals: tuple[Tensor, ...], tangents: tuple[Tensor, ...]) -> tuple[Any, Any]:
    """Forward-mode derivative: returns (function(*primals), J @ tangents)."""
    if len(primals) != len(tangents):
        raise ValueError("primals and tangents must have the same length")
    duals = tuple(_Dual(p, t) for p, t in zip(primals, tangents))
    return _split(function(*duals))


class _Dual:
    """Dual number (primal, tangent) over Tensor; each op applies its derivative rule."""

    def __init__(self, primal: Tensor, tangent: Tensor) -> None:
        if primal.shape != tangent.shape:
            raise ValueError(f"JVP tangent shape {tangent.shape} does not match primal shape {primal.shape}")
        self.primal = primal
        self.tangent = tangent

    shape = property(lambda self: self.primal.shape)
    ndim = property(lambda self: self.primal.ndim)
    dtype = property(lambda self: self.primal.dtype)
    device = property(lambda self: self.primal.device)
    layout = property(lambda self: self.primal.layout)

    def _lift(self, other: Any) -> "_Dual":
        if isinstance(other, _Dual):
            return other
        p = other if isinstance(other, Tensor) else tensor(other, dtype=self.primal.dtype, device=self.primal.device)
        return _Dual(p, Tensor._wrap(torch.zeros_like(p._data), like=p)) if p.shape else _Dual(p, p * 0.0)

    def __add__(self, o):
        o = self._lift(o)
        return _Dual(self.primal + o.primal, self.tangent + o.tangent)

    __radd__ = __add__

    def __sub__(self, o):
        o = self._lift(o)
        return _Dual(self.primal - o.primal, self.tangent - o.tangent)

    def __rsub__(self, o):
        return self._lift(o) - self

    def __mul__(self, o):
        o = self._lift(o)
        return _Dual(self.primal * o.primal, self.tangent * o.primal + self.primal * o.tangent)

    __rmul__ = __mul__

    def __truediv__(self, o):
        o = self._lift(o)
        return _Dual(self.primal / o.primal,
                     (self.tangent * o.primal - self.primal * o.tangent) / (o.primal * o.primal))

    def __rtruediv__(self, o):
        return self._lift(o) / self

    def __neg__(self):
        return _Dual(-self.primal, -self.tangent)

    def __pow__(self, k: float):
        return _Dual(self.primal ** k, self.tangent * (self.primal ** (k - 1) * k))

    def __matmul__(self, o):
        o = self._lift(o)
        return _Dual(self.primal @ o.primal, self.tangent @ o.primal + self.primal @ o.tangent)

    def __getitem__(self, key):
        return _Dual(self.primal[key], self.tangent[key])

    def sum(self):
        return _Dual(self.primal.sum(), self.tangent.sum())

    def mean(self):
        return _Dual(self.primal.mean(), self.tangent.mean())

    def view(self, *shape):
        return _Dual(self.primal.view(*shape), self.tangent.view(*shape))

    def reshape(self, *shape):
        return _Dual(self.primal.reshape(*shape), self.tangent.reshape(*shape))

    def flatten(self):
        return _Dual(self.primal.flatten(), self.tangent.flatten())

    def transpose(self):
        return _Dual(self.primal.transpose(), self.tangent.transpose())

    @property
    def T(self):
        return self.transpose()

    def relu(self):
        mask = Tensor._wrap((self.primal._data > 0).to(self.primal._data.dtype), like=self.primal)
        return _Dual(self.primal.relu(), self.tangent * mask)

    def tanh(self):
        y = self.primal.tanh()
        return _Dual(y, self.tangent * (1.0 - y * y))

    def exp(self):
        y = self.primal.exp()
        return _Dual(y, self.tangent * y)

    def log(self):
        return _Dual(self.primal.log(), self.tangent / self.primal)

    def sqrt(self):
        y = self.primal.sqrt()
        return _Dual(y, self.tangent / (y * 2.0))

    def softmax(self):
        if self.primal.ndim not in (1, 2):
            raise ValueError("softmax JVP supports 1D or 2D tensors")
        y = self.primal.softmax()
        yt = y._data.detach()
        tt = self.tangent._data.detach()
        dot = (yt * tt).sum(-1, keepdim=True)
        return _Dual(y, Tensor._wrap(yt * (tt - dot), like=self.primal))


def _split(value: Any) -> tuple[Any, Any]:
    if isinstance(value, _Dual):
        return value.primal, value.tangent
    if isinstance(value, (tuple, list)):
        pairs = [_split(v) for v in value]
        return type(value)(p for p, _ in pairs), type(value)(t for _, t in pairs)
    if isinstance(value, dict):
        pairs = {k: _split(v) for k, v in value.items()}
        return {k: p for k, (p, _) in pairs.items()}, {k: t for k, (_, t) in pairs.items()}
    return value, None
