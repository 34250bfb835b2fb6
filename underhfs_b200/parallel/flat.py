"""Flat parameter / master-weight / gradient storage.

Every trainable parameter of a model becomes a view into three contiguous
buffers allocated once:

* ``params``  -- compute copy (bf16 on B200) read by the GEMMs;
* ``master``  -- fp32 master weights updated by the fused optimizer;
* ``grads``   -- fp32 gradients; weight-gradient GEMMs accumulate into them
  directly (split-K atomics), so autograd never allocates per-parameter grads.

One launch of the fused AdamW kernel then updates the whole model, DDP
buckets are contiguous slices of ``grads`` and ZeRO shards are equal slices of
all three.  Views start on 64-element boundaries so every one is 128-byte
aligned for TMA and 16-byte vector access.

The reference keeps each parameter as its own Python list
(tensor.py:149-192) and updates it with one kernel call per parameter
(optim.py:158-192); there is no equivalent of this layout there.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable, Sequence

import torch

ALIGN = 64


def _round_up(n: int, a: int) -> int:
    return (n + a - 1) // a * a


@dataclass
class FlatSlot:
    name: str
    shape: tuple[int, ...]
    offset: int
    numel: int


@dataclass
class FlatLayout:
    slots: list[FlatSlot] = field(default_factory=list)
    total: int = 0

    def add(self, name: str, shape: Sequence[int], *, align: int = ALIGN) -> FlatSlot:
        numel = 1
        for d in shape:
            numel *= int(d)
        off = _round_up(self.total, align)
        slot = FlatSlot(name, tuple(int(d) for d in shape), off, numel)
        self.slots.append(slot)
        self.total = off + numel
        return slot

    def add_group(self, names_shapes: Sequence[tuple[str, Sequence[int]]]) -> list[FlatSlot]:
        """Add slots back to back with no padding between them (e.g. q/k/v weights
        that one fused GEMM reads as a single [3F, F] matrix)."""
        first = True
        out = []
        for name, shape in names_shapes:
            if first:
                out.append(self.add(name, shape))
                first = False
            else:
                numel = 1
                for d in shape:
                    numel *= int(d)
                slot = FlatSlot(name, tuple(int(d) for d in shape), self.total, numel)
                self.slots.append(slot)
                self.total += numel
                out.append(slot)
        return out

    def padded_total(self, multiple: int) -> int:
        return _round_up(max(self.total, 1), multiple)


class FlatBuffers:
    """The three flat buffers of one model and named views into them."""

    def __init__(
        self,
        layout: FlatLayout,
        device: torch.device,
        *,
        param_dtype: torch.dtype = torch.bfloat16,
        pad_multiple: int = ALIGN,
        grad_alloc: Callable[[int], torch.Tensor] | None = None,
        keep_master: bool = True,
    ) -> None:
        self.layout = layout
        self.device = torch.device(device)
        self.numel = layout.padded_total(pad_multiple)
        self.params = torch.zeros(self.numel, dtype=param_dtype, device=self.device)
        self.master = torch.zeros(self.numel, dtype=torch.float32, device=self.device) if keep_master else None
        if grad_alloc is not None:
            self.grads = grad_alloc(self.numel)
            self.grads.zero_()
        else:
            self.grads = torch.zeros(self.numel, dtype=torch.float32, device=self.device)
        self.by_name = {slot.name: slot for slot in layout.slots}

    def param(self, name: str) -> torch.Tensor:
        s = self.by_name[name]
        return self.params[s.offset : s.offset + s.numel].view(s.shape)

    def grad(self, name: str) -> torch.Tensor:
        s = self.by_name[name]
        return self.grads[s.offset : s.offset + s.numel].view(s.shape)

    def master_view(self, name: str) -> torch.Tensor:
        s = self.by_name[name]
        assert self.master is not None
        return self.master[s.offset : s.offset + s.numel].view(s.shape)

    def span(self, first: str, last: str) -> tuple[int, int]:
        a = self.by_name[first]
        b = self.by_name[last]
        return a.offset, b.offset + b.numel

    def load_from(self, name: str, value: torch.Tensor) -> None:
        v = value.detach().to(self.device, torch.float32).reshape(self.by_name[name].shape)
        if self.master is not None:
            self.master_view(name).copy_(v)
        self.param(name).copy_(v.to(self.params.dtype))

    def zero_grad(self) -> None:
        self.grads.zero_()
