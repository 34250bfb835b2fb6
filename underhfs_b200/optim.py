"""Optimizers (reference optim.py:10-225).

Semantics kept from the reference: validation messages, ``step_count``,
``state_dict`` as nested lists, and the L2-coupled weight decay
(``g += wd * p`` before the moments, optim.py:147).  ``decoupled=True``
selects the AdamW-paper form instead.

Execution on B200:

* parameters that live in one flat buffer (a TransformerLM moved to CUDA in
  bf16) are updated by ONE launch of the fused AdamW kernel over the fp32
  master weights, writing the bf16 compute copy in the same pass;
* other CUDA parameters use the same kernel per tensor (fp32 moments);
* CPU parameters use PyTorch float64 math with identical formulas.

``ZeroAwareAdamW`` is a real ZeRO optimizer: with ``world_size > 1`` the
moments and master weights are sharded and the update runs as a fused
reduce-scatter + AdamW + all-gather kernel over NVLink (parallel/zero.py).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Iterable

import torch

from underhfs_b200.tensor import DType, Tensor


class Optimizer:
    def __init__(self, params: Iterable[Tensor]) -> None:
        self.params = list(params)

    def zero_grad(self) -> None:
        flat = _shared_flat(self.params)
        if flat is not None:
            flat.zero_grad()
            return
        for p in self.params:
            p.zero_grad()

    def step(self) -> None:
        raise NotImplementedError


@dataclass(frozen=True)
class OptimizerKernelStatus:
    name: str
    backend: str
    available: bool
    reason: str = ""

    def to_dict(self) -> dict[str, str | bool]:
        return {"name": self.name, "backend": self.backend, "available": self.available, "reason": self.reason}


def _shared_flat(params: list[Tensor]):
    """The FlatBuffers object if every parameter is a view of the same one and
    together they cover all its parameters."""
    if not params:
        return None
    flat = getattr(params[0], "_flat", None)
    if flat is None:
        return None
    if any(getattr(p, "_flat", None) is not flat for p in params):
        return None
    if len({id(p) for p in params}) != len(flat.layout.slots):
        return None
    return flat


def fused_adamw_kernel_status(params: Iterable[Tensor]) -> OptimizerKernelStatus:
    ps = list(params)
    if not ps:
        return OptimizerKernelStatus("fused_adamw", "python", True, "no parameters")
    if all(p.device.kind == "cuda" for p in ps):
        try:
            from underhfs_b200.native import status

            if status().cuda_enabled:
                if _shared_flat(ps) is not None:
                    return OptimizerKernelStatus("fused_adamw", "cuda-native", True,
                                                 "one sm_100a launch over the flat fp32 master buffer")
                return OptimizerKernelStatus("fused_adamw", "cuda-native", True, "sm_100a fused AdamW per tensor")
        except Exception as exc:  # noqa: BLE001
            return OptimizerKernelStatus("fused_adamw", "python", True, f"native core unavailable: {exc}")
        return OptimizerKernelStatus("fused_adamw", "python", True, "CUDA parameters without the native core")
    return OptimizerKernelStatus("fused_adamw", "python", True, "CPU/Python fused update loop")


class SGD(Optimizer):
    def __init__(self, params: Iterable[Tensor], lr: float = 1e-3) -> None:
        super().__init__(params)
        if lr < 0:
            raise ValueError("lr must be non-negative")
        self.lr = lr

    def step(self) -> None:
        flat = _shared_flat(self.params)
        if flat is not None:
            with torch.no_grad():
                flat.master.add_(flat.grads, alpha=-self.lr)
                flat.params.copy_(flat.master)
            return
        for p in self.params:
            g = p.grad
            if g is None:
                continue
            p.add_(g * -self.lr)


class AdamW(Optimizer):
    def __init__(
        self,
        params: Iterable[Tensor],
        lr: float = 1e-3,
        betas: tuple[float, float] = (0.9, 0.999),
        eps: float = 1e-8,
        weight_decay: float = 0.01,
        *,
        decoupled: bool = False,
    ) -> None:
        super().__init__(params)
        if lr < 0:
            raise ValueError("lr must be non-negative")
        if eps < 0:
            raise ValueError("eps must be non-negative")
        if weight_decay < 0:
            raise ValueError("weight_decay must be non-negative")
        if not 0 <= betas[0] < 1 or not 0 <= betas[1] < 1:
            raise ValueError("AdamW betas must be in the range [0, 1)")
        self.lr = lr
        self.betas = tuple(betas)
        self.eps = eps
        self.weight_decay = weight_decay
        self.decoupled = decoupled
        self.step_count = 0
        self._flat = _shared_flat(self.params)
        if self._flat is not None:
            self._m_flat = torch.zeros_like(self._flat.master)
            self._v_flat = torch.zeros_like(self._flat.master)
            self._step_t = torch.zeros((), dtype=torch.int32, device=self._flat.device)
        else:
            self._m32 = [self._zeros_state(p) for p in self.params]
            self._v32 = [self._zeros_state(p) for p in self.params]
            self._master32 = [None for _ in self.params]

    @staticmethod
    def _zeros_state(p: Tensor) -> torch.Tensor:
        dt = torch.float32 if p.device.kind == "cuda" else torch.float64
        return torch.zeros(p.shape, dtype=dt, device=p._data.device)

    # state views (reference exposes m / v as lists of Tensors on the param's dtype/device)
    def _state_views(self, which: str) -> list[Tensor]:
        if self._flat is not None:
            buf = self._m_flat if which == "m" else self._v_flat
            out = []
            for p in self.params:
                s = self._flat.by_name[self._name_of(p)]
                out.append(Tensor._wrap(buf[s.offset : s.offset + s.numel].view(s.shape), dtype=p.dtype))
            return out
        src = self._m32 if which == "m" else self._v32
        return [
            Tensor._wrap(s.to(p._data.dtype), like=p, backend=p.backend) for s, p in zip(src, self.params)
        ]

    def _name_of(self, p: Tensor) -> str:
        if not hasattr(self, "_names"):
            view_ptrs = {}
            for slot in self._flat.layout.slots:
                view_ptrs[self._flat.params.data_ptr() + 2 * slot.offset] = slot.name
            self._names = {id(q): view_ptrs[q._data.data_ptr()] for q in self.params}
        return self._names[id(p)]

    @property
    def m(self) -> list[Tensor]:
        return self._state_views("m")

    @property
    def v(self) -> list[Tensor]:
        return self._state_views("v")

    def state_dict(self) -> dict:
        return {
            "step_count": self.step_count,
            "lr": self.lr,
            "betas": list(self.betas),
            "eps": self.eps,
            "weight_decay": self.weight_decay,
            "m": [t.tolist() for t in self.m],
            "v": [t.tolist() for t in self.v],
        }

    def load_state_dict(self, state: dict) -> None:
        if len(state["m"]) != len(self.params) or len(state["v"]) != len(self.params):
            raise ValueError("optimizer state does not match parameter count")
        self.step_count = int(state["step_count"])
        self.lr = float(state["lr"])
        self.betas = (float(state["betas"][0]), float(state["betas"][1]))
        self.eps = float(state["eps"])
        self.weight_decay = float(state["weight_decay"])
        if self._flat is not None:
            for which, buf in (("m", self._m_flat), ("v", self._v_flat)):
                for value, p in zip(state[which], self.params):
                    s = self._flat.by_name[self._name_of(p)]
                    buf[s.offset : s.offset + s.numel].copy_(torch.tensor(value).reshape(-1))
            self._step_t.fill_(self.step_count)
            return
        for i, p in enumerate(self.params):
            self._m32[i].copy_(torch.tensor(state["m"][i], dtype=self._m32[i].dtype).reshape(p.shape))
            self._v32[i].copy_(torch.tensor(state["v"][i], dtype=self._v32[i].dtype).reshape(p.shape))

    def step(self) -> None:
        self.step_count += 1
        b1, b2 = self.betas
        if self._flat is not None:
            self._flat_step(b1, b2)
            return
        cpu: list = []
        for i, p in enumerate(self.params):
            g = p.grad
            if g is None:
                continue
            if p.device.kind == "cuda":
                self._cuda_step(i, p, g, b1, b2)
            else:
                cpu.append((i, p, g))
        if cpu:
            self._cpu_steps(cpu, b1, b2)

    def _flat_step(self, b1: float, b2: float, lo: int = 0, hi: int | None = None, increment: bool = True) -> None:
        from underhfs_b200.ops import kernels as K

        f = self._flat
        hi = f.master.numel() if hi is None else min(hi, f.master.numel())
        if increment:
            K.increment_(self._step_t)
        if hi <= lo:
            return
        K.adamw_(f.master[lo:hi], f.grads[lo:hi], self._m_flat[lo:hi], self._v_flat[lo:hi], f.params[lo:hi],
                 lr=self.lr, beta1=b1, beta2=b2, eps=self.eps, weight_decay=self.weight_decay,
                 decoupled=self.decoupled, step_t=self._step_t)

    def step_split(self, boundary: int, wait: Callable[[], None]) -> None:
        """One optimizer step in two launches for a flat-buffer model whose
        gradients below `boundary` are still being reduced: the parameters at
        or above it are updated first (overlapping that reduction), then
        `wait()` orders the stream after it and the rest is updated."""
        if self._flat is None:
            wait()
            self.step()
            return
        self.step_count += 1
        b1, b2 = self.betas
        self._flat_step(b1, b2, boundary, None, increment=True)
        wait()
        self._flat_step(b1, b2, 0, boundary, increment=False)

    def _cuda_step(self, i: int, p: Tensor, g: Tensor, b1: float, b2: float) -> None:
        from underhfs_b200.ops import kernels as K

        pd = p._data
        gd = g._data.detach()
        in_place = pd.dtype == torch.float32 and pd.is_contiguous()
        if in_place:
            master = pd.detach()
        else:
            if self._master32[i] is None:
                self._master32[i] = pd.detach().float().contiguous()
            master = self._master32[i]
        gd32 = gd.float().contiguous() if gd.dtype != torch.float32 else gd.contiguous()
        with torch.no_grad():
            K.adamw_(master, gd32, self._m32[i], self._v32[i], None, lr=self.lr, beta1=b1, beta2=b2, eps=self.eps,
                     weight_decay=self.weight_decay, decoupled=self.decoupled, step=self.step_count)
            # the kernel wrote the weights; the copy (or self-copy) bumps the
            # version counter exactly like the reference's in-place update
            pd.copy_(master if in_place else master.to(pd.dtype))
        p.backend = "native_cuda"

    def _cpu_steps(self, items: list, b1: float, b2: float) -> None:
        """Every CPU parameter in one pass of multi-tensor (foreach) ops; the
        per-element arithmetic and its order are those of the single-tensor
        update (weight decay multiplied, then added)."""
        with torch.no_grad():
            pds = [p._data for _, p, _ in items]
            gds = [g._data.to(p._data.dtype) for _, p, g in items]
            if self.decoupled:
                torch._foreach_mul_(pds, 1.0 - self.lr * self.weight_decay)
            else:
                gds = torch._foreach_add(gds, torch._foreach_mul(pds, self.weight_decay))
            ms = [self._m32[i] for i, _, _ in items]
            vs = [self._v32[i] for i, _, _ in items]
            torch._foreach_mul_(ms, b1)
            torch._foreach_add_(ms, gds, alpha=1 - b1)
            torch._foreach_mul_(vs, b2)
            torch._foreach_addcmul_(vs, gds, gds, value=1 - b2)
            mh = torch._foreach_div(ms, 1 - b1 ** self.step_count)
            den = torch._foreach_sqrt(torch._foreach_div(vs, 1 - b2 ** self.step_count))
            torch._foreach_add_(den, self.eps)
            torch._foreach_add_(pds, torch._foreach_div(mh, den), alpha=-self.lr)


class FusedAdamW(AdamW):
    """AdamW whose CUDA update is one fused kernel (see module docstring)."""

    def step(self) -> None:
        self.last_kernel_status = fused_adamw_kernel_status(self.params)
        super().step()

    def step_split(self, boundary: int, wait) -> None:
        self.last_kernel_status = fused_adamw_kernel_status(self.params)
        super().step_split(boundary, wait)


@dataclass
class ZeroShard:
    rank: int = 0
    world_size: int = 1


class ZeroAwareAdamW(AdamW):
    """AdamW whose state is partitioned across data-parallel ranks
    (the reference's surface: ``ZeroAwareAdamW(params, shard=ZeroShard(...))``,
    optim.py:216-225 of the reference, where it is a single-process stub).

    ``stage`` 1/2: master weights and moments are held for the local 1/W
    shard only; ``step()`` runs the fused reduce-scatter + AdamW + all-gather
    kernel.

    ``stage`` 3: the parameters of a TransformerLM on the CUDA engine are
    sharded too.  Construction builds the ZeRO-3 runtime
    (parallel.zero3.Zero3LM) from the model's current weights and attaches it
    to the model: every rank keeps 1/W of the bf16 weights, fp32 master and
    moments; forward gathers each unit's weights just before use (the gather
    fused into the first GEMM that reads them) and backward reduces each
    unit's gradients with a kernel that applies the AdamW update to the owned
    rows as it goes.  ``step()`` therefore only closes the step; call it after
    every backward (no gradient accumulation at stage 3).  ``offload`` places
    the Adam moments: ``"auto"`` (default) asks the memory planner, which
    keeps them in device memory when they fit next to the step's other
    buffers and ``activation_bytes``, else pinned host RAM; ``"host"`` /
    ``"device"`` force it.  ``world_size == 1`` is allowed at every stage.
    """

    def __init__(self, params: Iterable[Tensor], shard: ZeroShard | None = None, *, stage: int = 2,
                 group=None, offload: str = "auto", planner=None, activation_bytes: int = 0,
                 **kwargs) -> None:
        params = list(params)
        self.shard = shard or ZeroShard()
        self.stage = stage
        if stage not in (1, 2, 3):
            raise ValueError("ZeRO stage must be 1, 2 or 3")
        self._zero = None
        self._zero3 = None
        flat = _shared_flat(params)
        if stage == 3:
            self._set_hparams(params, kwargs)
            self._init_stage3(flat, group, offload, planner, activation_bytes)
        elif self.shard.world_size > 1 and flat is not None:
            from underhfs_b200.parallel.zero import ZeroFlatOptimizer

            self._set_hparams(params, kwargs)
            self._flat = flat
            self._zero = ZeroFlatOptimizer(flat, self.shard, group=group, stage=stage)
        else:
            super().__init__(params, **kwargs)

    def _set_hparams(self, params: list, kwargs: dict) -> None:
        Optimizer.__init__(self, params)
        betas = kwargs.get("betas", (0.9, 0.999))
        if not 0 <= betas[0] < 1 or not 0 <= betas[1] < 1:
            raise ValueError("AdamW betas must be in the range [0, 1)")
        self.lr = kwargs.get("lr", 1e-3)
        self.betas = tuple(betas)
        self.eps = kwargs.get("eps", 1e-8)
        self.weight_decay = kwargs.get("weight_decay", 0.01)
        self.decoupled = kwargs.get("decoupled", False)
        self.step_count = 0
        self._flat = None

    def _init_stage3(self, flat, group, offload: str, planner, activation_bytes: int) -> None:
        model = getattr(flat, "owner", None) if flat is not None else None
        if model is None or not hasattr(model, "attach_zero3"):
            raise ValueError("ZeRO stage 3 shards a TransformerLM on the CUDA engine: pass the parameters of a "
                             "TransformerLM moved with .to('cuda', dtype='bf16')")
        if offload not in ("auto", "host", "device"):
            raise ValueError("offload must be 'auto', 'host' or 'device'")
        from underhfs_b200.parallel.zero3 import Zero3LM

        state = {slot.name: (flat.master_view(slot.name) if flat.master is not None else flat.param(slot.name))
                 .detach().float() for slot in flat.layout.slots}
        self._zero3 = Zero3LM(
            model.spec, rank=self.shard.rank, world=self.shard.world_size, device=flat.device, group=group,
            state=state, lr=self.lr, betas=self.betas, eps=self.eps, weight_decay=self.weight_decay,
            decoupled=self.decoupled, offload_moments={"auto": "auto", "host": True, "device": False}[offload],
            planner=planner, activation_bytes=activation_bytes, hparams=self)
        del state
        model.attach_zero3(self._zero3)

    @property
    def zero3(self):
        return self._zero3

    def zero_grad(self) -> None:
        if self._zero3 is None:
            super().zero_grad()

    def step(self) -> None:
        if self._zero3 is not None:
            self.step_count += 1
            self._zero3.step_done()
            return
        if self._zero is None:
            super().step()
            return
        self.step_count += 1
        self._zero.step(lr=self.lr, betas=self.betas, eps=self.eps, weight_decay=self.weight_decay,
                        decoupled=self.decoupled)

    def step_split(self, boundary: int, wait) -> None:
        if self._zero is None and self._zero3 is None:
            super().step_split(boundary, wait)
            return
        wait()  # the sharded update reduces every gradient itself
        self.step()

    def state_dict(self) -> dict:
        if self._zero is None and self._zero3 is None:
            return super().state_dict()
        out = {"step_count": self.step_count, "lr": self.lr, "betas": list(self.betas), "eps": self.eps,
               "weight_decay": self.weight_decay}
        if self._zero is not None:
            out["zero"] = self._zero.shard_state()
        else:
            out["zero3"] = {"stage": 3, "rank": self.shard.rank, "world_size": self.shard.world_size,
                            "moments_offloaded": bool(self._zero3.offload)}
        return out


_ = DType  # re-exported for callers that type-annotate with the optimizer module
