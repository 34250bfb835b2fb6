"""Distributed policy, process group and data parallelism.

Reference: distributed.py:12-285.  Kept: ``ParallelMode``, ``DistributedPolicy``,
``NcclRuntimePlan`` / ``nccl_runtime_plan``, ``ProcessGroup`` (barrier,
all_reduce_sum, broadcast, reduce_scatter, all_gather, no_sync) with the
world-size-1 identity semantics, ``init_process_group`` / ``process_group``
validation and messages, and ``DistributedDataParallel`` with ``no_sync`` and
``synchronize_gradients``.

B200 implementation: one process per GPU launched by torchrun (or
``python -m underhfs_b200.parallel.launch``), torch.distributed over NCCL for
bootstrap, barrier and broadcast, and this package's fused NVLink kernels for
the gradient all-reduce (bucketed, overlapped with backward) and the ZeRO
reduce-scatter + AdamW + all-gather.  ``backend="gloo"`` runs the same API on
CPU processes (used by the multi-process tests).  The reference's launcher
module is named but missing (distributed.py:47-55); here it exists.
"""

from __future__ import annotations

import os
from contextlib import contextmanager
from dataclasses import dataclass
from datetime import timedelta
from enum import Enum
from typing import Any, Iterator

import torch
import torch.distributed as dist

from underhfs_b200.tensor import Tensor


class ParallelMode(str, Enum):
    DATA = "data"
    TENSOR = "tensor"
    PIPELINE = "pipeline"
    ZERO = "zero"


@dataclass
class DistributedPolicy:
    world_size: int = 1
    rank: int = 0
    modes: tuple[ParallelMode, ...] = (ParallelMode.DATA,)
    backend: str = "nccl"
    zero_stage: int = 0
    bucket_mb: float = 25.0
    comm_backend: str = "p2p"  # p2p (fused NVLink kernels) | nccl
    overlap: bool = True
    local_rank: int | None = None
    timeout_s: float = 300.0


def policy_from_env(**overrides: Any) -> DistributedPolicy:
    """Policy from torchrun's RANK / WORLD_SIZE / LOCAL_RANK (or UNDERHFS_RANK /
    UNDERHFS_WORLD_SIZE)."""
    env = os.environ
    rank = int(env.get("RANK", env.get("UNDERHFS_RANK", "0")))
    world = int(env.get("WORLD_SIZE", env.get("UNDERHFS_WORLD_SIZE", "1")))
    local = int(env.get("LOCAL_RANK", str(rank)))
    pol = DistributedPolicy(world_size=world, rank=rank, local_rank=local)
    for k, v in overrides.items():
        setattr(pol, k, v)
    return pol


@dataclass(frozen=True)
class NcclRuntimePlan:
    world_size: int
    backend: str
    modes: tuple[ParallelMode, ...]
    launch_command: tuple[str, ...]

    def to_dict(self) -> dict[str, Any]:
        return {"world_size": self.world_size, "backend": self.backend, "modes": [m.value for m in self.modes],
                "launch_command": list(self.launch_command)}


def nccl_runtime_plan(policy: DistributedPolicy) -> NcclRuntimePlan:
    if policy.backend != "nccl":
        raise ValueError("NCCL runtime plan requires backend='nccl'")
    if policy.world_size <= 1:
        cmd = ("python", "-m", "underhfs_b200.parallel.launch", "--nproc-per-node=1")
    else:
        cmd = ("python", "-m", "underhfs_b200.parallel.launch", f"--nproc-per-node={policy.world_size}",
               "--master-addr=127.0.0.1")
    return NcclRuntimePlan(policy.world_size, policy.backend, policy.modes, cmd)


def _nccl_available() -> bool:
    try:
        from underhfs_b200.native import status

        return status().nccl_enabled
    except Exception:  # noqa: BLE001
        return False


def init_process_group(policy: DistributedPolicy | None = None) -> DistributedPolicy:
    pol = policy or DistributedPolicy()
    if pol.world_size <= 0:
        raise ValueError("world_size must be positive")
    if pol.rank < 0 or pol.rank >= pol.world_size:
        raise ValueError("rank must be in the range [0, world_size)")
    if pol.backend not in ("nccl", "gloo"):
        raise ValueError("only backend='nccl' (GPUs) or 'gloo' (CPU processes) is supported")
    if pol.world_size > 1:
        if pol.backend == "nccl" and not _nccl_available():
            raise RuntimeError(
                "world_size > 1 requires underHFS native core built with UNDERHFS_WITH_NCCL=ON "
                "and a visible CUDA device per rank (use backend='gloo' for CPU processes)"
            )
        _ensure_torch_group(pol)
    return pol


def _ensure_torch_group(pol: DistributedPolicy) -> None:
    if dist.is_available() and dist.is_initialized():
        return
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29511")
    kwargs: dict[str, Any] = {}
    if pol.backend == "nccl":
        local = pol.local_rank if pol.local_rank is not None else pol.rank % max(1, torch.cuda.device_count())
        torch.cuda.set_device(local)
        kwargs["device_id"] = torch.device("cuda", local)
    dist.init_process_group(pol.backend, rank=pol.rank, world_size=pol.world_size,
                            timeout=timedelta(seconds=pol.timeout_s), **kwargs)


def _require_collective(policy: DistributedPolicy) -> None:
    if policy.world_size == 1:
        return
    if policy.backend == "nccl" and not _nccl_available():
        raise RuntimeError("multi-process collectives require UNDERHFS_WITH_NCCL=ON")
    if not dist.is_initialized():
        raise RuntimeError("process group is not initialized")


def _coll_device(policy: DistributedPolicy) -> torch.device:
    if policy.backend == "nccl":
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")


@dataclass
class ProcessGroup:
    policy: DistributedPolicy
    synchronized: bool = True

    def __post_init__(self) -> None:
        if self.policy.world_size > 1:
            _ensure_torch_group(self.policy)

    @property
    def rank(self) -> int:
        return self.policy.rank

    @property
    def world_size(self) -> int:
        return self.policy.world_size

    @property
    def backend(self) -> str:
        return self.policy.backend

    # values are Tensors, torch tensors, lists of numbers or scalars
    def _payload(self, value: Any) -> tuple[torch.Tensor, Any]:
        dev = _coll_device(self.policy)
        if isinstance(value, Tensor):
            t = value._data.detach()
            return t.to(dev, torch.float32 if t.device.type == "cpu" else t.dtype).clone(), (
                lambda out: Tensor._wrap(out.to(value._data.device, value._data.dtype), like=value))
        if isinstance(value, torch.Tensor):
            return value.detach().to(dev).clone(), (lambda out: out.to(value.device, value.dtype))
        if isinstance(value, (list, tuple)):
            return torch.tensor([float(v) for v in value], dtype=torch.float64 if dev.type == "cpu"
                                else torch.float32, device=dev), (lambda out: out.tolist())
        return torch.tensor([float(value)], dtype=torch.float64 if dev.type == "cpu" else torch.float32,
                            device=dev), (lambda out: out.item())

    def barrier(self) -> None:
        _require_collective(self.policy)
        if self.world_size > 1:
            dist.barrier()

    def all_reduce_sum(self, value: Any) -> Any:
        _require_collective(self.policy)
        if self.world_size == 1:
            return value
        t, back = self._payload(value)
        dist.all_reduce(t)
        return back(t)

    def broadcast(self, value: Any, *, src: int = 0) -> Any:
        _require_collective(self.policy)
        if self.world_size == 1:
            if src != self.rank:
                raise RuntimeError("single-process broadcast only supports src equal to local rank")
            return value
        if isinstance(value, (Tensor, torch.Tensor, list, tuple, int, float)):
            t, back = self._payload(value)
            dist.broadcast(t, src)
            return back(t)
        box = [value]
        dist.broadcast_object_list(box, src=src)
        return box[0]

    def reduce_scatter(self, values: Any) -> Any:
        _require_collective(self.policy)
        if self.world_size == 1:
            if isinstance(values, (list, tuple)) and len(values) == 1:
                return values[0]
            return values
        t, back = self._payload(values)
        if t.numel() % self.world_size:
            raise ValueError("reduce_scatter input must divide by world_size")
        out = torch.empty(t.numel() // self.world_size, dtype=t.dtype, device=t.device)
        if t.device.type == "cpu":
            dist.all_reduce(t)
            out.copy_(t.reshape(self.world_size, -1)[self.rank])
        else:
            dist.reduce_scatter_tensor(out, t.reshape(-1))
        if isinstance(values, Tensor):
            return Tensor._wrap(out.to(values._data.device, values._data.dtype), like=values)
        return out.tolist()

    def all_gather(self, value: Any) -> list[Any]:
        _require_collective(self.policy)
        if self.world_size == 1:
            return [value]
        if isinstance(value, (Tensor, torch.Tensor, list, tuple, int, float)):
            t, back = self._payload(value)
            parts = [torch.empty_like(t) for _ in range(self.world_size)]
            dist.all_gather(parts, t)
            return [back(p) for p in parts]
        box: list[Any] = [None] * self.world_size
        dist.all_gather_object(box, value)
        return box

    @contextmanager
    def no_sync(self) -> Iterator[None]:
        prev = self.synchronized
        self.synchronized = False
        try:
            yield
        finally:
            self.synchronized = prev


def native_nccl_group(policy: DistributedPolicy | None = None):
    """The native ``_core.NcclProcessGroup`` (device-pointer collectives on its
    own stream), bootstrapped like the reference's runtime
    (distributed.py:190-201): from ``UNDERHFS_NCCL_UNIQUE_ID`` (hex) when set,
    otherwise rank 0 creates an id and shares it through the torch.distributed
    store (the process group must be initialised for that)."""
    from underhfs_b200.ops._lib import core

    pol = policy or policy_from_env()
    c = core()
    uid = os.environ.get("UNDERHFS_NCCL_UNIQUE_ID", "")
    if not uid and pol.world_size > 1:
        if not (dist.is_available() and dist.is_initialized()):
            raise RuntimeError("set UNDERHFS_NCCL_UNIQUE_ID (hex, from nccl_create_unique_id_hex) or initialise the "
                               "process group first")
        box = [c.nccl_create_unique_id_hex() if pol.rank == 0 else None]
        dist.broadcast_object_list(box, src=0)
        uid = box[0]
    local = pol.local_rank if pol.local_rank is not None else pol.rank % max(1, torch.cuda.device_count())
    return c.NcclProcessGroup(pol.rank, pol.world_size, uid, local)


def process_group(policy: DistributedPolicy | None = None) -> ProcessGroup:
    return ProcessGroup(init_process_group(policy))


class DistributedDataParallel:
    """Data parallelism over one process per GPU.

    For a TransformerLM running on the fused engine, gradients live in a
    flat fp32 buffer in symmetric memory; as backward finishes each block the
    engine reports the completed range, and full 25 MB buckets are
    all-reduced right away by the fused NVLink kernel on a side stream (1/world
    scale fused), overlapping the remaining backward.  ``synchronize_gradients``
    (reference API) then only joins the side stream.  Other modules get one
    coalesced all-reduce per call.  ``average=False`` sums like the reference
    (distributed.py:162-168); the default averages.
    """

    def __init__(self, module, policy: DistributedPolicy | None = None, *, bucket_mb: float | None = None,
                 average: bool = True, comm_blocks: int = 32) -> None:
        self.module = module
        self.policy = init_process_group(policy)
        self.group = ProcessGroup(self.policy)
        self.average = average
        self._bucketer = None
        flat = getattr(module, "flat", None)
        if flat is not None and self.policy.world_size > 1 and self.policy.backend == "nccl":
            from underhfs_b200.parallel.ddp import BucketedAllReduce

            self._bucketer = BucketedAllReduce(
                module, self.policy, bucket_bytes=int((bucket_mb or self.policy.bucket_mb) * 2**20),
                average=average, blocks=comm_blocks, use_nccl=self.policy.comm_backend == "nccl",
            )

    def __call__(self, *args: Any, **kwargs: Any) -> Any:
        if self._bucketer is not None:
            self._bucketer.arm(enabled=self.group.synchronized)
        return self.module(*args, **kwargs)

    def parameters(self):
        return self.module.parameters()

    def state_dict(self, **kw: Any):
        return self.module.state_dict(**kw)

    @contextmanager
    def no_sync(self) -> Iterator[None]:
        with self.group.no_sync():
            yield

    def synchronize_gradients(self, defer_tail: bool = False) -> int:
        """All-reduce (average) the gradients.  ``defer_tail=True`` (fused
        engine only) returns the flat offset below which the last reduction is
        still running (0: everything is final); call ``wait_gradients()``
        before reading gradients below it."""
        if not self.group.synchronized:
            return 0
        _require_collective(self.policy)
        if self.policy.world_size == 1:
            return 0
        if self._bucketer is not None:
            return self._bucketer.finish(defer_tail=defer_tail)
        params = [p for p in self.module.parameters() if p.grad is not None]
        if not params:
            return 0
        grads = [p.grad._data.detach() for p in params]
        dev = _coll_device(self.policy)
        flat = torch.cat([g.reshape(-1).to(dev, torch.float32) for g in grads])
        dist.all_reduce(flat)
        if self.average:
            flat /= self.policy.world_size
        off = 0
        for p, g in zip(params, grads):
            n = g.numel()
            p.grad = Tensor._wrap(flat[off : off + n].view(g.shape).to(g.device, g.dtype), like=p)
            off += n
        return 0

    def wait_gradients(self) -> None:
        """Complete a ``synchronize_gradients(defer_tail=True)``."""
        if self._bucketer is not None:
            self._bucketer.wait_tail()


DDP = DistributedDataParallel
