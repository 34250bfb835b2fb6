"""ZeRO-partitioned AdamW over the flat buffers.

Rank r owns elements [r*S, (r+1)*S) of the flat parameter space (S = padded
total / world).  It keeps fp32 master weights and Adam moments for that
shard only (1/W of the optimizer memory).  Parameters (bf16) and gradients
(fp32) live in one symmetric region, so a single fused kernel per step
(csrc/runtime/comm.cu: rs_adamw_ag_kernel)

  1. reads the owned gradient slice from every peer over NVLink and sums it
     (reduce-scatter, 1/world scale fused),
  2. applies the AdamW update to the owned master / moments,
  3. writes the updated bf16 weights into every peer's parameter buffer
     (all-gather),

replacing the reference's ZeroAwareAdamW stub (optim.py:216-225), which
neither partitions state nor communicates.

``offload="host"`` keeps the moments of the shard in pinned host RAM
(runtime.PinnedHostTier): they are fetched with an async copy on a side
stream before the update and written back after it.
"""

from __future__ import annotations

import torch

from underhfs_b200.ops import kernels as K
from underhfs_b200.ops._lib import core
from underhfs_b200.parallel.symmetric import SymmetricBuffer


class ZeroFlatOptimizer:
    def __init__(self, flat, shard, *, group=None, stage: int = 2, blocks: int = 132,
                 offload: str | None = None) -> None:
        if stage not in (1, 2):
            raise ValueError("ZeroFlatOptimizer implements stages 1 and 2 (stage 3 uses parallel.zero3)")
        self.flat = flat
        self.rank = shard.rank
        self.world = shard.world_size
        self.stage = stage
        self.blocks = blocks
        n = flat.numel
        unit = 4 * self.world
        self.padded = (n + unit - 1) // unit * unit
        self.shard_n = self.padded // self.world
        self.lo = self.rank * self.shard_n
        nbytes = self.padded * 2 + 256 + self.padded * 4
        self.sym = SymmetricBuffer(nbytes, rank=self.rank, world=self.world, group=group)
        params = self.sym.tensor(self.padded, torch.bfloat16)
        grads = self.sym.tensor(self.padded, torch.float32)
        params.zero_()
        self.p_off = params.data_ptr() - self.sym.heap.data_ptr(self.rank)
        self.g_off = grads.data_ptr() - self.sym.heap.data_ptr(self.rank)
        master_full = flat.master
        flat.rehome(params=params, grads=grads)
        dev = flat.device
        self.master = torch.zeros(self.shard_n, dtype=torch.float32, device=dev)
        hi = min(n, self.lo + self.shard_n)
        if hi > self.lo:
            self.master[: hi - self.lo].copy_(master_full[self.lo : hi])
        self.m = torch.zeros_like(self.master)
        self.v = torch.zeros_like(self.master)
        self.step_t = torch.zeros((), dtype=torch.int32, device=dev)
        self.offload = offload
        self.host = None
        if offload == "host":
            from underhfs_b200.runtime import PinnedHostTier

            self.host = PinnedHostTier(dev)
            self.host.offload("m", self.m)
            self.host.offload("v", self.v)
        flat.master = None  # the shard is authoritative now
        self.stream = torch.cuda.current_stream()

    def step(self, *, lr: float, betas: tuple[float, float], eps: float, weight_decay: float,
             decoupled: bool, grad_scale: float | None = None) -> None:
        if self.host is not None:
            self.host.fetch("m", self.m)
            self.host.fetch("v", self.v)
            self.host.wait("m")
            self.host.wait("v")
        K.increment_(self.step_t)
        core().comm_rs_adamw_ag(
            self.sym.heap, self.g_off, self.sym.heap, self.p_off, self.lo, self.shard_n, self.master.data_ptr(),
            self.m.data_ptr(), self.v.data_ptr(), float(lr), float(betas[0]), float(betas[1]), float(eps),
            float(weight_decay), float(1.0 / self.world if grad_scale is None else grad_scale), bool(decoupled),
            self.step_t.data_ptr(), self.blocks, torch.cuda.current_stream().cuda_stream,
        )
        if self.host is not None:
            self.host.offload("m", self.m)
            self.host.offload("v", self.v)

    def shard_state(self) -> dict:
        return {"rank": self.rank, "world": self.world, "lo": self.lo, "shard_n": self.shard_n,
                "master": self.master.detach().cpu(), "m": self.m.detach().cpu(), "v": self.v.detach().cpu(),
                "step": int(self.step_t.item())}
