"""Training loop front-end: model presets and the ``Trainer``.

A ``Trainer`` owns one TransformerLM on the fused CUDA engine, its optimizer
(FusedAdamW, or ZeRO-partitioned AdamW) and, for several GPUs, the
data-parallel wrapper.  ``step(ids, targets)`` runs zero-grad, forward with
the fused loss, backward with bucketed gradient all-reduce overlapped, and
the optimizer update.  With ``cuda_graph=True`` the whole step is captured
once into a CUDA graph and every later step is one graph launch fed through
static input buffers; ``step_from_host`` adds the pinned host->device copy of
the batch and returns the loss to the host, which is the end-to-end path a
user drives.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from underhfs_b200.models.transformer import LMSpec

PRESETS: dict[str, LMSpec] = {
    # reference-scale byte LM (CPU path, d_model 64, 2 blocks, 4 heads)
    "tiny": LMSpec(256, 64, 64, 256, 2, heads=4, tied=False),
    "125m": LMSpec(32000, 1024, 768, 3072, 12, heads=12, tied=True),
    "1.3b": LMSpec(32000, 2048, 2048, 8192, 24, heads=16, tied=True),
    "7b": LMSpec(32000, 4096, 4096, 11008, 32, heads=32, tied=False),
}


@dataclass
class TrainConfig:
    model: str = "125m"
    batch: int = 16
    seq_len: int = 1024
    lr: float = 3e-4
    betas: tuple[float, float] = (0.9, 0.95)
    eps: float = 1e-8
    weight_decay: float = 0.0
    decoupled: bool = True
    zero_stage: int = 0
    bucket_mb: float = 25.0
    cuda_graph: bool = True
    seed: int = 0
    init: str = "normal"
    # every rank trains on its zigzag shard of the same sequences (the whole
    # world is one context-parallel group; gradients are averaged by DDP)
    context_parallel: bool = False
    # ZeRO-3 Adam moments: "auto" (the memory planner decides), "host", "device"
    offload: str = "auto"


def build_model(cfg: TrainConfig, device: str = "cuda"):
    from underhfs_b200.nn import TransformerLM

    spec = PRESETS[cfg.model]
    model = TransformerLM(spec.vocab_size, spec.max_seq_len, spec.features, spec.hidden_features, spec.layers,
                          heads=spec.heads, tied=spec.tied, init=cfg.init, seed=cfg.seed, eps=1e-6)
    if device.startswith("cuda"):
        model.to(device, dtype="bf16")
    return model


class StepMeter:
    """Per-step training metrics for logs: device time of the step from CUDA
    events on the current stream (taken as the max over ranks, a small
    all-reduce), tokens/s of the whole job, model FLOPs utilisation against
    ``peak_tflops`` per GPU, and the peak device memory of the step."""

    def __init__(self, *, world: int, tokens_per_rank: int, flops_per_token: float, peak_tflops: float) -> None:
        self.world = world
        self.tokens_per_rank = tokens_per_rank
        self.flops_per_token = flops_per_token
        self.peak_tflops = peak_tflops
        self._t0 = self._t1 = None

    def start(self) -> None:
        torch.cuda.reset_peak_memory_stats()
        self._t0 = torch.cuda.Event(enable_timing=True)
        self._t1 = torch.cuda.Event(enable_timing=True)
        self._t0.record()

    def stop(self) -> dict:
        self._t1.record()
        self._t1.synchronize()
        ms = self._t0.elapsed_time(self._t1)
        if self.world > 1:
            import torch.distributed as dist

            t = torch.tensor([ms], dtype=torch.float64, device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        tokens = self.tokens_per_rank * self.world
        tps = tokens / (ms / 1e3)
        achieved = tps * self.flops_per_token / self.world / 1e12  # TFLOP/s per GPU
        return {"ms": ms, "tokens_per_s": tps, "tflops_per_gpu": achieved,
                "mfu": achieved / self.peak_tflops if self.peak_tflops else None,
                "max_memory_gb": torch.cuda.max_memory_allocated() / 2**30}


class PendingLoss:
    """A step's loss on its way to the host: the device-to-host copy is queued
    on the stream behind the step, and result() waits for that copy only."""

    def __init__(self, host: torch.Tensor, ready: torch.cuda.Event) -> None:
        self._host = host
        self._ready = ready

    def result(self) -> float:
        self._ready.synchronize()
        return float(self._host.item())


class Trainer:
    def __init__(self, model, cfg: TrainConfig, *, policy=None) -> None:
        from underhfs_b200.distributed import DistributedDataParallel, policy_from_env
        from underhfs_b200.optim import FusedAdamW, ZeroAwareAdamW, ZeroShard

        self.model = model
        self.cfg = cfg
        self.policy = policy or policy_from_env(bucket_mb=cfg.bucket_mb, zero_stage=cfg.zero_stage)
        self.world = self.policy.world_size
        self.ddp = None
        if self.world > 1 and cfg.zero_stage == 0:
            self.ddp = DistributedDataParallel(model, self.policy, bucket_mb=cfg.bucket_mb)
        self.cp = None
        if cfg.context_parallel:
            if self.world < 2 or cfg.zero_stage != 0:
                raise ValueError("context_parallel needs world_size > 1 and data-parallel (zero_stage 0) gradients")
            from underhfs_b200.parallel.context import enable_context_parallel

            self.cp = enable_context_parallel(model.engine, cfg.seq_len)
            # the attention's K/V all-gather / dK-dV reduce-scatter run as
            # NCCL collectives from Python; the step stays eager
            cfg.cuda_graph = False
        if cfg.zero_stage > 0:
            if self.world > 1:
                from underhfs_b200.distributed import init_process_group

                init_process_group(self.policy)
            extra = {}
            if cfg.zero_stage == 3:
                # per-unit gathers and reductions synchronise with peers through
                # flags whose epochs advance on the host: the step stays eager
                cfg.cuda_graph = False
                extra = dict(offload=cfg.offload,
                             activation_bytes=model.spec.activation_bytes(cfg.batch, cfg.seq_len))
            self.opt = ZeroAwareAdamW(model.parameters(), ZeroShard(self.policy.rank, self.world),
                                      stage=cfg.zero_stage, lr=cfg.lr, betas=cfg.betas, eps=cfg.eps,
                                      weight_decay=cfg.weight_decay, decoupled=cfg.decoupled, **extra)
        else:
            self.opt = FusedAdamW(model.parameters(), lr=cfg.lr, betas=cfg.betas, eps=cfg.eps,
                                  weight_decay=cfg.weight_decay, decoupled=cfg.decoupled)
        dev = model._engine_device()
        local_len = cfg.seq_len // self.world if self.cp is not None else cfg.seq_len
        self.static_ids = torch.zeros((cfg.batch, local_len), dtype=torch.int64, device=dev)
        self.static_tg = torch.zeros_like(self.static_ids)
        self.static_batch = torch.zeros((2, cfg.batch, local_len), dtype=torch.int64, device=dev)
        self._full_batch = (torch.zeros((2, cfg.batch, cfg.seq_len), dtype=torch.int64, device=dev)
                            if self.cp is not None else None)
        self._graph = None
        self._graph_loss = None
        self.steps_done = 0

    def _eager_step(self, ids: torch.Tensor, tg: torch.Tensor) -> torch.Tensor:
        self.model.zero_grad()
        runner = self.ddp if self.ddp is not None else self.model
        loss = runner(ids, tg)
        loss.backward()
        if self.ddp is not None and hasattr(self.opt, "step_split"):
            # the embedding gradients are final last (tied head): update every
            # other parameter while their all-reduce is still running
            boundary = self.ddp.synchronize_gradients(defer_tail=True)
            if boundary > 0:
                self.opt.step_split(boundary, self.ddp.wait_gradients)
            else:
                self.opt.step()
        else:
            if self.ddp is not None:
                self.ddp.synchronize_gradients()
            self.opt.step()
        return loss._data if hasattr(loss, "_data") else loss

    def _state_tensors(self) -> list[torch.Tensor]:
        """Every tensor a training step mutates (weights, master, moments, step counters)."""
        f = self.model.flat
        out = [f.params]
        if f.master is not None:
            out.append(f.master)
        for name in ("_m_flat", "_v_flat", "_step_t"):
            t = getattr(self.opt, name, None)
            if isinstance(t, torch.Tensor):
                out.append(t)
        z = getattr(self.opt, "_zero", None)
        if z is not None:
            out += [z.master, z.m, z.v, z.step_t]
        return out

    def _capture(self) -> None:
        # warm-up steps (kernel attributes, allocator pool, workspaces) must not
        # change the training trajectory: snapshot and restore the state
        saved = [t.detach().clone() for t in self._state_tensors()]
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(2):
                self._eager_step(self.static_batch[0], self.static_batch[1])
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self._graph_loss = self._eager_step(self.static_batch[0], self.static_batch[1])
        self._graph = g
        for t, s in zip(self._state_tensors(), saved):
            t.copy_(s)
        torch.cuda.synchronize()

    def step(self, ids: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        """One optimizer step on device-resident ids/targets [B, T]; returns the device loss."""
        self.steps_done += 1
        if not self.cfg.cuda_graph:
            return self._eager_step(ids, targets)
        if ids.data_ptr() != self.static_batch[0].data_ptr():
            self.static_batch[0].copy_(ids, non_blocking=True)
            self.static_batch[1].copy_(targets, non_blocking=True)
        if self._graph is None:
            self._capture()
        self._graph.replay()
        return self._graph_loss

    def local_batch(self, ids: torch.Tensor, targets: torch.Tensor):
        """This rank's part of full-sequence ids / targets [B, T] (the identity
        without context parallelism)."""
        if self.cp is None:
            return ids, targets
        from underhfs_b200.parallel.context import shard_sequence

        return (shard_sequence(ids, self.cp.rank, self.cp.size), shard_sequence(targets, self.cp.rank, self.cp.size))

    def step_from_host(self, host_batch: torch.Tensor, *, wait: bool = True):
        """End-to-end step: pinned host [2, B, T] int64 batch in, host float loss out.
        With context parallelism every rank passes the same full sequences.

        ``wait=False`` queues the step and the copy of its loss to pinned host
        memory and returns a PendingLoss at once, so the host can queue the
        next step before reading this one's loss (``.result()``).  A
        PendingLoss stays valid until two more asynchronous steps have been
        queued; the host batch must not change until its result() returned."""
        if self.cp is not None:
            self._full_batch.copy_(host_batch, non_blocking=True)
            ids, tg = self.local_batch(self._full_batch[0], self._full_batch[1])
            self.static_batch[0].copy_(ids)
            self.static_batch[1].copy_(tg)
        else:
            self.static_batch.copy_(host_batch, non_blocking=True)
        loss = self.step(self.static_batch[0], self.static_batch[1])
        if wait:
            return float(loss.item())
        if not hasattr(self, "_loss_ring"):
            self._loss_ring = [torch.empty((), dtype=torch.float32, pin_memory=True) for _ in range(2)]
            self._ring_pos = 0
        host = self._loss_ring[self._ring_pos]
        self._ring_pos ^= 1
        host.copy_(loss.detach().reshape(()).float(), non_blocking=True)
        ready = torch.cuda.Event()
        ready.record()
        return PendingLoss(host, ready)

    def release(self) -> None:
        """Drop the captured graph and, at ZeRO stage 3, the sharded runtime's
        symmetric buffers (before destroying the process group)."""
        self._graph = None
        self._graph_loss = None
        z = getattr(self.opt, "zero3", None)
        if z is not None:
            torch.cuda.synchronize()
            z.close()
