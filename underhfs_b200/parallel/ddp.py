"""Bucketed gradient all-reduce overlapped with backward.

The engine's flat fp32 gradient buffer is re-homed into symmetric memory.
Bucket boundaries are fixed at construction (every rank identical): equal
``bucket_bytes`` slices counted from the END of the buffer, because backward
completes the last blocks first.  ``on_ready(lo, hi)`` (called by the engine
after each block) launches the buckets that are now entirely final -- as one
launch over their contiguous range -- with the fused two-shot all-reduce
kernel on a high-priority side stream, after an event recorded on the compute
stream.  ``finish()`` flushes the remaining
buckets and makes the compute stream wait for the side stream, so the
optimizer step sees reduced gradients.

Reference: distributed.py:162-168 (one host-staged fp32 NCCL all-reduce per
parameter after backward, no overlap).
"""

from __future__ import annotations

import os

import torch

from underhfs_b200.ops._lib import core
from underhfs_b200.parallel.symmetric import SymmetricBuffer
from underhfs_b200.utils import nvtx


class BucketedAllReduce:
    def __init__(self, model, policy, *, bucket_bytes: int, average: bool, blocks: int = 32,
                 use_nccl: bool = False) -> None:
        self.model = model
        self.policy = policy
        self.world = policy.world_size
        self.rank = policy.rank
        self.scale = 1.0 / self.world if average else 1.0
        self.blocks = blocks
        self.tail_blocks = int(os.environ.get("UNDERHFS_DDP_TAIL_BLOCKS", "148"))
        self.use_nccl = use_nccl
        flat = model.flat
        # UNDERHFS_DDP_WIRE=bf16: gradients cross NVLink as bf16 (cast and
        # scale fused into the all-reduce kernel, fp32 accumulation; every rank
        # ends with the same bf16-rounded gradient), half the bytes of fp32
        self.wire = os.environ.get("UNDERHFS_DDP_WIRE", "fp32") == "bf16" and not use_nccl
        n = (flat.numel + 7) // 8 * 8
        # UNDERHFS_NVLS=1: gradients in memory bound to an NVLink multicast
        # object (allocated through torch's symmetric memory), reduced in the
        # switch by allreduce_nvls_f32_kernel; this heap then only carries the
        # barrier signal pads.  Falls back to the peer-to-peer kernel when the
        # system offers no multicast.
        self.mc = 0
        grads = self._nvls_grads(n) if os.environ.get("UNDERHFS_NVLS", "0") == "1" and not use_nccl else None
        if grads is not None:
            self.wire = False
        nbytes = 4096 if grads is not None else n * 4 + (n * 2 + 256 if self.wire else 0)
        self.sym = SymmetricBuffer(nbytes, rank=self.rank, world=self.world)
        if grads is None:
            grads = self.sym.tensor(n, torch.float32)
        self.wire_off = self.sym.tensor(n, torch.bfloat16).data_ptr() - self.sym.heap.data_ptr(self.rank) \
            if self.wire else 0
        model.rehome_buffers(grads=grads)
        self.flat = model.flat
        self.n = n
        per = max(8, (bucket_bytes // 4) // 8 * 8)
        edges = list(range(n, 0, -per)) + [0]
        self.buckets = [(edges[i + 1], edges[i]) for i in range(len(edges) - 1)]  # descending ranges
        self.stream = torch.cuda.Stream(priority=-1)
        self._next = 0
        self._last = None
        self._enabled = True
        self._launched_any = False
        model.engine.grad_ready = self.on_ready
        # UNDERHFS_DDP_TRACE=1: CUDA events around every bucket (eager steps
        # only) and a per-step report of how much reduction time overlapped
        # the backward kernels
        self.trace = os.environ.get("UNDERHFS_DDP_TRACE", "0") == "1"
        self._trace_events: list = []

    def _nvls_grads(self, n: int):
        """fp32 [n] gradient buffer bound to a multicast object, or None."""
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem

        try:
            group = dist.group.WORLD
            if hasattr(symm_mem, "enable_symm_mem_for_group"):
                symm_mem.enable_symm_mem_for_group(group.group_name)
            buf = symm_mem.empty(n, dtype=torch.float32, device=torch.device("cuda", torch.cuda.current_device()))
            handle = symm_mem.rendezvous(buf, group.group_name)
            mc = int(handle.multicast_ptr)
        except Exception as e:  # no symmetric memory / multicast on this system
            print(f"[ddp] NVLS unavailable ({type(e).__name__}: {e}); using the peer-to-peer all-reduce", flush=True)
            return None
        if mc == 0:
            print("[ddp] NVLS unavailable (no multicast support); using the peer-to-peer all-reduce", flush=True)
            return None
        self._nvls_handle = handle  # keeps the mapping alive
        self.mc = mc + (buf.data_ptr() - int(handle.buffer_ptrs[handle.rank]))
        buf.zero_()
        return buf

    def arm(self, enabled: bool = True) -> None:
        self._next = 0
        self._last = None
        self._enabled = enabled
        self._launched_any = False
        self.model.engine.grad_ready = self.on_ready if enabled else None

    def _launch(self, lo: int, hi: int, blocks: int | None = None) -> None:
        blocks = self.blocks if blocks is None else blocks
        nvtx.push(f"allreduce/bucket[{lo},{hi})")
        compute = torch.cuda.current_stream()
        # every reduction launched before this one is done at `pre`
        pre = torch.cuda.Event()
        pre.record(self.stream)
        self._last = (hi, pre)
        ev = torch.cuda.Event()
        ev.record(compute)
        self.stream.wait_event(ev)
        if self.trace:
            t0 = torch.cuda.Event(enable_timing=True)
            t0.record(compute)  # compute reached this point (bucket final)
        with torch.cuda.stream(self.stream):
            if self.trace:
                s0 = torch.cuda.Event(enable_timing=True)
                s0.record(self.stream)
            if self.use_nccl:
                import torch.distributed as dist

                view = self.flat.grads[lo:hi]
                dist.all_reduce(view)
                if self.scale != 1.0:
                    view.mul_(self.scale)
            elif self.wire:
                core().comm_allreduce_f32_wire_bf16(self.sym.heap, lo * 4, self.wire_off + lo * 2, hi - lo,
                                                    self.scale, blocks, self.stream.cuda_stream)
            elif self.mc:
                core().comm_allreduce_f32_nvls(self.sym.heap, self.mc, lo * 4, hi - lo, self.scale, blocks,
                                               self.stream.cuda_stream)
            else:
                core().comm_allreduce_f32(self.sym.heap, lo * 4, hi - lo, self.scale, blocks,
                                          self.stream.cuda_stream)
            if self.trace:
                s1 = torch.cuda.Event(enable_timing=True)
                s1.record(self.stream)
                self._trace_events.append((t0, s0, s1, hi - lo))
        self._launched_any = True
        nvtx.pop()

    def on_ready(self, lo: int, hi: int) -> None:
        if not self._enabled:
            return
        # buckets that became final together are contiguous: one launch
        first = self._next
        while self._next < len(self.buckets) and self.buckets[self._next][0] >= lo:
            self._next += 1
        if self._next > first:
            self._launch(self.buckets[self._next - 1][0], self.buckets[first][1])

    def finish(self, defer_tail: bool = False) -> int:
        """Launch the remaining buckets and order the compute stream after the
        reductions.  With ``defer_tail`` the compute stream only waits for the
        buckets launched during the backward and the offset below which
        gradients are still being reduced is returned (0 when nothing is
        pending); ``wait_tail()`` completes the wait."""
        # the rest (the embeddings, final only after the last kernel of the
        # backward) in one launch: no per-bucket synchronisation in the tail
        if self._next < len(self.buckets):
            # nothing else runs once the backward is done: the tail reduction
            # gets enough CTAs to keep every SM's peer loads in flight
            self._launch(self.buckets[-1][0], self.buckets[self._next][1], blocks=self.tail_blocks)
            self._next = len(self.buckets)
        if self.trace:
            end = torch.cuda.Event(enable_timing=True)
            end.record(torch.cuda.current_stream())  # backward kernels done
        last, self._last = self._last, None
        if defer_tail and last is not None and not self.trace:
            # the last launch (the embeddings, made final by the end of the
            # backward) covers [.., boundary); everything above is reduced
            boundary, pre = last
            torch.cuda.current_stream().wait_event(pre)
            self._next = 0
            return boundary
        torch.cuda.current_stream().wait_stream(self.stream)
        self._next = 0
        if self.trace and self._trace_events:
            done = torch.cuda.Event(enable_timing=True)
            done.record(torch.cuda.current_stream())
            done.synchronize()
            first = self._trace_events[0][0]
            busy = sum(s0.elapsed_time(s1) for _, s0, s1, _ in self._trace_events)
            start_lag = sum(t0.elapsed_time(s0) for t0, s0, _, _ in self._trace_events)
            tail = end.elapsed_time(done)
            print(f"[ddp trace rank {self.rank}] buckets {len(self._trace_events)}, reduce kernels {busy:.3f} ms, "
                  f"launch lag {start_lag:.3f} ms, from first bucket to backward end {first.elapsed_time(end):.3f} ms, "
                  f"reduction tail after backward {tail:.3f} ms", flush=True)
            self._trace_events = []
        return 0

    def wait_tail(self) -> None:
        """The compute stream waits for every reduction (after finish(defer_tail=True))."""
        torch.cuda.current_stream().wait_stream(self.stream)
