"""Failure detection and elastic restart for multi-process training (host side).

GPU kernels never fault, trap or spin forever on purpose: every device wait
is bounded and reports a status code (csrc/kernels/common.cuh).  Failures of
whole ranks are detected on the host, between steps, before any rank enters
the next collective with a dead peer:

* ``Heartbeat``: every rank publishes ``(step, wall time)`` under its own key
  in a key-value store after each step; a watchdog thread compares every
  peer's last beat with a deadline and records the first peer that is dead
  (never beats again) or stalled (beats too slowly).  ``check()`` raises
  ``PeerFailure`` naming the rank; the training loop calls it between steps.
* ``rendezvous``: process-group start-up with a deadline, so a rank that
  never joins becomes a ``RendezvousTimeout`` on the others instead of a hang.
* Collectives inside a step are bounded by the process group's (short)
  timeout, which ends them with an error if a peer died mid-step.
* Elastic restart lives in the launcher (``parallel/launch.py
  --max-restarts``): when a rank fails every rank is stopped and the job is
  started again with ``UNDERHFS_RESTART_COUNT`` incremented; the script
  resumes from its last complete checkpoint (``serialization.load_training_state``),
  whose checksums reject a corrupted shard.

The reference has no heartbeat, restart or fault injection; it only turns
NCCL error codes into exceptions (cpp/nccl_runtime.cpp:25-29).
"""

from __future__ import annotations

import os
import threading
import time
from datetime import timedelta


class PeerFailure(RuntimeError):
    """A peer rank stopped making progress (dead or stalled)."""

    def __init__(self, rank: int, reason: str) -> None:
        super().__init__(f"rank {rank} failed: {reason}")
        self.rank = rank
        self.reason = reason


class RendezvousTimeout(RuntimeError):
    pass


def make_store(rank: int, world: int, *, host: str | None = None, port: int | None = None,
               timeout_s: float = 10.0):
    """TCP key-value store shared by the ranks (rank 0 hosts it)."""
    import torch.distributed as dist

    host = host or os.environ.get("MASTER_ADDR", "127.0.0.1")
    port = port if port is not None else int(os.environ.get("MASTER_PORT", "29511")) + 1
    return dist.TCPStore(host, port, world, rank == 0, timedelta(seconds=timeout_s), wait_for_workers=False)


def rendezvous(rank: int, world: int, *, backend: str = "gloo", timeout_s: float = 10.0, store=None) -> None:
    """init_process_group with a deadline on every rank having joined."""
    import torch.distributed as dist

    store = store or make_store(rank, world, timeout_s=timeout_s)
    store.set(f"rdzv/{rank}", "1")
    deadline = time.time() + timeout_s
    keys = [f"rdzv/{r}" for r in range(world)]
    while not store.check(keys):
        if time.time() > deadline:
            missing = [r for r in range(world) if not store.check([f"rdzv/{r}"])]
            raise RendezvousTimeout(f"ranks {missing} did not join within {timeout_s:.1f} s")
        time.sleep(0.02)
    dist.init_process_group(backend, store=store, rank=rank, world_size=world,
                            timeout=timedelta(seconds=timeout_s))


class Heartbeat:
    """Per-rank liveness over a key-value store, checked by a watchdog thread."""

    def __init__(self, store, rank: int, world: int, *, deadline_s: float = 5.0, interval_s: float = 0.05,
                 grace_s: float | None = None) -> None:
        self.store = store
        self.rank, self.world = rank, world
        self.deadline_s = deadline_s
        self.interval_s = interval_s
        self.grace_s = deadline_s if grace_s is None else grace_s
        self._failed: PeerFailure | None = None
        self._stop = threading.Event()
        self._t0 = time.time()
        self.beat(-1)
        self._thread = threading.Thread(target=self._watch, daemon=True)
        self._thread.start()

    def beat(self, step: int) -> None:
        self.store.set(f"hb/{self.rank}", f"{step}:{time.time():.6f}")

    def _last(self, r: int) -> tuple[int, float] | None:
        key = f"hb/{r}"
        if not self.store.check([key]):
            return None
        step, t = self.store.get(key).decode().split(":")
        return int(step), float(t)

    def _watch(self) -> None:
        while not self._stop.wait(self.interval_s):
            now = time.time()
            for r in range(self.world):
                if r == self.rank:
                    continue
                try:
                    last = self._last(r)
                except Exception as e:  # the store itself went away (its host rank died)
                    self._failed = self._failed or PeerFailure(0, f"store unreachable (rank 0 hosts it): {e}")
                    return
                if last is None:
                    if now - self._t0 > self.grace_s:
                        self._failed = self._failed or PeerFailure(r, "never joined the heartbeat")
                    continue
                step, t = last
                if now - t > self.deadline_s:
                    self._failed = self._failed or PeerFailure(
                        r, f"no heartbeat for {now - t:.2f} s (last step {step})")

    def check(self) -> None:
        """Raise PeerFailure if any peer is dead or stalled; call between steps."""
        if self._failed is not None:
            raise self._failed

    def close(self) -> None:
        self._stop.set()
        self._thread.join(timeout=2 * self.interval_s + 1.0)


def restart_count() -> int:
    """How many times the launcher has restarted this job (0 on the first run)."""
    return int(os.environ.get("UNDERHFS_RESTART_COUNT", "0"))
