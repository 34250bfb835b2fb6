"""Benchmarks (reference benchmarks.py:14-293) plus device-timed B200 suites.

The reference API (``BenchmarkResult``, ``run_microbenchmarks``,
``run_benchmark_suite``, ``run_memory_benchmark``) is kept; its host
wall-clock timer remains for CPU ops, while CUDA ops are timed with CUDA
events on the launching stream (warm-up first, synchronize on both sides).

Added: ``time_cuda`` (event timing helper), ``op_sweep`` (tcgen05 GEMM vs
cuBLAS at M=N=K in {1024, 4096, 8192}; add/mul on 2^26 elements in
fp32/fp16/bf16 with GB/s) and ``collective_sweep`` (fused all-reduce /
all-gather bus bandwidth at 1 KB .. 1 GB, device-timed, max over ranks).
"""

from __future__ import annotations

from dataclasses import dataclass
from statistics import median
from time import perf_counter
from typing import Any, Callable

import torch

from underhfs_b200.cuda import MemoryPolicy, MemoryTier
from underhfs_b200.native import status as native_status
from underhfs_b200.runtime import MemoryPlanner, OffloadExecutor
from underhfs_b200.tensor import tensor


@dataclass(frozen=True)
class BenchmarkResult:
    name: str
    backend: str
    iterations: int
    seconds: float
    ops_per_second: float
    latency_p50_ms: float
    latency_p95_ms: float
    output_sample: float

    def to_dict(self) -> dict[str, Any]:
        return dict(vars(self))


@dataclass(frozen=True)
class MemoryBenchmarkResult:
    requested_bytes: int
    placements: dict[str, int]
    offload_events: int
    oom_avoided: bool
    bottlenecks: tuple[str, ...]
    prefetch_verified: bool = False

    def to_dict(self) -> dict[str, Any]:
        d = dict(vars(self))
        d["bottlenecks"] = list(self.bottlenecks)
        return d


@dataclass(frozen=True)
class BenchmarkSuiteResult:
    op_microbenchmarks: tuple[BenchmarkResult, ...]
    training: dict[str, Any]
    memory: MemoryBenchmarkResult
    oracle: dict[str, Any]

    def to_dict(self) -> dict[str, Any]:
        return {"op_microbenchmarks": [r.to_dict() for r in self.op_microbenchmarks], "training": self.training,
                "memory": self.memory.to_dict(), "oracle": self.oracle}


def _pct(values: list[float], q: float) -> float:
    if not values:
        return 0.0
    s = sorted(values)
    return s[min(len(s) - 1, max(0, int(round((len(s) - 1) * q))))]


def time_cuda(fn: Callable[[], Any], *, iterations: int = 20, warmup: int = 3) -> list[float]:
    """Per-iteration device milliseconds measured with CUDA events."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(iterations)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(iterations)]
    for i in range(iterations):
        starts[i].record()
        fn()
        ends[i].record()
    torch.cuda.synchronize()
    return [s.elapsed_time(e) for s, e in zip(starts, ends)]


def _bench(name: str, backend: str, iterations: int, warmup: int, fn: Callable[[], float]) -> BenchmarkResult:
    sample = 0.0
    if backend == "cuda":
        box: list[float] = []
        lat = [ms / 1e3 for ms in time_cuda(lambda: box.append(fn()), iterations=iterations, warmup=warmup)]
        sample = box[-1] if box else 0.0
    else:
        for _ in range(warmup):
            sample = fn()
        lat = []
        for _ in range(iterations):
            t0 = perf_counter()
            sample = fn()
            lat.append(perf_counter() - t0)
    total = sum(lat)
    return BenchmarkResult(name, backend, iterations, total, iterations / total if total > 0 else float("inf"),
                           median(lat) * 1e3, _pct(lat, 0.95) * 1e3, float(sample))


def _vec(n: int, off: float = 0.0) -> list[float]:
    return [float((i % 17) + 1) + off for i in range(n)]


def _mat(n: int, off: float = 0.0) -> list[list[float]]:
    return [[float(((r * n + c) % 17) + 1) + off for c in range(n)] for r in range(n)]


def run_microbenchmarks(*, size: int = 32, iterations: int = 20, warmup: int = 3,
                        include_cuda: bool = True) -> list[BenchmarkResult]:
    if size <= 0:
        raise ValueError("size must be positive")
    if iterations <= 0:
        raise ValueError("iterations must be positive")
    if warmup < 0:
        raise ValueError("warmup must be non-negative")
    a, b = tensor(_vec(size)), tensor(_vec(size, 1.0))
    m1, m2 = tensor(_mat(size)), tensor(_mat(size, 1.0))
    out = [
        _bench("add", "cpu", iterations, warmup, lambda: (a + b)._data.reshape(-1)[0].item()),
        _bench("matmul", "cpu", iterations, warmup, lambda: (m1 @ m2)._data.reshape(-1)[0].item()),
    ]
    if include_cuda and native_status().cuda_enabled:
        ca, cb, cm1, cm2 = a.cuda(), b.cuda(), m1.cuda(), m2.cuda()
        out.append(_bench("add", "cuda", iterations, warmup, lambda: (ca + cb)._data.reshape(-1)[0]))
        out.append(_bench("matmul", "cuda", iterations, warmup, lambda: (cm1 @ cm2)._data.reshape(-1)[0]))
        out = [r if r.backend != "cuda" else BenchmarkResult(r.name, r.backend, r.iterations, r.seconds,
               r.ops_per_second, r.latency_p50_ms, r.latency_p95_ms, float(r.output_sample)) for r in out]
    return out


def _training_benchmark(*, steps: int) -> dict[str, Any]:
    from underhfs_b200.functional import mse_loss
    from underhfs_b200.nn import Linear
    from underhfs_b200.optim import SGD

    model = Linear(4, 4)
    opt = SGD(model.parameters(), lr=1e-3)
    x = tensor([[1.0, 2.0, 3.0, 4.0]])
    y = tensor([[0.5, 1.0, 1.5, 2.0]])
    losses = []
    t0 = perf_counter()
    for _ in range(steps):
        opt.zero_grad()
        loss = mse_loss(model(x), y)
        losses.append(loss.item())
        loss.backward()
        opt.step()
    dt = perf_counter() - t0
    return {"name": "linear_mse_training", "backend": "underhfs", "steps": steps, "seconds": dt,
            "steps_per_second": steps / dt if dt > 0 else float("inf"), "initial_loss": losses[0],
            "final_loss": losses[-1]}


def _oracle_benchmark(*, size: int) -> dict[str, Any]:
    left, right = _mat(size), _mat(size, 1.0)
    t0 = perf_counter()
    ours = tensor(left) @ tensor(right)
    t1 = perf_counter()
    ref = torch.tensor(left, dtype=torch.float32) @ torch.tensor(right, dtype=torch.float32)
    t2 = perf_counter()
    return {"available": True, "backend": "torch", "op": "matmul", "size": size, "underhfs_seconds": t1 - t0,
            "torch_seconds": t2 - t1,
            "max_sample_abs_diff": abs(float(ours._storage[0]) - float(ref.reshape(-1)[0].item()))}


def run_memory_benchmark(*, tensor_bytes: tuple[int, ...] = (64, 128, 256), policy: MemoryPolicy | None = None,
                         budgets: dict[MemoryTier, int] | None = None) -> MemoryBenchmarkResult:
    pol = policy or MemoryPolicy(tiers=(MemoryTier.VRAM, MemoryTier.RAM, MemoryTier.NVME))
    caps = budgets or {MemoryTier.VRAM: 128, MemoryTier.RAM: 256, MemoryTier.NVME: 512}
    planner = MemoryPlanner(pol, caps)
    placed = {t.value: 0 for t in pol.tiers}
    events = 0
    for n in tensor_bytes:
        p = planner.place_bytes(n)
        placed[p.tier.value] += p.bytes
        if p.reason == "oversubscribed-offload" or p.tier is not pol.tiers[0]:
            events += 1
    snap = planner.snapshot()
    hot = tuple(t for t, s in snap.items() if s["capacity_bytes"] > 0 and s["used_bytes"] > s["capacity_bytes"])
    verified = False
    if MemoryTier.NVME in pol.tiers:
        ex = OffloadExecutor(pol)
        h = ex.offload_tensor(tensor([1.0, 2.0]), MemoryTier.NVME)
        try:
            verified = ex.load_tensor(ex.prefetch_tensor(h)).tolist() == [1.0, 2.0]
        finally:
            ex.release(h)
    return MemoryBenchmarkResult(sum(tensor_bytes), placed, events, events > 0 and pol.allow_offload, hot, verified)


def run_benchmark_suite(*, size: int = 16, iterations: int = 5, warmup: int = 1, include_cuda: bool = True,
                        include_oracle: bool = True) -> BenchmarkSuiteResult:
    micro = tuple(run_microbenchmarks(size=size, iterations=iterations, warmup=warmup, include_cuda=include_cuda))
    return BenchmarkSuiteResult(micro, _training_benchmark(steps=max(2, iterations)), run_memory_benchmark(),
                                _oracle_benchmark(size=size) if include_oracle
                                else {"available": False, "reason": "disabled"})


# ----------------------------------------------------------- B200 sweeps
def op_sweep(*, sizes=(1024, 4096, 8192), ew_elems: int = 1 << 26, iterations: int = 20) -> dict[str, Any]:
    """Device-timed tcgen05 GEMM vs cuBLAS (TFLOP/s) and elementwise GB/s."""
    from underhfs_b200.ops import kernels as K

    out: dict[str, Any] = {"gemm_bf16": [], "elementwise": []}
    for n in sizes:
        a = torch.randn(n, n, device="cuda", dtype=torch.bfloat16)
        b = torch.randn(n, n, device="cuda", dtype=torch.bfloat16)
        ours = median(time_cuda(lambda: K.linear_fwd(a, b), iterations=iterations))
        cub = median(time_cuda(lambda: a @ b.t(), iterations=iterations))
        fl = 2.0 * n ** 3
        out["gemm_bf16"].append({"M=N=K": n, "tflops": fl / ours / 1e9, "cublas_tflops": fl / cub / 1e9,
                                 "ms": ours, "cublas_ms": cub})
    for dt in (torch.float32, torch.float16, torch.bfloat16):
        x = torch.randn(ew_elems, device="cuda").to(dt)
        y = torch.randn(ew_elems, device="cuda").to(dt)
        for name, op in (("add", K.OP_ADD), ("mul", K.OP_MUL)):
            ms = median(time_cuda(lambda: K.ew_binary(op, x, y), iterations=iterations))
            nbytes = 3 * ew_elems * x.element_size()
            out["elementwise"].append({"op": name, "dtype": str(dt).replace("torch.", ""), "elements": ew_elems,
                                       "ms": ms, "gbs": nbytes / ms / 1e6})
    return out


def main(argv: list[str] | None = None) -> int:
    """``python -m underhfs_b200.benchmarks ops``: the op sweep as one JSON document
    (bf16 GEMM at M=N=K 1024 / 4096 / 8192 against cuBLAS, add / mul on 2^26
    elements in fp32 / fp16 / bf16)."""
    import argparse
    import json

    ap = argparse.ArgumentParser(description="device-timed op microbenchmarks")
    ap.add_argument("suite", choices=("ops",))
    ap.add_argument("--iterations", type=int, default=20)
    args = ap.parse_args(argv)
    if not torch.cuda.is_available():
        print(json.dumps({"suite": args.suite, "unavailable": "no CUDA device"}))
        return 0
    print(json.dumps(op_sweep(iterations=args.iterations), indent=2))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
