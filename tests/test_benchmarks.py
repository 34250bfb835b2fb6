"""Benchmark API contracts (CPU results, memory pressure, suite)."""

from underhfs.benchmarks import run_benchmark_suite, run_memory_benchmark, run_microbenchmarks
from underhfs.cuda import MemoryPolicy, MemoryTier


def test_cpu_microbenchmarks():
    rows = [r.to_dict() for r in run_microbenchmarks(size=2, iterations=1, warmup=1, include_cuda=False)]
    assert [r["name"] for r in rows] == ["add", "matmul"]
    assert all(r["backend"] == "cpu" and r["ops_per_second"] > 0 for r in rows)
    assert all(r["latency_p95_ms"] >= r["latency_p50_ms"] >= 0 for r in rows)


def test_memory_pressure_and_prefetch():
    d = run_memory_benchmark(tensor_bytes=(16, 16, 16),
                             policy=MemoryPolicy(tiers=(MemoryTier.VRAM, MemoryTier.NVME), allow_offload=True),
                             budgets={MemoryTier.VRAM: 16, MemoryTier.NVME: 16}).to_dict()
    assert d["requested_bytes"] == 48
    assert d["placements"] == {"vram": 16, "nvme": 32}
    assert d["offload_events"] == 2 and d["oom_avoided"] is True and d["prefetch_verified"] is True


def test_suite_contract():
    d = run_benchmark_suite(size=2, iterations=2, warmup=0, include_cuda=False, include_oracle=False).to_dict()
    assert d["op_microbenchmarks"]
    assert d["training"]["steps"] == 2 and d["training"]["steps_per_second"] > 0
    assert d["memory"]["oom_avoided"] is True
    assert d["oracle"]["available"] is False
