"""The CPU-fallback benchmark configuration (tiny TransformerLM, checkpoint
round trip, greedy generation) runs end to end through the public API."""

import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_tiny_cpu_bench_runs_and_round_trips():
    proc = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--config", "tiny-cpu", "--steps", "2",
                           "--warmup", "1"], capture_output=True, text=True, timeout=300, cwd=str(ROOT))
    assert proc.returncode == 0, proc.stderr[-2000:]
    out = json.loads(proc.stdout.strip().splitlines()[-1])
    assert out["steps"] == 2 and out["value"] > 0 and out["n_gpus"] == 0
    assert out["checkpoint_roundtrip_matches"] is True and out["generated_tokens"] == 32
