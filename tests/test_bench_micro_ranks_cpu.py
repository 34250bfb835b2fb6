"""Two ranks of ``bench.py --config micro --impl reference`` on the CPU host:
rank 0's measuring process creates the NCCL id and both ranks reach the
reference's ``ncclCommInitRank`` (which then fails for want of a GPU) instead
of losing NCCL's bootstrap root with a short-lived helper process."""

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_rank_reference_collectives_bootstrap():
    import torch

    if torch.cuda.is_available():
        pytest.skip("with GPUs the collectives really run (a measurement, not a test)")
    if not (ROOT / "baseline" / "_ref" / "underhfs" / "__init__.py").exists():
        pytest.skip("reference not installed under baseline/_ref")
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", UNDERHFS_REF_COLL_MAX_BYTES="1024")
    cmd = ["timeout", "-k", "10", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", f"--master-port={_free_port()}", str(ROOT / "bench.py"),
           "--config", "micro", "--impl", "reference", "--steps", "1", "--warmup", "0"]
    proc = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True)
    assert proc.returncode == 0, proc.stderr[-3000:]
    rows = [json.loads(l) for l in proc.stdout.splitlines() if l.startswith("{")]
    errors = [r.get("error", "") for r in rows]
    assert rows and all("ncclCommInitRank" in e for e in errors), rows
    assert not any("remote process exited" in e for e in errors), rows
