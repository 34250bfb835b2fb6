"""Two-GPU correctness of the fused collectives, DDP overlap and ZeRO-2.

Each case runs tests/multigpu_worker.py under torchrun with one process per
GPU; the worker compares against NCCL / single-buffer references.
"""

import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _gpus() -> int:
    try:
        import torch

        return torch.cuda.device_count()
    except Exception:
        return 0

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("case", ["allreduce", "ddp", "ddp_wire", "zero", "zero3", "zero3_api", "native", "cp", "nvls"])
def test_two_gpu_case(case):
    if _gpus() < 2:
        pytest.skip("needs two GPUs")
    if case == "nvls" and os.environ.get("UNDERHFS_TEST_NVLS") != "1":
        pytest.skip("NVLS (multimem) all-reduce is opt-in: UNDERHFS_TEST_NVLS=1 runs its check")
    env = dict(os.environ)
    env["PYTHONPATH"] = str(ROOT) + os.pathsep + env.get("PYTHONPATH", "")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", f"--master-port={_free_port()}",
           str(ROOT / "tests" / "multigpu_worker.py"), case]
    proc = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True)
    if proc.returncode != 0 or f"OK {case}" not in proc.stdout:
        # shown by pytest under "Captured stdout call"
        print(proc.stdout[-4000:])
        print(proc.stderr[-12000:])
    assert proc.returncode == 0 and f"OK {case}" in proc.stdout, f"worker {case} exited {proc.returncode}"
