"""Single-node launcher: one process per GPU (torchrun-compatible environment).

``python -m underhfs_b200.parallel.launch --nproc-per-node 8 train.py ...``
spawns N copies of the script with RANK / LOCAL_RANK / WORLD_SIZE /
MASTER_ADDR / MASTER_PORT set, forwards signals, and fails fast: when one
rank exits non-zero the others are terminated and the launcher returns that
exit code.  With ``--max-restarts K`` a failed job is started again (all
ranks, ``UNDERHFS_RESTART_COUNT`` incremented) up to K times; the script is
expected to resume from its last complete checkpoint.  This is the module the
reference's launch plan names but does not ship (distributed.py:47-55).
"""

from __future__ import annotations

import argparse
import os
import signal
import subprocess
import sys
import time


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(prog="underhfs_b200.parallel.launch")
    ap.add_argument("--nproc-per-node", type=int, default=1)
    ap.add_argument("--master-addr", default="127.0.0.1")
    ap.add_argument("--master-port", type=int, default=29511)
    ap.add_argument("--standalone", action="store_true")
    ap.add_argument("--timeout", type=float, default=0.0, help="kill all ranks after this many seconds (0 = none)")
    ap.add_argument("--max-restarts", type=int, default=0, help="restart the whole job this many times on failure")
    ap.add_argument("script")
    ap.add_argument("args", nargs=argparse.REMAINDER)
    a = ap.parse_args(argv)
    code = 0
    for attempt in range(max(0, a.max_restarts) + 1):
        code = _run_once(a, attempt)
        if code == 0 or code == 130:
            break
        if attempt < a.max_restarts:
            print(f"[launch] job failed with exit code {code}; restart {attempt + 1} of {a.max_restarts}",
                  file=sys.stderr, flush=True)
    return code


def _run_once(a, attempt: int) -> int:
    n = max(1, a.nproc_per_node)
    procs: list[subprocess.Popen] = []
    for rank in range(n):
        env = dict(os.environ)
        env.update(RANK=str(rank), LOCAL_RANK=str(rank), WORLD_SIZE=str(n), LOCAL_WORLD_SIZE=str(n),
                   MASTER_ADDR=a.master_addr, MASTER_PORT=str(a.master_port + 2 * attempt),
                   UNDERHFS_RESTART_COUNT=str(attempt))
        cmd = [sys.executable, a.script, *a.args] if a.script.endswith(".py") else \
            [sys.executable, "-m", a.script, *a.args]
        procs.append(subprocess.Popen(cmd, env=env, start_new_session=True))

    def kill_all(sig=signal.SIGTERM) -> None:
        for p in procs:
            if p.poll() is None:
                try:
                    os.killpg(p.pid, sig)
                except ProcessLookupError:
                    pass

    start = time.time()
    code = 0
    try:
        while True:
            states = [p.poll() for p in procs]
            failed = [c for c in states if c not in (None, 0)]
            if failed:
                code = failed[0]
                kill_all()
                break
            if all(c == 0 for c in states):
                break
            if a.timeout and time.time() - start > a.timeout:
                code = 124
                kill_all()
                break
            time.sleep(0.05)
    except KeyboardInterrupt:
        code = 130
        kill_all(signal.SIGINT)
    for p in procs:
        try:
            p.wait(timeout=30)
        except subprocess.TimeoutExpired:
            os.killpg(p.pid, signal.SIGKILL)
    return code


if __name__ == "__main__":
    raise SystemExit(main())
