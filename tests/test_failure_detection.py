"""Host-side failure detection on CPU processes (no GPU is involved).

Every scenario makes the failure on the host -- a rank that exits, stalls,
never joins, or a checkpoint shard with a flipped byte -- and checks that the
survivors report it with a clear error within a deadline instead of hanging.
"""

from __future__ import annotations

import multiprocessing as mp
import os
import socket
import sys
import time
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _heartbeat_worker(rank, world, port, scenario, q):
    sys.path.insert(0, str(ROOT))
    from underhfs_b200.parallel.elastic import Heartbeat, PeerFailure, make_store

    store = make_store(rank, world, port=port, timeout_s=30.0)
    # start together: process start-up (spawn + imports) can differ by seconds
    # under load, which must not read as a rank that never joined
    store.set(f"up/{rank}", "1")
    store.wait([f"up/{r}" for r in range(world)])
    hb = Heartbeat(store, rank, world, deadline_s=1.0, interval_s=0.05, grace_s=20.0)
    try:
        for step in range(200):
            hb.beat(step)
            if scenario == "dead" and rank == world - 1 and step == 3:
                os._exit(7)  # the process dies without any goodbye
            if scenario == "stalled" and rank == 1 and step == 3:
                time.sleep(4.0)
            time.sleep(0.05)
            hb.check()
        q.put((rank, "missed", -1))
    except PeerFailure as e:
        q.put((rank, "detected", e.rank))
    finally:
        hb.close()


def _run(target, world, args, timeout=60.0, ranks=None):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=target, args=(r, world, *args, q)) for r in (ranks or range(world))]
    for p in procs:
        p.start()
    deadline = time.time() + timeout
    for p in procs:
        p.join(timeout=max(0.1, deadline - time.time()))
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()  # these exact child processes only
        p.join(timeout=5)
    results = []
    while not q.empty():
        results.append(q.get())
    return results, alive


def test_dead_rank_is_detected_by_survivors():
    port = _port()
    results, hung = _run(_heartbeat_worker, 3, (port, "dead"))
    assert not hung
    survivors = {r: (kind, who) for r, kind, who in results}
    assert survivors.get(0) == ("detected", 2) and survivors.get(1) == ("detected", 2), results


def test_stalled_rank_is_detected():
    port = _port()
    results, hung = _run(_heartbeat_worker, 2, (port, "stalled"))
    assert not hung
    assert (0, "detected", 1) in results, results


def _rendezvous_worker(rank, world, port, q):
    sys.path.insert(0, str(ROOT))
    from underhfs_b200.parallel.elastic import RendezvousTimeout, make_store, rendezvous

    t0 = time.time()
    try:
        rendezvous(rank, world, timeout_s=1.5, store=make_store(rank, world, port=port, timeout_s=3.0))
        q.put((rank, "joined", time.time() - t0))
    except RendezvousTimeout as e:
        q.put((rank, "timeout:" + str(e), time.time() - t0))


def test_dropped_rendezvous_times_out():
    port = _port()
    results, hung = _run(_rendezvous_worker, 2, (port,), ranks=[0])  # rank 1 never starts
    assert not hung
    (rank, kind, waited), = results
    assert kind.startswith("timeout:") and "[1]" in kind and waited < 10, results


def _collective_worker(rank, world, port, q):
    sys.path.insert(0, str(ROOT))
    import torch
    import torch.distributed as dist

    from underhfs_b200.parallel.elastic import make_store, rendezvous

    rendezvous(rank, world, timeout_s=3.0, store=make_store(rank, world, port=port, timeout_s=3.0))
    if rank == 1:
        os._exit(5)  # leaves between steps; never enters the collective
    t0 = time.time()
    try:
        dist.all_reduce(torch.ones(4))
        q.put((rank, "completed", time.time() - t0))
    except Exception as e:  # gloo reports the closed peer or the group timeout
        q.put((rank, "error:" + type(e).__name__, time.time() - t0))


def test_collective_with_dead_peer_errors_instead_of_hanging():
    port = _port()
    results, hung = _run(_collective_worker, 2, (port,))
    assert not hung
    mine = [r for r in results if r[0] == 0]
    assert mine and mine[0][1].startswith("error:") and mine[0][2] < 30, results


def test_corrupted_checkpoint_shard_is_rejected(tmp_path):
    import torch

    from underhfs_b200.serialization import load_sharded_checkpoint, save_sharded_checkpoint

    for r in range(2):
        save_sharded_checkpoint(tmp_path, rank=r, world_size=2, state={"w": torch.arange(64.0) + r})
    assert torch.equal(load_sharded_checkpoint(tmp_path, rank=1)["shards"][1]["w"], torch.arange(64.0) + 1)
    shard = tmp_path / "rank1.uhfsbin"
    data = bytearray(shard.read_bytes())
    data[-5] ^= 0x40  # one flipped bit in the payload
    shard.write_bytes(bytes(data))
    with pytest.raises(Exception, match="checksum mismatch"):
        load_sharded_checkpoint(tmp_path, rank=1)


def test_launcher_restarts_a_failed_job(tmp_path):
    from underhfs_b200.parallel import launch

    marker = tmp_path / "done"
    script = tmp_path / "job.py"
    script.write_text(
        "import os, sys\n"
        f"marker = {str(marker)!r}\n"
        "if os.environ['UNDERHFS_RESTART_COUNT'] == '0' and os.environ['RANK'] == '1':\n"
        "    sys.exit(3)\n"
        "if os.environ['UNDERHFS_RESTART_COUNT'] == '1' and os.environ['RANK'] == '0':\n"
        "    open(marker, 'w').write('ok')\n"
    )
    code = launch.main(["--nproc-per-node", "2", "--master-port", str(_port()), "--max-restarts", "1",
                        "--timeout", "60", str(script)])
    assert code == 0 and marker.read_text() == "ok"
    assert launch.main(["--nproc-per-node", "2", "--master-port", str(_port()), "--timeout", "60",
                        str(script)]) == 3  # no restarts allowed: the failure is reported
