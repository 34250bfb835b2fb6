"""Tier stores behind one interface, planner-driven placement and the
optimizer-state decision that selects ZeRO-3 moment offload."""

import pytest

from underhfs_b200.cuda import MemoryPolicy, MemoryTier
from underhfs_b200.runtime import (
    FileStore,
    MemoryPlanner,
    NetworkOffloadClient,
    NetworkOffloadServer,
    OffloadExecutor,
    PinnedHostTier,
    Placement,
)
from underhfs_b200.tensor import DType, tensor


def test_optimizer_state_stays_on_device_when_it_fits():
    pl = MemoryPlanner(MemoryPolicy(tiers=(MemoryTier.VRAM, MemoryTier.RAM)),
                       budgets={MemoryTier.VRAM: 1000, MemoryTier.RAM: 10_000})
    p = pl.place_optimizer_state(600, device_headroom=300)
    assert p.tier is MemoryTier.VRAM and pl.snapshot()["vram"]["used_bytes"] == 600
    # the next 600 no longer fit next to the headroom: pinned host RAM
    q = pl.place_optimizer_state(600, device_headroom=300)
    assert q.tier is MemoryTier.RAM and q.reason == "device-full-pinned-host"
    pl.release(p)
    assert pl.snapshot()["vram"]["used_bytes"] == 0


def test_optimizer_state_without_room_anywhere_raises():
    pl = MemoryPlanner(MemoryPolicy(tiers=(MemoryTier.VRAM, MemoryTier.RAM), allow_offload=False),
                       budgets={MemoryTier.VRAM: 10, MemoryTier.RAM: 10})
    with pytest.raises(MemoryError):
        pl.place_optimizer_state(100)


def test_reserve_counts_existing_bytes():
    pl = MemoryPlanner(MemoryPolicy(tiers=(MemoryTier.VRAM, MemoryTier.RAM)),
                       budgets={MemoryTier.VRAM: 16, MemoryTier.RAM: 64})
    pl.reserve(MemoryTier.VRAM, 12)
    assert pl.place_tensor(tensor([1.0, 2.0], dtype=DType.FP32)).tier is MemoryTier.RAM


def test_for_device_on_cpu_has_host_budget_only():
    pl = MemoryPlanner.for_device("cpu", host_bytes=1 << 20)
    snap = pl.snapshot()
    assert snap["vram"]["capacity_bytes"] == 0 and snap["ram"]["capacity_bytes"] == 1 << 20
    assert pl.place_optimizer_state(1000).tier is MemoryTier.RAM


def test_executor_routes_every_tier_through_one_interface(tmp_path):
    srv = NetworkOffloadServer(port=0).start()
    try:
        ex = OffloadExecutor(MemoryPolicy(scratch_path=str(tmp_path)), network=NetworkOffloadClient(srv.url),
                             host=PinnedHostTier("cpu"))
        value = tensor([[1.0, -2.0], [3.5, 4.0]])
        for tier in (MemoryTier.NVME, MemoryTier.NETWORK, MemoryTier.RAM):
            h = ex.offload_tensor(value, tier)
            assert h.tier is tier
            assert ex.load_tensor(h).tolist() == value.tolist()
            cached = ex.prefetch_tensor(h)
            assert cached.cached and ex.load_tensor(cached).tolist() == value.tolist()
            ex.release(h)
        assert ex.cache_info()["prefetched_tensors"] == 0
    finally:
        srv.close()


def test_planned_offload_follows_the_planner(tmp_path):
    ex = OffloadExecutor(MemoryPolicy(scratch_path=str(tmp_path)))
    pl = MemoryPlanner(MemoryPolicy(tiers=(MemoryTier.VRAM, MemoryTier.NVME)),
                       budgets={MemoryTier.VRAM: 8, MemoryTier.NVME: 1 << 20})
    small = ex.offload_planned(tensor([1.0, 2.0]), pl)
    assert isinstance(small, Placement) and small.tier is MemoryTier.VRAM
    big = ex.offload_planned(tensor([1.0, 2.0, 3.0]), pl)
    assert big.tier is MemoryTier.NVME and ex.load_tensor(big).tolist() == [1.0, 2.0, 3.0]


def test_file_store_rejects_a_different_record(tmp_path):
    store = FileStore(tmp_path)
    h = store.put(tensor([1.0]))
    other = store.put(tensor([2.0]))
    # swap the files: the handle's digest catches it before decoding
    import shutil

    shutil.copyfile(other.path, h.path)
    with pytest.raises(ValueError, match="checksum mismatch"):
        store.get(h)


def test_unknown_route_is_not_found():
    srv = NetworkOffloadServer(port=0).start()
    try:
        cli = NetworkOffloadClient(srv.url)
        assert cli._call("GET", "/health")["status"] == "ok"
        with pytest.raises(RuntimeError, match="not found"):
            cli._call("GET", "/nothing-here")
    finally:
        srv.close()
