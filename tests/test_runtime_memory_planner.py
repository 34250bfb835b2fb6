"""Memory tiers, NVMe / network offload integrity, device parsing."""

from underhfs import tensor
from underhfs.cuda import MemoryPolicy, MemoryTier, _parse_nvidia_smi_devices
from underhfs.runtime import (
    MemoryPlanner,
    NetworkOffloadClient,
    NetworkOffloadServer,
    OffloadExecutor,
    planner_from_system,
)
from underhfs.tensor import DType


def test_first_fit_across_tiers():
    pl = MemoryPlanner(MemoryPolicy(tiers=(MemoryTier.VRAM, MemoryTier.RAM)),
                       budgets={MemoryTier.VRAM: 8, MemoryTier.RAM: 64})
    assert pl.place_tensor(tensor([1.0, 2.0], dtype=DType.FP32)).tier is MemoryTier.VRAM
    assert pl.place_tensor(tensor([1.0, 2.0, 3.0], dtype=DType.FP32)).tier is MemoryTier.RAM
    assert pl.snapshot()["vram"]["used_bytes"] == 8


def test_oversubscription_goes_to_last_tier():
    pl = MemoryPlanner(MemoryPolicy(tiers=(MemoryTier.VRAM, MemoryTier.NVME), allow_offload=True),
                       budgets={MemoryTier.VRAM: 0, MemoryTier.NVME: 1})
    p = pl.place_tensor(tensor([1.0], dtype=DType.FP32))
    assert p.tier is MemoryTier.NVME and p.reason == "oversubscribed-offload"


def test_no_offload_raises_memory_error():
    pl = MemoryPlanner(MemoryPolicy(tiers=(MemoryTier.VRAM,), allow_offload=False), budgets={MemoryTier.VRAM: 2})
    try:
        pl.place_bytes(16)
    except MemoryError:
        pass
    else:
        raise AssertionError("placement beyond every tier must fail without offload")


def test_nvidia_smi_line_parser():
    (dev,) = _parse_nvidia_smi_devices("0, NVIDIA B200, 183359, 180000, 580.159\n")
    assert dev.index == 0 and dev.name == "NVIDIA B200"
    assert dev.memory_total_bytes == 183359 * 1024 * 1024
    assert dev.memory_free_bytes == 180000 * 1024 * 1024
    assert dev.driver_version == "580.159"


def test_planner_from_system_has_configured_tiers():
    snap = planner_from_system(MemoryPolicy(tiers=(MemoryTier.VRAM, MemoryTier.RAM))).snapshot()
    assert set(snap) == {"vram", "ram"}


def test_nvme_offload_roundtrip_and_prefetch(tmp_path=None):
    ex = OffloadExecutor(MemoryPolicy(scratch_path=str(tmp_path or ".underhfs-offload-test")))
    h = ex.offload_tensor(tensor([[1.0, 2.0]]), MemoryTier.NVME)
    assert h.sha256 and h.tier is MemoryTier.NVME
    assert ex.load_tensor(h).tolist() == [[1.0, 2.0]]
    cached = ex.prefetch_tensor(h)
    assert cached.cached and ex.cache_info()["prefetched_tensors"] == 1
    assert ex.load_tensor(cached).tolist() == [[1.0, 2.0]]
    ex.release(h)
    assert ex.cache_info()["prefetched_tensors"] == 0


def test_nvme_offload_detects_corruption(tmp_path=None):
    ex = OffloadExecutor(MemoryPolicy(scratch_path=str(tmp_path or ".underhfs-offload-corrupt")))
    h = ex.offload_tensor(tensor([1.0, 2.0]), MemoryTier.NVME)
    with open(h.path, "ab") as fh:
        fh.write(b"junk")
    try:
        ex.load_tensor(h)
    except ValueError as exc:
        assert "checksum mismatch" in str(exc)
    else:
        raise AssertionError("appended bytes must fail the digest")
    finally:
        ex.release(h)


def test_network_offload_roundtrip_and_release():
    srv = NetworkOffloadServer(port=0).start()
    try:
        cli = NetworkOffloadClient(srv.url)
        h = cli.offload_tensor(tensor([[1.0, 2.0]]))
        assert h.tier is MemoryTier.NETWORK
        assert cli.load_tensor(h).tolist() == [[1.0, 2.0]]
        cli.release(h)
        try:
            cli.load_tensor(h)
        except Exception as exc:  # noqa: BLE001
            assert "not found" in str(exc).lower() or "404" in str(exc)
        else:
            raise AssertionError("released tensor must not load")
    finally:
        srv.close()


def test_network_offload_detects_tampering():
    srv = NetworkOffloadServer(port=0).start()
    try:
        cli = NetworkOffloadClient(srv.url)
        h = cli.offload_tensor(tensor([1.0, 2.0]))
        srv._store[h.id]["data"] = [9.0, 9.0]
        try:
            cli.load_tensor(h)
        except ValueError as exc:
            assert "checksum mismatch" in str(exc)
        else:
            raise AssertionError("tampered payload must fail")
    finally:
        srv.close()
