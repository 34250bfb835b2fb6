"""ZeRO-3 row sharding: every parameter element is owned by exactly one rank,
shard offsets are dense, and every segment is a whole number of 16-byte
vectors (CPU only: the layout, not the kernels)."""

import pytest

from underhfs_b200.models.transformer import LMSpec, build_layout
from underhfs_b200.parallel.zero3 import Zero3LM


def _units(spec, rank, world):
    z = Zero3LM.__new__(Zero3LM)
    z.spec, z.rank, z.world = spec, rank, world
    z.layout = build_layout(spec)
    z.by_name = {s.name: s for s in z.layout.slots}
    z.units = {}
    z._build_units()
    return z


@pytest.mark.parametrize("tied", [True, False])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_segments_partition_every_parameter(tied, world):
    spec = LMSpec(1024, 256, 256, 1024, 3, heads=4, tied=tied)
    owned = {}
    for r in range(world):
        z = _units(spec, r, world)
        cursor = 0
        for key in ["embed"] + list(range(spec.layers)) + ["tail"]:
            u = z.units[key]
            assert len(u.segs) <= 16
            for slot, (nat, soff, ln) in zip(u.slots, u.segs):
                assert nat % 8 == 0 and soff % 8 == 0 and ln % 8 == 0
                assert soff == cursor
                cursor += ln
                start = slot.offset - u.lo
                assert start <= nat and nat + ln <= start + slot.numel
                for e in range(nat, nat + ln, max(1, ln // 4)):
                    owned.setdefault((key, e), []).append(r)
        assert cursor <= z.shard_total
    # every sampled element has exactly one owner, and the owners cover all ranks
    assert all(len(v) == 1 for v in owned.values())
    assert {v[0] for v in owned.values()} == set(range(world))


def test_rows_must_split_evenly():
    spec = LMSpec(1000, 256, 256, 1024, 1, heads=4, tied=True)  # 1000 rows / 16 ranks
    with pytest.raises(ValueError):
        _units(spec, 0, 16)


def test_zero3_engine_has_every_engine_hook():
    """Zero3Engine builds its own state instead of calling LMEngine.__init__;
    every optional hook the shared forward/backward reads must still exist."""
    from underhfs_b200.models.transformer import LMEngine
    from underhfs_b200.parallel.zero3 import Zero3Engine

    eng = Zero3Engine.__new__(Zero3Engine)
    for name in ("context_attention", "positions"):
        assert hasattr(eng, name) and getattr(eng, name) is None
    assert issubclass(Zero3Engine, LMEngine)


@pytest.mark.parametrize("tied", [True, False])
@pytest.mark.parametrize("world", [1, 2, 8])
def test_unit_shard_ranges_are_contiguous_for_moment_staging(tied, world):
    """Moment offload copies each unit's [shard_lo, shard_lo + shard_len) as
    one block: the unit ranges must tile the shard in order and contain every
    segment of the unit."""
    spec = LMSpec(1024, 256, 256, 1024, 3, heads=4, tied=tied)
    z = _units(spec, 0, world)
    cursor = 0
    for key in ["embed"] + list(range(spec.layers)) + ["tail"]:
        u = z.units[key]
        assert u.shard_lo == cursor
        for _nat, soff, ln in u.segs:
            assert u.shard_lo <= soff and soff + ln <= u.shard_lo + u.shard_len
        cursor += u.shard_len
    assert cursor <= z.shard_total
