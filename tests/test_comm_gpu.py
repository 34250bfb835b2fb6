"""Single-GPU checks of the communication runtime.

With one rank the fused all-reduce / ZeRO kernels exercise their full code
path (barrier flags, epochs, peer-pointer table with one entry).  The
failure path is tested without a fault: a bounded wait on a flag that nothing
sets must return and record kErrPeerTimeout, leaving the context usable.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_world1_allreduce_scales_in_place():
    from underhfs_b200.ops._lib import core
    from underhfs_b200.parallel.symmetric import SymmetricBuffer

    sym = SymmetricBuffer(1 << 20, rank=0, world=1)
    t = sym.tensor(1000, torch.float32)
    t.copy_(torch.arange(1000, dtype=torch.float32, device="cuda"))
    off = t.data_ptr() - sym.heap.data_ptr(0)
    for _ in range(3):  # repeated launches advance the per-block epochs
        core().comm_allreduce_f32(sym.heap, off, 1000, 0.5, 8, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert torch.allclose(t, torch.arange(1000, dtype=torch.float32, device="cuda") / 8)
    assert core().device_status(True)["code"] == 0


def test_world1_rs_adamw_ag_matches_flat_adamw():
    from underhfs_b200.ops import kernels as K
    from underhfs_b200.ops._lib import core
    from underhfs_b200.parallel.symmetric import SymmetricBuffer

    n = 4096
    sym = SymmetricBuffer(n * 6 + 1024, rank=0, world=1)
    params = sym.tensor(n, torch.bfloat16)
    grads = sym.tensor(n, torch.float32)
    g = torch.randn(n, device="cuda")
    grads.copy_(g)
    master = torch.randn(n, device="cuda")
    m, v = torch.zeros(n, device="cuda"), torch.zeros(n, device="cuda")
    rp, rm, rv = master.clone(), m.clone(), v.clone()
    step = torch.ones((), dtype=torch.int32, device="cuda")
    base = sym.heap.data_ptr(0)
    core().comm_rs_adamw_ag(sym.heap, grads.data_ptr() - base, sym.heap, params.data_ptr() - base, 0, n,
                            master.data_ptr(), m.data_ptr(), v.data_ptr(), 1e-2, 0.9, 0.95, 1e-8, 0.1, 1.0, True,
                            step.data_ptr(), 16, torch.cuda.current_stream().cuda_stream)
    K.adamw_(rp, g, rm, rv, None, lr=1e-2, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1, decoupled=True,
             step=1)
    torch.cuda.synchronize()
    assert torch.allclose(master, rp, atol=1e-6)
    assert torch.equal(params, rp.to(torch.bfloat16))
    assert core().device_status(True)["code"] == 0


def test_bounded_wait_reports_timeout_without_hanging():
    from underhfs_b200.ops._lib import core
    from underhfs_b200.parallel.symmetric import SymmetricBuffer

    sym = SymmetricBuffer(4096, rank=0, world=1)
    core().device_status(True)
    core().comm_wait_probe(sym.heap, 7, 200_000_000, torch.cuda.current_stream().cuda_stream)  # 0.2 s bound
    torch.cuda.synchronize()
    st = core().device_status(True)
    assert st["code"] == 4 and st["where"] == 140, st  # kErrPeerTimeout from the probe
    x = torch.ones(4, device="cuda")  # context still healthy
    assert float((x + x).sum().item()) == 8.0


def test_pinned_host_tier_roundtrip():
    from underhfs_b200.runtime import PinnedHostTier

    tier = PinnedHostTier("cuda")
    src = torch.randn(1 << 16, device="cuda")
    tier.offload("x", src)
    out = torch.empty_like(src)
    tier.fetch("x", out)
    tier.wait("x")
    assert torch.equal(out, src)
    assert tier.bytes_resident() == src.numel() * 4
