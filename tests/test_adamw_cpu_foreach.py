"""The CPU AdamW update runs as one multi-tensor (foreach) pass.  It must give
bit-identical results to the per-tensor arithmetic it replaced, for fp64
parameter storage (the CPU default) and fp32 storage next to the fp64 CPU
moments (the mixed case), with decoupled and L2-coupled decay."""

import pytest
import torch

from underhfs_b200.optim import AdamW
from underhfs_b200.tensor import Tensor


def _per_tensor_reference(params, grads, steps, lr, betas, eps, wd, decoupled, moment_dtype):
    """The single-tensor update, element by element in the same order."""
    b1, b2 = betas
    ps = [p.clone() for p in params]
    ms = [torch.zeros(p.shape, dtype=moment_dtype) for p in params]
    vs = [torch.zeros(p.shape, dtype=moment_dtype) for p in params]
    for t in range(1, steps + 1):
        for pd, g, m, v in zip(ps, grads[t - 1], ms, vs):
            gd = g.to(pd.dtype)
            if decoupled:
                pd.mul_(1.0 - lr * wd)
            else:
                gd = gd + wd * pd
            m.mul_(b1).add_(gd, alpha=1 - b1)
            v.mul_(b2).addcmul_(gd, gd, value=1 - b2)
            mh = m / (1 - b1 ** t)
            vh = v / (1 - b2 ** t)
            pd.add_(mh / (vh.sqrt() + eps), alpha=-lr)
    return ps


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
@pytest.mark.parametrize("decoupled", [True, False])
def test_foreach_cpu_adamw_is_bitwise_per_tensor(dtype, decoupled):
    gen = torch.Generator().manual_seed(7)
    shapes = [(5, 3), (17,), (2, 4, 6)]
    init = [torch.randn(s, generator=gen, dtype=torch.float64).to(dtype) for s in shapes]
    steps = 4
    grads = [[torch.randn(s, generator=gen, dtype=torch.float64).to(dtype) for s in shapes] for _ in range(steps)]
    kw = dict(lr=3e-2, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1, decoupled=decoupled)

    params = [Tensor(p.clone(), requires_grad=True) for p in init]
    for p, x in zip(params, init):
        p._data = x.clone().requires_grad_(True)  # storage of exactly `dtype`
    opt = AdamW(params, **kw)
    moment_dtype = opt._m32[0].dtype
    for t in range(steps):
        for p, g in zip(params, grads[t]):
            p.grad = Tensor(g.clone())
        opt.step()

    ref = _per_tensor_reference(init, grads, steps, kw["lr"], kw["betas"], kw["eps"], kw["weight_decay"], decoupled,
                                moment_dtype)
    for p, r in zip(params, ref):
        assert p._data.dtype == r.dtype
        assert torch.equal(p._data, r)
