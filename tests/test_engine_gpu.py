"""The TransformerLM engine (all native kernels) against an fp32 PyTorch oracle."""

import pytest
import torch

from tests import oracles as O

pytestmark = pytest.mark.gpu


def _build(spec, seed=0):
    from underhfs_b200.models.transformer import LMEngine, build_layout, initial_value
    from underhfs_b200.parallel.flat import FlatBuffers

    flat = FlatBuffers(build_layout(spec), torch.device("cuda"))
    gen = torch.Generator().manual_seed(seed)
    for slot in flat.layout.slots:
        flat.load_from(slot.name, initial_value(spec, slot.name, slot.shape, "normal", gen) * 2.0)
    return flat, LMEngine(spec, flat)


@pytest.mark.parametrize("tied,heads", [(True, 2), (False, 1)])
def test_engine_matches_fp32_oracle(tied, heads):
    from underhfs_b200.models.transformer import LMSpec

    D = 64
    spec = LMSpec(vocab_size=512, max_seq_len=160, features=heads * D, hidden_features=4 * heads * D, layers=2,
                  heads=heads, tied=tied, eps=1e-6)
    flat, eng = _build(spec)
    B, T = 3, 144
    ids = torch.randint(0, spec.vocab_size, (B, T), device="cuda")
    tg = torch.randint(0, spec.vocab_size, (B, T), device="cuda")
    loss, _ = eng.forward(ids, tg, fuse_loss_grad=True)
    eng.backward()
    params = {s.name: flat.param(s.name).float().clone().requires_grad_(True) for s in flat.layout.slots}
    ref = O.lm_loss(params, ids, tg, spec)
    ref.backward()
    assert abs(loss.item() - ref.item()) < 2e-2 * max(1.0, abs(ref.item()))
    for s in flat.layout.slots:
        g = flat.grad(s.name)
        r = params[s.name].grad
        if s.name.endswith("k_proj.bias"):
            # softmax is invariant to a per-query constant: dL/db_k is exactly 0
            assert g.abs().max().item() < 1e-3, (s.name, g.abs().max().item())
            continue
        err = O.rel_err(g, r)
        assert err < 8e-2, (s.name, err)


def test_engine_loss_grad_paths_agree():
    from underhfs_b200.models.transformer import LMSpec

    spec = LMSpec(vocab_size=256, max_seq_len=64, features=128, hidden_features=256, layers=1, heads=2, tied=True)
    flat, eng = _build(spec, seed=1)
    ids = torch.randint(0, 256, (2, 64), device="cuda")
    tg = torch.randint(0, 256, (2, 64), device="cuda")
    eng.forward(ids, tg, fuse_loss_grad=True)
    eng.backward()
    g1 = flat.grads.clone()
    flat.zero_grad()
    eng.forward(ids, tg, fuse_loss_grad=False, keep_logits=True)
    eng.backward(loss_grad=torch.tensor(1.0, device="cuda"))
    assert O.rel_err(flat.grads, g1) < 2e-2
