"""nn / optimizer semantics (version bumps, state dicts, validation, kernel status)."""

from underhfs import DType, tensor
from underhfs.native import status
from underhfs.nn import Conv2d, Linear, ReLU, Sequential, TransformerLM
from underhfs.optim import SGD, AdamW, FusedAdamW, fused_adamw_kernel_status


def test_sgd_step_bumps_versions():
    net = Sequential(Linear(2, 3), ReLU(), Linear(3, 1))
    opt = SGD(net.parameters(), lr=0.01)
    v0 = [p.version for p in net.parameters()]
    net(tensor([[1.0, -1.0]], requires_grad=True)).sum().backward()
    opt.step()
    assert any(b > a for a, b in zip(v0, [p.version for p in net.parameters()]))


def test_module_state_dict_roundtrip():
    src, dst = Linear(2, 1), Linear(2, 1)
    dst.load_state_dict(src.state_dict())
    assert dst.state_dict() == src.state_dict()


def test_adamw_state_roundtrip_and_beta_validation():
    lin = Linear(2, 1)
    opt = AdamW(lin.parameters(), lr=0.01, weight_decay=0.0)
    lin(tensor([[1.0, 2.0]])).sum().backward()
    opt.step()
    snap = opt.state_dict()
    other = AdamW(lin.parameters(), lr=0.001)
    other.load_state_dict(snap)
    assert other.state_dict() == snap
    try:
        AdamW(lin.parameters(), betas=(1.0, 0.9))
    except ValueError as exc:
        assert "betas" in str(exc)
    else:
        raise AssertionError("beta1 == 1 must be rejected")


def test_adamw_l2_coupled_first_step_matches_formula():
    lin = Linear(1, 1, bias=False)
    w0 = lin.weight.tolist()[0][0]
    opt = AdamW(lin.parameters(), lr=0.1, weight_decay=0.5)
    lin(tensor([[2.0]])).sum().backward()
    opt.step()
    g = 2.0 + 0.5 * w0  # reference semantics: weight decay added to the gradient
    m_hat, v_hat = g, g * g
    expect = w0 - 0.1 * m_hat / (v_hat ** 0.5 + 1e-8)
    assert abs(lin.weight.tolist()[0][0] - expect) < 1e-9


def test_fused_adamw_updates_and_reports_status():
    lin = Linear(2, 1)
    opt = FusedAdamW(lin.parameters(), lr=0.01, weight_decay=0.0)
    w = lin.weight.tolist()
    lin(tensor([[1.0, 2.0]])).sum().backward()
    opt.step()
    assert lin.weight.tolist() != w
    assert opt.last_kernel_status.available
    assert fused_adamw_kernel_status(lin.parameters()).backend == "python"


def test_fused_adamw_native_status_on_cuda():
    if not status().cuda_enabled:
        return
    p = tensor([1.0, 2.0], requires_grad=True).cuda()
    rep = fused_adamw_kernel_status([p])
    assert rep.available and rep.backend == "cuda-native"


def test_conv2d_backend_status_contract():
    conv = Conv2d(1, 1, 1)
    assert conv.backend_status().available
    if status().cuda_enabled:
        assert conv.backend_status(tensor([[[[1.0]]]]).cuda()).backend == "cudnn"


def test_adamw_moments_keep_cuda_dtype():
    if not status().cuda_enabled:
        return
    p = tensor([1.0, 2.0], dtype=DType.FP16, requires_grad=True).cuda()
    (p * p).sum().backward()
    opt = AdamW([p], lr=0.01, weight_decay=0.0)
    opt.step()
    assert opt.m[0].dtype is DType.FP16
    assert str(opt.m[0].device) == "cuda:0"
    assert p.backend == "native_cuda"


def test_rmsnorm_propagates_gradient_unless_reference_compat():
    from underhfs.nn import RMSNorm

    x = tensor([[1.0, 2.0, 3.0]], requires_grad=True)
    (RMSNorm(3)(x) * tensor([[1.0, 0.0, 0.0]])).sum().backward()
    assert x.grad is not None and any(abs(v) > 0 for v in x.grad.tolist()[0])
    y = tensor([[1.0, 2.0, 3.0]], requires_grad=True)
    RMSNorm(3, compat="reference")(y).sum().backward()
    assert y.grad is None


def test_transformer_lm_batched_multihead_shapes():
    lm = TransformerLM(vocab_size=16, max_seq_len=8, features=8, hidden_features=16, layers=1, heads=2)
    logits = lm(tensor([[1, 2, 3], [4, 5, 6]]))
    assert logits.shape == (2, 3, 16)
    loss = lm(tensor([[1, 2, 3], [4, 5, 6]]), tensor([[2, 3, 4], [5, 6, 7]]))
    loss.backward()
    assert all(p.grad is not None for p in lm.parameters())


def test_step_split_without_flat_buffer_is_one_step():
    """AdamW.step_split on ordinary (non-flat) parameters waits, then takes one
    normal step: same parameters and step count as step()."""
    import torch

    from underhfs_b200.nn import Linear
    from underhfs_b200.optim import AdamW
    from underhfs_b200.tensor import tensor

    torch.manual_seed(0)
    a, b = Linear(4, 3), Linear(4, 3)
    for pa, pb in zip(a.parameters(), b.parameters()):
        pb._data.data.copy_(pa._data)
    oa = AdamW(a.parameters(), lr=1e-2, weight_decay=0.1)
    ob = AdamW(b.parameters(), lr=1e-2, weight_decay=0.1)
    x = tensor([[1.0, -2.0, 0.5, 3.0]])
    waited = []
    for _ in range(3):
        for m, o in ((a, oa), (b, ob)):
            o.zero_grad()
            m(x).sum().backward()
        oa.step()
        ob.step_split(2, lambda: waited.append(1))
    assert len(waited) == 3 and oa.step_count == ob.step_count == 3
    for (na, pa), (nb, pb) in zip(a.named_parameters(), b.named_parameters()):
        assert na == nb and torch.equal(pa._data, pb._data)
