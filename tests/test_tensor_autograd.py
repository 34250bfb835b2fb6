"""Tensor metadata, views, version counter, autograd, JVP and checkpoint contracts."""

from underhfs import tensor, zeros
from underhfs.autograd import checkpoint, checkpoint_sequential, jvp, no_grad


def test_shape_strides_version_and_add_():
    t = zeros((2, 3))
    assert (t.shape, t.strides, t.version) == ((2, 3), (3, 1), 0)
    t.add_(1)
    assert t.version == 1
    assert t.tolist() == [[1.0] * 3, [1.0] * 3]


def test_scalar_chain_rule():
    a = tensor(3.0, requires_grad=True)
    (a * a + a).backward()
    assert abs(a.grad.item() - 7.0) < 1e-12


def test_matmul_gradients():
    a = tensor([[1.0, 2.0]], requires_grad=True)
    b = tensor([[3.0], [4.0]], requires_grad=True)
    (a @ b).sum().backward()
    assert a.grad.tolist() == [[3.0, 4.0]]
    assert b.grad.tolist() == [[1.0], [2.0]]


def test_views_share_storage_and_version():
    base = tensor([[1.0, 2.0], [3.0, 4.0]])
    flat = base.view(4)
    assert flat.shape == (4,) and flat.strides == (1,)
    flat.add_(1.0)
    assert base.tolist() == [[2.0, 3.0], [4.0, 5.0]]
    assert base.version == flat.version == 1
    assert base.flatten().tolist() == [2.0, 3.0, 4.0, 5.0]


def test_slice_view_strides_and_scatter_backward():
    m = tensor([[1.0, 2.0, 3.0], [4.0, 5.0, 6.0]], requires_grad=True)
    s = m[:, 1:]
    assert s.shape == (2, 2) and s.strides == (3, 1)
    assert s.tolist() == [[2.0, 3.0], [5.0, 6.0]]
    s.sum().backward()
    assert m.grad.tolist() == [[0.0, 1.0, 1.0], [0.0, 1.0, 1.0]]


def test_strided_view_needs_reshape():
    m = tensor([[1.0, 2.0, 3.0], [4.0, 5.0, 6.0]])
    odd = m[:, ::2]
    try:
        odd.view(4)
    except ValueError as exc:
        assert "contiguous" in str(exc)
    else:
        raise AssertionError("view of a strided tensor must fail")
    assert odd.reshape(4).tolist() == [1.0, 3.0, 4.0, 6.0]


def test_jvp_matmul_sum():
    primal, tangent = jvp(lambda a, b: (a @ b).sum(), (tensor([[1.0, 2.0]]), tensor([[3.0], [4.0]])),
                          (tensor([[1.0, 1.0]]), tensor([[0.5], [0.5]])))
    assert primal.item() == 11.0
    assert tangent.item() == 8.5


def test_jvp_softmax_tangent_sums_to_zero():
    x = tensor([[1.0, 2.0], [3.0, 4.0]])
    dx = tensor([[0.1, 0.2], [0.3, 0.4]])
    primal, tangent = jvp(lambda v: v[:, :].reshape(4).softmax(), (x,), (dx,))
    assert primal.shape == tangent.shape == (4,)
    assert abs(sum(tangent.tolist())) < 1e-9


def test_checkpoint_tag_and_recompute_gradient():
    a = tensor(3.0, requires_grad=True)
    out = checkpoint(lambda v: v * v, a)
    assert out._underhfs_checkpoint["mode"] == "eager-recompute-contract"
    out.backward()
    assert a.grad.item() == 6.0


def test_checkpoint_sequential_chunks():
    a = tensor(2.0, requires_grad=True)
    out = checkpoint_sequential([lambda v: v * v, lambda v: v + v], 2, a)
    assert out._underhfs_checkpoint["mode"] == "eager-recompute-contract"
    out.backward()
    assert a.grad.item() == 8.0


def test_no_grad_is_honoured():
    a = tensor(2.0, requires_grad=True)
    with no_grad():
        b = a * a
    assert not b.requires_grad
