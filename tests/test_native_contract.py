"""Native core contract: probe values, backend tags, allocator / stream stats."""

from underhfs.cuda import allocator_stats, empty_cache, stream_stats, synchronize
from underhfs.native import probe, status
from underhfs.nn import Conv2d
from underhfs.tensor import DType, tensor


def test_probe_values():
    st = status()
    if not st.available:
        assert st.reason
        return
    r = probe()
    assert isinstance(r["cuda_enabled"], bool) and isinstance(r["nccl_enabled"], bool)
    assert r["add"] == [6.0, 8.0, 10.0, 12.0]
    assert r["matmul"] == [19.0, 22.0, 43.0, 50.0]
    assert r["sum"] == [134.0]
    if r["cuda_enabled"]:
        assert r["cuda_add_f32"] == [4.0, 6.0]
        assert r["cuda_tensor_add_f32"] == [4.0, 6.0]
        assert r["cuda_tensor_mul_f32"] == [3.0, 8.0]
        assert r["cuda_tensor_sum_f32"] == [3.0]
        assert r["cuda_tensor_matmul_f32"] == [19.0, 22.0, 43.0, 50.0]
        assert abs(r["cuda_fused_adamw_f32"]["m"][0] - 0.01) < 1e-6
        assert abs(r["cuda_fused_adamw_f32"]["m"][1] - 0.02) < 1e-6
        assert len(r["cuda_attention_f32"]) == 4
        for key in ("cuda_tensor_add_f16", "cuda_tensor_add_bf16"):
            assert r[key] == [4.0, 6.0]
        for key in ("cuda_tensor_mul_f16", "cuda_tensor_mul_bf16"):
            assert r[key] == [3.0, 8.0]
        assert r["cuda_allocator"]["allocated_bytes"] > 0
        assert r["cuda_stream"]["non_blocking_streams"] == 1
        assert r["cuda_stream"]["launches"] > 0


def test_cpu_fast_path_tags():
    if not status().available:
        return
    a = tensor([[1.0, 2.0], [3.0, 4.0]], requires_grad=True)
    b = tensor([[5.0, 6.0], [7.0, 8.0]], requires_grad=True)
    prod = a @ b
    total = prod.sum()
    assert {(a + b).backend, (a * b).backend, prod.backend, total.backend} == {"native_cpu"}
    assert prod.tolist() == [[19.0, 22.0], [43.0, 50.0]]
    total.backward()
    assert a.grad is not None and b.grad is not None


def test_cuda_elementwise_matmul_sum_tags():
    if not status().cuda_enabled:
        return
    s = tensor([1.0, 2.0]).cuda() + tensor([3.0, 4.0]).cuda()
    assert s.backend == "native_cuda" and str(s.device) == "cuda:0" and s.tolist() == [4.0, 6.0]
    p = tensor([1.0, 2.0, 3.0]).cuda() * tensor([4.0, 5.0, 6.0]).cuda()
    total = p.sum()
    assert p.backend == total.backend == "native_cuda"
    assert p.tolist() == [4.0, 10.0, 18.0] and total.tolist() == 32.0
    for dt in (DType.FP16, DType.BF16):
        x, y = tensor([1.0, 2.0], dtype=dt).cuda(), tensor([3.0, 4.0], dtype=dt).cuda()
        assert (x + y).dtype is dt and (x + y).tolist() == [4.0, 6.0] and (x * y).tolist() == [3.0, 8.0]
    m = tensor([[1.0, 2.0], [3.0, 4.0]]).cuda() @ tensor([[5.0, 6.0], [7.0, 8.0]]).cuda()
    assert m.backend == "native_cuda" and m.tolist() == [[19.0, 22.0], [43.0, 50.0]]
    r = tensor([[1.0, 2.0, 3.0], [4.0, 5.0, 6.0]]).cuda() @ tensor([[7.0, 8.0], [9.0, 10.0], [11.0, 12.0]]).cuda()
    assert r.tolist() == [[58.0, 64.0], [139.0, 154.0]]


def test_cuda_autograd_through_native_kernels():
    if not status().cuda_enabled:
        return
    a = tensor([[1.0, 2.0]], requires_grad=True).cuda()
    b = tensor([[3.0], [4.0]], requires_grad=True).cuda()
    (a @ b).sum().backward()
    assert a.grad.tolist() == [[3.0, 4.0]] and b.grad.tolist() == [[1.0], [2.0]]


def test_allocator_and_stream_stats():
    if not status().cuda_enabled:
        for fn in (allocator_stats, stream_stats):
            try:
                fn()
            except RuntimeError:
                pass
            else:
                raise AssertionError("stats need a CUDA device")
        return
    probe()
    st = allocator_stats()
    assert set(st) == {"active_bytes", "cached_bytes", "allocated_bytes", "allocations", "reuses"}
    empty_cache()
    assert allocator_stats()["cached_bytes"] == 0
    ss = stream_stats()
    assert ss["non_blocking_streams"] == 1 and ss["launches"] > 0
    synchronize()


def test_cuda_conv2d_runs_native_kernels():
    if not status().cuda_enabled:
        return
    conv = Conv2d(2, 3, kernel_size=3, padding=1)
    conv.to("cuda")
    x = tensor([[[[float(i + j + c) for j in range(5)] for i in range(5)] for c in range(2)]], requires_grad=True)
    y = conv(x.cuda())
    assert y.backend == "native_cudnn" and y.shape == (1, 3, 5, 5)
    ref = Conv2d(2, 3, kernel_size=3, padding=1)(x)
    assert max(abs(a - b) for a, b in zip(y.cpu()._storage, ref._storage)) < 1e-4
