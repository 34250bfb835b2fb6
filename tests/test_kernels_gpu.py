"""Numerics of every sm_100a kernel against a plain PyTorch fp32 oracle."""

import math

import pytest
import torch

from tests import oracles as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def K():
    from underhfs_b200.ops import kernels

    torch.manual_seed(0)
    return kernels


def _status_ok():
    from underhfs_b200.ops._lib import core

    st = core().device_status(True)
    assert st["code"] == 0, st


def bf(x):
    return x.to(torch.bfloat16)


GEMM_SHAPES = [(128, 256, 64), (300, 264, 200), (1024, 768, 768), (2048, 2304, 768), (777, 1032, 1000)]


@pytest.mark.parametrize("M,N,K_", GEMM_SHAPES)
def test_gemm_forward_epilogues(K, M, N, K_):
    dev = "cuda"
    x = bf(torch.randn(M, K_, device=dev))
    w = bf(torch.randn(N, K_, device=dev) / math.sqrt(K_))
    b = bf(torch.randn(N, device=dev))
    ref = x.float() @ w.float().t()
    y = K.linear_fwd(x, w)
    assert O.rel_err(y, ref) < 2e-2
    y = K.linear_fwd(x, w, b)
    assert O.rel_err(y, ref + b.float()) < 2e-2
    r = bf(torch.randn(M, N, device=dev))
    y = K.linear_fwd_resid(x, w, b, r)
    assert O.rel_err(y, ref + b.float() + r.float()) < 2e-2
    u, g = K.linear_fwd_gelu(x, w, b)
    assert O.rel_err(u, ref + b.float()) < 2e-2
    assert O.rel_err(g, O.gelu_tanh(ref + b.float())) < 2e-2
    _status_ok()


@pytest.mark.parametrize("M,N,K_", GEMM_SHAPES)
def test_gemm_dgrad_wgrad(K, M, N, K_):
    dev = "cuda"
    dy = bf(torch.randn(M, N, device=dev))
    w = bf(torch.randn(N, K_, device=dev) / math.sqrt(N))
    x = bf(torch.randn(M, K_, device=dev))
    dx = K.linear_dgrad(dy, w)
    assert O.rel_err(dx, dy.float() @ w.float()) < 2e-2
    u = bf(torch.randn(M, K_, device=dev))
    dx2 = K.linear_dgrad(dy, w, gelu_in=u)
    gu = u.float().requires_grad_(True)
    gd = torch.autograd.grad(O.gelu_tanh(gu).sum(), gu)[0]
    assert O.rel_err(dx2, (dy.float() @ w.float()) * gd) < 3e-2
    dw = torch.zeros(N, K_, device=dev)
    K.linear_wgrad_accum(dy, x, dw)
    ref = dy.float().t() @ x.float()
    assert O.rel_err(dw, ref) < 1e-2
    K.linear_wgrad_accum(dy, x, dw)  # accumulates (stream-K)
    assert O.rel_err(dw, 2 * ref) < 1e-2
    K.linear_wgrad_accum(dy, x, dw, splits=3)  # classic split-K
    assert O.rel_err(dw, 3 * ref) < 1e-2
    _status_ok()


PAIR_SHAPES = [(296, 264, 200), (776, 1032, 1000), (2048, 2304, 768), (1536, 4096, 2048)]  # MN-major copies need M % 8 == 0


@pytest.mark.parametrize("M,N,K_", PAIR_SHAPES)
def test_gemm_cta_pair_layouts_and_epilogues(K, M, N, K_):
    """256 x 256 tiles on CTA pairs (tcgen05 cta_group::2): every operand
    layout and epilogue the pair kernel takes, ragged M / N / K edges."""
    dev = "cuda"

    def run(a, lda, a_mn, b, ldb, b_mn, epi, **kw):
        dt = torch.float32 if epi == K.EPI_F32_STORE else torch.bfloat16
        c = torch.empty(M, N, device=dev, dtype=dt)
        K.gemm_raw(M, N, K_, a, lda, a_mn, b, ldb, b_mn, c, N, epi, cta_pair=1, **kw)
        return c

    xa = bf(torch.randn(M, K_, device=dev))
    xb = bf(torch.randn(N, K_, device=dev) / math.sqrt(K_))
    at, bt = xa.t().contiguous(), xb.t().contiguous()  # MN-major copies
    ref = xa.float() @ xb.float().t()
    for a, lda, a_mn in ((xa, K_, False), (at, M, True)):
        for b, ldb, b_mn in ((xb, K_, False), (bt, N, True)):
            assert O.rel_err(run(a, lda, a_mn, b, ldb, b_mn, K.EPI_BF16), ref) < 2e-2, (a_mn, b_mn)
    assert O.rel_err(run(xa, K_, False, xb, K_, False, K.EPI_F32_STORE), ref) < 1e-2
    assert O.rel_err(run(at, M, True, bt, N, True, K.EPI_F32_STORE), ref) < 1e-2
    bias = bf(torch.randn(N, device=dev))
    pre = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
    g = run(xa, K_, False, xb, K_, False, K.EPI_BIAS_GELU, bias=bias, aux_out=pre, ld_aux_out=N)
    assert O.rel_err(pre, ref + bias.float()) < 2e-2
    assert O.rel_err(g, O.gelu_tanh(ref + bias.float())) < 2e-2
    r = bf(torch.randn(M, N, device=dev))
    y = run(xa, K_, False, xb, K_, False, K.EPI_RESID, bias=bias, aux=r, ld_aux=N)
    assert O.rel_err(y, ref + bias.float() + r.float()) < 2e-2
    y = run(xa, K_, False, bt, N, True, K.EPI_RESID, aux=r, ld_aux=N)
    assert O.rel_err(y, ref + r.float()) < 2e-2
    u = bf(torch.randn(M, N, device=dev))
    gu = u.float().requires_grad_(True)
    gd = torch.autograd.grad(O.gelu_tanh(gu).sum(), gu)[0]
    y = run(xa, K_, False, bt, N, True, K.EPI_DGELU, aux=u, ld_aux=N)
    assert O.rel_err(y, ref * gd) < 3e-2
    # fp32 accumulate (weight-gradient layout), stream-K and one pass per tile
    acc = torch.zeros(M, N, device=dev)
    K.gemm_raw(M, N, K_, at, M, True, bt, N, True, acc, N, K.EPI_F32_ACCUM, splits=0, cta_pair=1)
    assert O.rel_err(acc, ref) < 1e-2
    K.gemm_raw(M, N, K_, at, M, True, bt, N, True, acc, N, K.EPI_F32_ACCUM, splits=1, cta_pair=1)
    assert O.rel_err(acc, 2 * ref) < 1e-2
    K.gemm_raw(M, N, K_, xa, K_, False, bt, N, True, acc, N, K.EPI_F32_ACCUM, splits=0, cta_pair=1)
    assert O.rel_err(acc, 3 * ref) < 1e-2
    # the same problem on one SM per tile agrees with the pair kernel
    c1 = torch.empty(M, N, device=dev, dtype=torch.float32)
    K.gemm_raw(M, N, K_, xa, K_, False, xb, K_, False, c1, N, K.EPI_F32_STORE, cta_pair=0)
    c2 = run(xa, K_, False, xb, K_, False, K.EPI_F32_STORE)
    assert torch.allclose(c1, c2, rtol=1e-5, atol=1e-4)
    _status_ok()


def test_matmul_bf16_and_f32(K):
    a = torch.randn(130, 72, device="cuda")
    b = torch.randn(72, 200, device="cuda")
    assert O.rel_err(K.matmul_bf16(bf(a), bf(b)), a @ b) < 3e-2
    c = K.matmul_f32(a, b)
    assert torch.allclose(c, a @ b, atol=1e-4, rtol=1e-4)
    exact = K.matmul_f32(torch.tensor([[1.0, 2.0], [3.0, 4.0]], device="cuda"),
                         torch.tensor([[5.0, 6.0], [7.0, 8.0]], device="cuda"))
    assert exact.tolist() == [[19.0, 22.0], [43.0, 50.0]]


@pytest.mark.parametrize("M,N,Kd", [(1024, 1024, 1024), (700, 520, 333), (300, 2048, 4096), (512, 256, 16384)])
def test_matmul_f32_3xtf32(K, M, N, Kd):
    """Large fp32 products run as 3xTF32 on the tensor cores, accumulated in
    chunks folded into a round-to-nearest running sum: against an fp64 oracle
    they are as close as the exact SIMT kernel (about one fp32 ulp of the
    largest entry), at every K."""
    torch.manual_seed(0)
    a = torch.randn(M, Kd, device="cuda")
    b = torch.randn(Kd, N, device="cuda")
    ref = (a.double() @ b.double())
    c = K.matmul_f32(a, b)
    simt = torch.empty(M, N, device="cuda")
    K.core().gemm_f32(K.ptr(a), K.ptr(b), K.ptr(simt), M, N, Kd, False, K.stream())
    scale = ref.abs().max().item()
    err_tc = (c.double() - ref).abs().max().item() / scale
    err_simt = (simt.double() - ref).abs().max().item() / scale
    assert err_tc < 3e-6, (err_tc, err_simt)
    assert err_tc < 2 * err_simt + 5e-7, (err_tc, err_simt)
    _status_ok()


@pytest.mark.parametrize("rows,cols", [(16384, 768), (16384, 3072), (300, 264), (1000, 130), (7, 8)])
def test_bias_gradient_colsum(K, rows, cols):
    """out[c] += sum_r x[r, c] (fp32 accumulate) against the fp32 oracle,
    vectorised (cols % 8 == 0) and scalar paths, accumulating twice."""
    x = bf(torch.randn(rows, cols, device="cuda"))
    out = torch.zeros(cols, device="cuda")
    K.colsum_accum(x, out)
    ref = x.float().sum(0)
    assert torch.allclose(out, ref, rtol=1e-4, atol=1e-3 * rows ** 0.5)
    K.colsum_accum(x, out)
    assert torch.allclose(out, 2 * ref, rtol=1e-4, atol=2e-3 * rows ** 0.5)
    _status_ok()


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_elementwise_reduce_cast(K, dtype):
    n = (1 << 20) + 7
    a = torch.randn(n, device="cuda").to(dtype)
    b = torch.randn(n, device="cuda").to(dtype)
    for op, fn in ((K.OP_ADD, torch.add), (K.OP_MUL, torch.mul), (K.OP_SUB, torch.sub)):
        out = K.ew_binary(op, a, b)
        ref = fn(a.float(), b.float()).to(dtype)
        assert torch.equal(out, ref)
    s = K.reduce_sum(a)
    assert abs(s.item() - a.float().sum().item()) < 1e-3 * n ** 0.5
    c = K.cast(a, torch.float32)
    assert torch.equal(c, a.float())
    odd = a[1:]  # misaligned start exercises the scalar path
    assert torch.equal(K.ew_binary(K.OP_ADD, odd.contiguous(), odd.contiguous()), (odd.float() * 2).to(dtype))


@pytest.mark.parametrize("rows,cols", [(64, 768), (33, 200), (4096, 2048), (300, 1024), (1000, 512)])
def test_rmsnorm(K, rows, cols):
    x = bf(torch.randn(rows, cols, device="cuda"))
    w = bf(torch.rand(cols, device="cuda") + 0.5)
    y, rstd = K.rmsnorm(x, w, 1e-6)
    xf = x.float().requires_grad_(True)
    wf = w.float().requires_grad_(True)
    ref = O.rmsnorm(xf, wf, 1e-6)
    assert O.rel_err(y, ref) < 1e-2
    dy = bf(torch.randn(rows, cols, device="cuda"))
    dres = bf(torch.randn(rows, cols, device="cuda"))
    dw = torch.zeros(cols, device="cuda")
    dx = K.rmsnorm_backward(dy, x, w, rstd, dres, dw)
    gx, gw = torch.autograd.grad(ref, (xf, wf), dy.float())
    assert O.rel_err(dx, gx + dres.float()) < 2e-2
    assert O.rel_err(dw, gw) < 1e-2


def test_embedding(K):
    V, F, B, T = 1000, 256, 3, 17
    tok = bf(torch.randn(V, F, device="cuda"))
    pos = bf(torch.randn(32, F, device="cuda"))
    ids = torch.randint(0, V, (B, T), device="cuda")
    out = K.embedding(ids.reshape(-1), tok, pos, T)
    ref = tok.float()[ids] + pos.float()[:T]
    assert O.rel_err(out, ref.reshape(-1, F)) < 1e-2
    dout = bf(torch.randn(B * T, F, device="cuda"))
    dtok = torch.zeros(V, F, device="cuda")
    dpos = torch.zeros(32, F, device="cuda")
    K.embedding_backward(ids.reshape(-1), dout, dtok, dpos, T)
    rt = torch.zeros(V, F, device="cuda").index_add_(0, ids.reshape(-1), dout.float())
    rp = torch.zeros(32, F, device="cuda")
    rp[:T] = dout.float().view(B, T, F).sum(0)
    assert torch.allclose(dtok, rt, atol=1e-3)
    assert torch.allclose(dpos, rp, atol=1e-3)


@pytest.mark.parametrize("rows,cols", [(8, 32000), (5, 1003), (3, 50000), (64, 1024)])
def test_softmax_cross_entropy(K, rows, cols):
    logits = bf(torch.randn(rows, cols, device="cuda") * 3)
    tg = torch.randint(0, cols, (rows,), device="cuda")
    lf = logits.float().requires_grad_(True)
    ref = torch.nn.functional.cross_entropy(lf, tg, reduction="none")
    dl = torch.empty_like(logits)
    loss = K.softmax_cross_entropy(logits, tg, dl, 1.0 / rows)
    assert torch.allclose(loss, ref, atol=2e-3, rtol=1e-3)
    g = torch.autograd.grad(ref.mean(), lf)[0]
    assert O.rel_err(dl, g) < 2e-2
    scale = torch.tensor(2.0, device="cuda")
    K.softmax_cross_entropy(logits, tg, dl, 1.0 / rows, scale)
    assert O.rel_err(dl, 2 * g) < 2e-2
    # in place
    buf = logits.clone()
    K.softmax_cross_entropy(buf, tg, buf, 1.0 / rows)
    assert O.rel_err(buf, g) < 2e-2


@pytest.mark.parametrize("B,T,H,D,causal", [(2, 256, 2, 64, True), (1, 200, 3, 64, True), (2, 128, 2, 64, False),
                                            (1, 190, 2, 128, True), (2, 1024, 4, 64, True), (1, 300, 2, 64, False),
                                            (2, 640, 2, 128, True), (1, 333, 2, 128, False)])
def test_flash_attention(K, B, T, H, D, causal):
    F = H * D
    qkv = bf(torch.randn(B * T, 3 * F, device="cuda"))
    o, lse = K.flash_attn_qkv(qkv, B, T, H, D, causal)
    q, k, v = (qkv.float().view(B, T, 3, H, D)[:, :, i].clone().requires_grad_(True) for i in range(3))
    ref = O.attention(q, k, v, causal, 1.0 / math.sqrt(D))
    assert O.rel_err(o.view(B, T, H, D), ref) < 2e-2
    do = bf(torch.randn(B * T, F, device="cuda"))
    dqkv = K.flash_attn_qkv_backward(qkv, o, lse, do, B, T, H, D, causal)
    gq, gk, gv = torch.autograd.grad(ref, (q, k, v), do.float().view(B, T, H, D))
    d = dqkv.float().view(B, T, 3, H, D)
    assert O.rel_err(d[:, :, 0], gq) < 3e-2
    assert O.rel_err(d[:, :, 1], gk) < 3e-2
    assert O.rel_err(d[:, :, 2], gv) < 3e-2
    _status_ok()


def test_adamw_flat(K):
    n = 10007
    p = torch.randn(n, device="cuda")
    g = torch.randn(n, device="cuda")
    m = torch.zeros(n, device="cuda")
    v = torch.zeros(n, device="cuda")
    p16 = torch.empty(n, dtype=torch.bfloat16, device="cuda")
    rp, rm, rv = p.clone(), m.clone(), v.clone()
    lr, b1, b2, eps, wd = 1e-2, 0.9, 0.999, 1e-8, 0.1
    for step in (1, 2):
        K.adamw_(p, g, m, v, p16, lr=lr, beta1=b1, beta2=b2, eps=eps, weight_decay=wd, decoupled=False, step=step)
        gg = g + wd * rp
        rm = b1 * rm + (1 - b1) * gg
        rv = b2 * rv + (1 - b2) * gg * gg
        rp = rp - lr * (rm / (1 - b1 ** step)) / ((rv / (1 - b2 ** step)).sqrt() + eps)
    assert torch.allclose(p, rp, atol=1e-5, rtol=1e-5)
    assert torch.allclose(m, rm, atol=1e-6)
    assert torch.equal(p16, p.to(torch.bfloat16))


def test_reference_contract_kernels(K):
    from underhfs_b200.ops._lib import core

    c = core()
    assert c.cuda_add_f32([1.0, 2.0], [3.0, 4.0]) == [4.0, 6.0]
    r = c.cuda_fused_adamw_f32([1.0, 2.0], [0.1, 0.2], [0.0, 0.0], [0.0, 0.0], 0.01, 0.9, 0.999, 1e-8, 0.0, 1)
    assert abs(r["m"][0] - 0.01) < 1e-6 and abs(r["m"][1] - 0.02) < 1e-6
    a = c.cuda_attention_f32([1.0, 0.0, 0.0, 1.0], [1.0, 0.0, 0.0, 1.0], [1.0, 2.0, 3.0, 4.0], 2, 2, 1.0, False)
    assert len(a) == 4
    t = c.CudaTensorF32([1.0, 2.0, 3.0, 4.0], [2, 2])
    u = c.CudaTensorF32([5.0, 6.0, 7.0, 8.0], [2, 2])
    assert t.matmul(u).to_host() == [19.0, 22.0, 43.0, 50.0]
    assert t.sum().to_host() == [10.0]
    for ctor in (c.CudaTensorF16, c.CudaTensorBF16):
        x = ctor([1.0, 2.0], [2])
        y = ctor([3.0, 4.0], [2])
        assert x.add(y).to_host() == [4.0, 6.0]
        assert x.mul(y).to_host() == [3.0, 8.0]
    assert c.cudnn_conv2d_backward_input_f32([1.0], [2.0], 1, 1, 1, 1, 1, 1, 1, 1, 1, 0, 0) == [2.0]
    stats = c.cuda_stream_stats()
    assert stats["non_blocking_streams"] == 1 and stats["launches"] > 0
    assert c.cuda_allocator_stats()["allocated_bytes"] > 0


def test_out_of_range_ids_and_targets_are_reported_not_read(K):
    """Invalid token ids / targets never index outside a table: the kernels
    record kErrBounds (5) in the device status word and skip the row."""
    tok = bf(torch.randn(100, 64, device="cuda"))
    ids = torch.tensor([3, 100, -1, 7], device="cuda", dtype=torch.int64)
    out = K.embedding(ids, tok, None, 4)
    torch.cuda.synchronize()
    st = K.core().device_status(True)
    assert st["code"] == 5 and st["count"] >= 2, st
    assert torch.equal(out[0].float(), tok[3].float()) and not out[1].float().any()
    dtok = torch.zeros(100, 64, device="cuda")
    K.embedding_backward(ids, out, dtok, None, 4)
    torch.cuda.synchronize()
    assert K.core().device_status(True)["code"] == 5
    assert torch.equal(dtok[3], out[0].float())
    logits = bf(torch.randn(3, 1024, device="cuda"))
    tg = torch.tensor([5, 1024, -3], device="cuda", dtype=torch.int64)
    loss = K.softmax_cross_entropy(logits, tg, None, 1.0)
    torch.cuda.synchronize()
    assert K.core().device_status(True)["code"] == 5
    assert torch.isfinite(loss[0]) and torch.isnan(loss[1]) and torch.isnan(loss[2])
    _status_ok()


@pytest.mark.parametrize("N,C,H,W,K,R,S,stride,pad", [
    (2, 3, 17, 13, 5, 3, 3, (1, 1), (1, 1)),
    (3, 7, 20, 9, 11, 5, 3, (2, 1), (2, 0)),
    (1, 16, 15, 15, 130, 3, 3, (2, 2), (0, 1)),
    (2, 65, 8, 8, 70, 1, 1, (1, 1), (0, 0)),
])
def test_conv2d_implicit_gemm_matches_fp32_torch(N, C, H, W, K, R, S, stride, pad):
    """Forward, data gradient, weight and bias gradients of the implicit-GEMM
    conv kernels against torch's conv2d in fp32 (TF32 off) at ragged shapes,
    strides and paddings."""
    from underhfs_b200.ops import kernels as K_

    torch.backends.cudnn.allow_tf32 = False
    gen = torch.Generator(device="cuda").manual_seed(N * 1000 + C * 10 + K)
    x = torch.randn(N, C, H, W, device="cuda", generator=gen)
    w = torch.randn(K, C, R, S, device="cuda", generator=gen) * 0.2
    b = torch.randn(K, device="cuda", generator=gen)
    y = K_.conv2d_fwd(x, w, b, stride, pad)
    xr, wr, br = (t.clone().requires_grad_(True) for t in (x, w, b))
    yr = torch.nn.functional.conv2d(xr, wr, br, stride, pad)
    assert y.shape == yr.shape
    assert torch.allclose(y, yr, rtol=1e-4, atol=1e-4), (y - yr).abs().max()
    dy = torch.randn_like(yr)
    yr.backward(dy)
    dx, dw, db = K_.conv2d_bwd(dy, x, w, stride, pad, True)
    for got, want in ((dx, xr.grad), (dw, wr.grad), (db, br.grad)):
        err = ((got - want).abs().max() / want.abs().max()).item()
        assert err < 1e-5, err
    assert K_.core().device_status(True)["code"] == 0
