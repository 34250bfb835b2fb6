"""CUDA paths of the public API on a real device (native kernels, no fallback)."""

import pytest
import torch

from tests import test_native_contract as NC
from tests import test_nn_optim as NO
from tests import test_runtime_surface as RS

pytestmark = pytest.mark.gpu


def _cuda():
    from underhfs.native import status

    st = status()
    assert st.cuda_enabled, st
    return st


def test_probe_on_gpu():
    _cuda()
    NC.test_probe_values()


def test_cuda_tags_and_autograd():
    _cuda()
    NC.test_cuda_elementwise_matmul_sum_tags()
    NC.test_cuda_autograd_through_native_kernels()
    NC.test_allocator_and_stream_stats()
    NC.test_cuda_conv2d_runs_native_kernels()


def test_cuda_optimizer_and_conv_contracts():
    _cuda()
    NO.test_fused_adamw_native_status_on_cuda()
    NO.test_conv2d_backend_status_contract()
    NO.test_adamw_moments_keep_cuda_dtype()


def test_compile_native_dispatch():
    _cuda()
    RS.test_native_attention_dispatch_on_gpu()
    RS.test_native_fused_dispatch_on_gpu()
    RS.test_to_cpu_dtype_and_cuda_contract()


def test_bf16_modules_on_cuda():
    _cuda()
    from underhfs import tensor
    from underhfs.nn import CausalSelfAttention, Linear, RMSNorm

    lin = Linear(64, 32)
    lin.to("cuda", dtype="bf16")
    x = tensor([[float(i % 7) / 7 for i in range(64)]] * 3, requires_grad=True).to("cuda", dtype="bf16")
    y = lin(x)
    assert y.backend == "native_cuda" and y.shape == (3, 32)
    y.sum().backward()
    assert lin.weight.grad is not None and x.grad is not None
    attn = CausalSelfAttention(128, heads=2)
    attn.to("cuda", dtype="bf16")
    z = attn(tensor([[[0.01 * ((i * 7 + j) % 11) for j in range(128)] for i in range(16)]]).to("cuda", dtype="bf16"))
    assert z.backend == "native_cuda_attention" and z.shape == (1, 16, 128)
    norm = RMSNorm(128)
    norm.to("cuda", dtype="bf16")
    assert norm(z).backend == "native_cuda"


def _engine_model(tied=True, seed=0):
    from underhfs.nn import TransformerLM

    m = TransformerLM(vocab_size=1024, max_seq_len=256, features=256, hidden_features=1024, layers=2, heads=4,
                      tied=tied, init="normal", seed=seed)
    m.to("cuda", dtype="bf16")
    return m


def test_engine_model_trains_and_state_dict_roundtrips(tmp_path):
    _cuda()
    from underhfs.optim import FusedAdamW
    from underhfs.serialization import load_training_state, save_training_state

    m = _engine_model()
    assert m.engine is not None
    opt = FusedAdamW(m.parameters(), lr=2e-3, weight_decay=0.0, decoupled=True)
    assert opt.last_kernel_status.backend if hasattr(opt, "last_kernel_status") else True
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(0, 1024, (4, 256), generator=g).cuda()
    tg = torch.roll(ids, -1, 1)
    losses = []
    for _ in range(15):
        m.zero_grad()
        loss = m(ids, tg)
        loss.backward()
        opt.step()
        losses.append(loss.item())
    assert opt.last_kernel_status.backend == "cuda-native"
    assert losses[-1] < losses[0] - 0.5, losses
    save_training_state(tmp_path / "ck", model=m, optimizer=opt, step=15)
    m2 = _engine_model(seed=7)
    opt2 = FusedAdamW(m2.parameters(), lr=2e-3, weight_decay=0.0, decoupled=True)
    meta = load_training_state(tmp_path / "ck", model=m2, optimizer=opt2)
    assert meta["step"] == 15
    with torch.no_grad():
        l1 = m(ids, tg).item()
        l2 = m2(ids, tg).item()
    assert abs(l1 - l2) < 1e-3


def test_engine_logits_path_matches_fused_loss_path():
    _cuda()
    from underhfs.functional import cross_entropy

    m = _engine_model(tied=False)
    g = torch.Generator().manual_seed(1)
    ids = torch.randint(0, 1024, (2, 128), generator=g).cuda()
    tg = torch.randint(0, 1024, (2, 128), generator=g).cuda()
    m.zero_grad()
    m(ids, tg).backward()
    g1 = m.flat.grads.clone()
    m.zero_grad()
    from underhfs import Tensor

    logits = m(ids)
    assert logits.shape == (2, 128, 1024)
    loss = cross_entropy(logits.reshape(-1, 1024), Tensor._wrap(tg.reshape(-1)))
    loss.backward()
    err = ((m.flat.grads - g1).abs().max() / g1.abs().max()).item()
    assert err < 3e-2, err


def test_trainer_cuda_graph_matches_eager():
    _cuda()
    from underhfs_b200.train import TrainConfig, Trainer, build_model
    from underhfs_b200.train import PRESETS
    from underhfs_b200.models.transformer import LMSpec

    PRESETS["test"] = LMSpec(2048, 256, 256, 1024, 2, heads=4, tied=True)
    ids = torch.randint(0, 2048, (4, 256), generator=torch.Generator().manual_seed(3)).cuda()
    tg = torch.roll(ids, -1, 1)
    out = {}
    for graph in (False, True):
        cfg = TrainConfig(model="test", batch=4, seq_len=256, lr=1e-3, cuda_graph=graph, seed=5)
        tr = Trainer(build_model(cfg), cfg)
        out[graph] = [float(tr.step(ids, tg).item()) for _ in range(6)]
        tr.release()
    for a, b in zip(out[False], out[True]):
        assert abs(a - b) < 2e-2 * max(1.0, abs(a)), out
    assert out[True][-1] < out[True][0]


def test_livesee_gpu_raster_matches_cpu_oracle():
    _cuda()
    import importlib.util
    import sys
    from pathlib import Path

    import numpy as np

    root = Path(__file__).resolve().parents[1] / "project" / "liveSee"
    sys.path.insert(0, str(root))
    sys.path.insert(0, str(root.parent))
    mods = {}
    for name in ("raster", "play_live_world"):
        spec = importlib.util.spec_from_file_location(name, root / f"{name}.py")
        mods[name] = importlib.util.module_from_spec(spec)
        sys.modules[name] = mods[name]
        spec.loader.exec_module(mods[name])
    chunk = mods["play_live_world"].LiveWorldSession(steps=1).state()
    gpu = mods["raster"].render_frame(chunk, 480, 270)
    cpu = mods["raster"].render_frame_cpu(chunk, 480, 270)
    diff = np.zeros(gpu.shape, dtype=np.int64)
    for s in (0, 8, 16):
        diff = np.maximum(diff, np.abs(((gpu >> s) & 255).astype(np.int64) - ((cpu >> s) & 255).astype(np.int64)))
    assert (diff == 0).mean() > 0.995 and diff.max() <= 1 or (diff == 0).mean() > 0.999
