"""The allocation-free flash-attention backward entry point.

``uhfs_flash_attn_bwd_noalloc`` is for callers that cannot allocate device
memory themselves (C or other-language callers without a CUDA allocator,
fixed-budget deployments that forbid allocation after set-up, code running
where cudaMalloc is not allowed).  It keeps its scratch in a static device
array of the native library.  This test calls it through its exported C
symbol (ctypes), twice in a row, and compares each result with the regular
entry point, which takes caller-allocated scratch.  The file name sorts last
so a run that stops at the first failure has already run every other test.
"""

import ctypes
import math
import subprocess
import sys
import textwrap
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    import underhfs_b200._core as core_mod

    lib = ctypes.CDLL(core_mod.__file__)
    fn = lib.uhfs_flash_attn_bwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_void_p] + [ctypes.c_int] * 4 + [ctypes.c_float, ctypes.c_int,
                                                                                    ctypes.c_void_p]
    lib.uhfs_flash_attn_bwd_noalloc_error.restype = ctypes.c_char_p
    lib.uhfs_flash_attn_bwd_noalloc_capacity.restype = ctypes.c_ulonglong
    lib.uhfs_flash_attn_bwd_noalloc_status.restype = ctypes.c_int
    lib.uhfs_flash_attn_bwd_noalloc_status.argtypes = [ctypes.c_int]
    return lib


def _rel(a, b):
    return ((a.float() - b.float()).abs().max() / b.float().abs().max()).item()


def test_noalloc_matches_regular_entry_point_twice():
    from underhfs_b200.ops import kernels as K

    lib = _lib()
    B, T, H, D = 2, 384, 4, 64
    torch.manual_seed(0)
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        qkv = torch.randn(B * T, 3 * H * D, device="cuda", dtype=torch.bfloat16)
        o, lse = K.flash_attn_qkv(qkv, B, T, H, D, True)
        do = torch.randn_like(o)
        ref = K.flash_attn_qkv_backward(qkv, o, lse, do, B, T, H, D, True)
        out = torch.full_like(ref, float("nan"))
        rc = lib.uhfs_flash_attn_bwd_noalloc(qkv.data_ptr(), o.data_ptr(), lse.data_ptr(), do.data_ptr(),
                                            out.data_ptr(), B, T, H, D, 1.0 / math.sqrt(D), 1, stream)
        assert rc == 0, lib.uhfs_flash_attn_bwd_noalloc_error()
        torch.cuda.synchronize()
        assert torch.isfinite(out.float()).all(), f"call {call}"
        assert _rel(out, ref) < 2e-2, f"call {call}"


def test_noalloc_rejects_oversized_problem():
    lib = _lib()
    cap = lib.uhfs_flash_attn_bwd_noalloc_capacity()
    B, H, D = 8, 16, 128
    T = int(cap // (B * H * (D + 1) * 4)) + 64  # just past the capacity
    dummy = torch.empty(16, device="cuda")
    rc = lib.uhfs_flash_attn_bwd_noalloc(dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(),
                                        dummy.data_ptr(), B, T, H, D, 0.1, 1, 0)
    assert rc == 2
    assert b"scratch" in lib.uhfs_flash_attn_bwd_noalloc_error()


# Run in a fresh interpreter: the allocation-free entry point is the first
# call into the native library on the device, so it must resolve its scratch
# array and the device status word by itself.  Inputs come from plain torch
# (the forward output and its base-2 log-sum-exp computed in fp32), and the
# result is checked against torch autograd in fp32 and against the regular
# entry point called afterwards.
_FIRST_CALL = textwrap.dedent("""
    import ctypes, math, sys
    import torch
    sys.path.insert(0, sys.argv[1])
    from tests.test_zz_no_alloc import _lib, _rel
    B, T, H, D = 2, 256, 2, 64
    F = H * D
    scale = 1.0 / math.sqrt(D)
    torch.manual_seed(1)
    qkv = (0.5 * torch.randn(B * T, 3 * F, device="cuda")).to(torch.bfloat16)
    do = torch.randn(B * T, F, device="cuda").to(torch.bfloat16)

    def heads(x):
        return x.float().view(B, T, H, D).permute(0, 2, 1, 3)

    q, k, v = (heads(qkv[:, i * F:(i + 1) * F]).requires_grad_(True) for i in range(3))
    s = (q @ k.transpose(-1, -2)) * scale
    s = s.masked_fill(torch.ones(T, T, device="cuda", dtype=torch.bool).triu(1), float("-inf"))
    o32 = torch.softmax(s, -1) @ v
    lse = (torch.logsumexp(s, -1) / math.log(2.0)).detach().contiguous()
    o32.backward(heads(do))
    ref = torch.cat([t.grad.permute(0, 2, 1, 3).reshape(B * T, F) for t in (q, k, v)], 1)
    o = o32.detach().permute(0, 2, 1, 3).reshape(B * T, F).to(torch.bfloat16).contiguous()
    lib = _lib()
    out = torch.full((B * T, 3 * F), float("nan"), device="cuda", dtype=torch.bfloat16)
    rc = lib.uhfs_flash_attn_bwd_noalloc(qkv.data_ptr(), o.data_ptr(), lse.data_ptr(), do.data_ptr(),
                                        out.data_ptr(), B, T, H, D, scale, 1, 0)
    assert rc == 0, lib.uhfs_flash_attn_bwd_noalloc_error()
    torch.cuda.synchronize()
    assert lib.uhfs_flash_attn_bwd_noalloc_status(1) == 0
    assert torch.isfinite(out.float()).all()
    err = _rel(out, ref)
    assert err < 2e-2, err
    from underhfs_b200.ops import kernels as K
    reg = K.flash_attn_qkv_backward(qkv, o, lse, do, B, T, H, D, True)
    assert _rel(out, reg) < 2e-2
    print("FIRST-CALL OK", err)
""")


def test_noalloc_first_call_in_fresh_process():
    root = Path(__file__).resolve().parents[1]
    proc = subprocess.run([sys.executable, "-c", _FIRST_CALL, str(root)], cwd=str(root), capture_output=True,
                          text=True, timeout=600)
    assert proc.returncode == 0 and "FIRST-CALL OK" in proc.stdout, proc.stdout[-2000:] + proc.stderr[-4000:]
