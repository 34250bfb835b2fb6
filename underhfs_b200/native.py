"""Status, loading and self-test of the native core ``underhfs_b200._core``.

Contract kept from the reference (native.py:13-178): ``status()`` never
raises and reports availability plus the cuda / cudnn / nccl feature flags,
``require_native()`` raises ``RuntimeError`` with the reason, and ``probe()``
exercises every binding on fixed tiny inputs whose exact outputs the tests
assert.  On this framework ``cuda_enabled`` additionally requires a visible
CUDA device, so a CPU-only host reports CUDA as unavailable instead of failing
on the first launch; ``cudnn_enabled`` means "conv2d kernels present" (they are
this library's own kernels, not cuDNN).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any


@dataclass(frozen=True)
class NativeStatus:
    available: bool
    reason: str | None = None
    cuda_enabled: bool = False
    cudnn_enabled: bool = False
    nccl_enabled: bool = False


_STATUS: NativeStatus | None = None


def _load():
    from underhfs_b200.ops._lib import core

    return core()


def status() -> NativeStatus:
    global _STATUS
    if _STATUS is not None:
        return _STATUS
    try:
        core = _load()
    except Exception as exc:  # noqa: BLE001 - report, never raise
        return NativeStatus(False, str(exc))
    try:
        import torch

        have_device = torch.cuda.is_available()
    except Exception:  # noqa: BLE001
        have_device = False
    built_cuda = bool(getattr(core, "cuda_enabled", False))
    reason = None if have_device else "no CUDA device is visible to this process"
    _STATUS = NativeStatus(
        True,
        reason,
        built_cuda and have_device,
        bool(getattr(core, "cudnn_enabled", False)) and have_device,
        bool(getattr(core, "nccl_enabled", False)) and have_device,
    )
    return _STATUS


def require_native():
    st = status()
    if not st.available:
        raise RuntimeError(f"underHFS native core is unavailable: {st.reason}")
    return _load()


def probe() -> dict[str, Any]:
    """Run every native entry point once on fixed inputs (see module doc)."""
    core = require_native()
    st = status()
    a = core.TensorCore([1.0, 2.0, 3.0, 4.0], [2, 2])
    b = core.TensorCore([5.0, 6.0, 7.0, 8.0], [2, 2])
    prod = a.matmul(b)
    out: dict[str, Any] = {
        "version": getattr(core, "__version__", "unknown"),
        "arch": getattr(core, "arch", "unknown"),
        "cuda_enabled": st.cuda_enabled,
        "cudnn_enabled": st.cudnn_enabled,
        "nccl_enabled": st.nccl_enabled,
        "numel": a.numel(),
        "shape": list(a.shape),
        "strides": list(a.strides),
        "add": list(a.add(b).storage),
        "matmul": list(prod.storage),
        "sum": list(prod.sum().storage),
    }
    if not st.cuda_enabled:
        return out
    out["cuda_add_f32"] = list(core.cuda_add_f32([1.0, 2.0], [3.0, 4.0]))
    x = core.CudaTensorF32([1.0, 2.0], [2])
    y = core.CudaTensorF32([3.0, 4.0], [2])
    out["cuda_tensor_add_f32"] = list(x.add(y).to_host())
    out["cuda_tensor_mul_f32"] = list(x.mul(y).to_host())
    out["cuda_tensor_sum_f32"] = list(x.sum().to_host())
    m1 = core.CudaTensorF32([1.0, 2.0, 3.0, 4.0], [2, 2])
    m2 = core.CudaTensorF32([5.0, 6.0, 7.0, 8.0], [2, 2])
    out["cuda_tensor_matmul_f32"] = list(m1.matmul(m2).to_host())
    adam = core.cuda_fused_adamw_f32([1.0, 2.0], [0.1, 0.2], [0.0, 0.0], [0.0, 0.0], 0.01, 0.9, 0.999, 1e-8, 0.0, 1)
    out["cuda_fused_adamw_f32"] = {k: list(v) for k, v in adam.items()}
    out["cuda_attention_f32"] = list(
        core.cuda_attention_f32([1.0, 0.0, 0.0, 1.0], [1.0, 0.0, 0.0, 1.0], [1.0, 2.0, 3.0, 4.0], 2, 2, 1.0, False)
    )
    if st.cudnn_enabled:
        out["cudnn_conv2d_backward_input_f32"] = list(
            core.cudnn_conv2d_backward_input_f32([1.0], [2.0], 1, 1, 1, 1, 1, 1, 1, 1, 1, 0, 0)
        )
        out["cudnn_conv2d_backward_weight_f32"] = list(
            core.cudnn_conv2d_backward_weight_f32([2.0], [1.0], 1, 1, 1, 1, 1, 1, 1, 1, 1, 0, 0)
        )
    for name, ctor in (("f16", core.CudaTensorF16), ("bf16", core.CudaTensorBF16)):
        p = ctor([1.0, 2.0], [2])
        q = ctor([3.0, 4.0], [2])
        out[f"cuda_tensor_add_{name}"] = list(p.add(q).to_host())
        out[f"cuda_tensor_mul_{name}"] = list(p.mul(q).to_host())
    out["cuda_allocator"] = {str(k): int(v) for k, v in core.cuda_allocator_stats().items()}
    out["cuda_stream"] = {str(k): int(v) for k, v in core.cuda_stream_stats().items()}
    return out
