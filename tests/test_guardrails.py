"""Loud failures: in-place guard, dtype / device mismatch, doctor + CLI."""

from underhfs import tensor
from underhfs.cli import main
from underhfs.diagnostics import doctor
from underhfs.tensor import DType


def test_inplace_mutation_detected_at_backward():
    a = tensor(2.0, requires_grad=True)
    b = a * a
    a.add_(1.0)
    try:
        b.backward()
    except RuntimeError as exc:
        assert "in-place mutation" in str(exc)
    else:
        raise AssertionError("in-place mutation of a saved tensor must be detected")


def test_dtype_mismatch_is_explicit():
    try:
        _ = tensor([1.0, 2.0], dtype=DType.FP32) + tensor([1.0, 2.0], dtype=DType.FP16)
    except RuntimeError as exc:
        assert "different dtypes" in str(exc)
    else:
        raise AssertionError("mixed dtypes must not broadcast silently")


def test_scalar_dtype_mixing_allowed():
    out = tensor([1.0, 2.0], dtype=DType.FP16) * 2.0
    assert out.tolist() == [2.0, 4.0]


def test_doctor_report_and_cli():
    rep = doctor()
    assert rep.python
    assert "git" in rep.tools
    assert isinstance(rep.native_cudnn, bool) and isinstance(rep.native_nccl, bool)
    for dep in ("onnx", "grpcio", "opencv-python", "websockets"):
        assert dep in rep.optional_dependencies
    assert isinstance(rep.cuda_devices, list)
    assert "vram" in rep.memory_budgets or not rep.cuda_visible
    d = rep.to_dict()
    assert "native_cudnn" in d and "optional_dependencies" in d
    assert main(["doctor"]) == 0
