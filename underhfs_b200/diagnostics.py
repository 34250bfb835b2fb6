"""Environment report (reference diagnostics.py:16-138)."""

from __future__ import annotations

import platform
import sys
from dataclasses import dataclass, field
from importlib.util import find_spec
from shutil import which
from subprocess import run

from underhfs_b200.cuda import device_count, devices, is_available, memory_budgets
from underhfs_b200.native import probe as native_probe
from underhfs_b200.native import status as native_status


@dataclass
class DoctorReport:
    python: str
    platform: str
    cuda_visible: bool
    cuda_device_count: int
    cuda_devices: list[dict]
    memory_budgets: dict[str, int]
    native_core: bool
    native_cuda: bool
    native_cudnn: bool
    native_nccl: bool
    native_probe: dict | None
    optional_dependencies: dict[str, bool]
    tools: dict[str, str | None]
    warnings: list[str] = field(default_factory=list)
    native_arch: str | None = None
    torch_version: str | None = None

    def to_dict(self) -> dict:
        return dict(vars(self))


def _optional_dependencies() -> dict[str, bool]:
    return {"onnx": find_spec("onnx") is not None, "grpcio": find_spec("grpc") is not None,
            "opencv-python": find_spec("cv2") is not None, "websockets": find_spec("websockets") is not None}


def doctor() -> DoctorReport:
    st = native_status()
    tools = {t: which(t) for t in ("git", "cmake", "ninja", "nvcc", "cl", "nvidia-smi")}
    deps = _optional_dependencies()
    warns: list[str] = []
    if not st.available:
        warns.append(f"native core unavailable: {st.reason}")
    if tools["nvcc"] is None:
        warns.append("CUDA Toolkit nvcc is not on PATH; the sm_100a native core cannot be rebuilt.")
    if tools["ninja"] is None:
        warns.append("Ninja is not on PATH; native builds need it.")
    probe = None
    arch = None
    if st.available:
        if not st.cuda_enabled:
            warns.append(f"native core loaded, CUDA paths inactive: {st.reason}")
        if not deps["onnx"]:
            warns.append("optional dependency 'onnx' is missing; ONNX export uses the underhfs.onnx-lite fallback.")
        if not deps["grpcio"]:
            warns.append("optional dependency 'grpcio' is missing; gRPC serving is manifest-only.")
        if not deps["opencv-python"]:
            warns.append("optional dependency 'opencv-python' is missing; webcam streams are disabled.")
        try:
            probe = native_probe()
            arch = probe.get("arch")
        except Exception as exc:  # noqa: BLE001
            warns.append(f"native probe failed: {exc}")
    try:
        import torch

        tv = torch.__version__
    except Exception:  # noqa: BLE001
        tv = None
    return DoctorReport(
        python=sys.version.split()[0], platform=platform.platform(), cuda_visible=is_available(),
        cuda_device_count=device_count(), cuda_devices=[d.to_dict() for d in devices()],
        memory_budgets={t.value: n for t, n in memory_budgets().items()}, native_core=st.available,
        native_cuda=st.cuda_enabled, native_cudnn=st.cudnn_enabled, native_nccl=st.nccl_enabled,
        native_probe=probe, optional_dependencies=deps, tools=tools, warnings=warns, native_arch=arch,
        torch_version=tv,
    )


def nvidia_smi_summary() -> str | None:
    exe = which("nvidia-smi")
    if exe is None:
        return None
    res = run([exe], capture_output=True, text=True, check=False)
    return (res.stdout if res.returncode == 0 else res.stderr).strip()
