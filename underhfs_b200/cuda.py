"""Runtime policies, kernel capability matrix, device discovery and CUDA hooks.

Reference: cuda.py:12-315.  The policy dataclasses and the capability /
device / budget API keep their names and fields; ``PrecisionPolicy`` gains
``dtype`` (bf16 is the training dtype on B200).  The capability matrix lists
the kernels this build really has (tcgen05 bf16 GEMM, flash attention,
RMSNorm, GELU, embedding, softmax cross-entropy, fused AdamW, conv2d,
elementwise / reduction for fp32/fp16/bf16).  RAM is read from
``/proc/meminfo`` on Linux (the reference only implements Windows).
"""

from __future__ import annotations

import os
from dataclasses import dataclass, field
from enum import Enum
from shutil import which
from subprocess import run

from underhfs_b200.tensor import DType


class MemoryTier(str, Enum):
    VRAM = "vram"
    RAM = "ram"
    NVME = "nvme"
    NETWORK = "network"


@dataclass
class MemoryPolicy:
    tiers: tuple[MemoryTier, ...] = (MemoryTier.VRAM, MemoryTier.RAM)
    allow_offload: bool = True
    allow_prefetch: bool = True
    activation_checkpointing: bool = True
    recompute: bool = True
    scratch_path: str | None = None


@dataclass
class PrecisionPolicy:
    strict: bool = False
    allow_fp8: bool = True
    allow_int4: bool = True
    loss_scaling: str = "dynamic"
    dtype: str = "bf16"


@dataclass
class RuntimePolicy:
    memory: MemoryPolicy = field(default_factory=MemoryPolicy)
    precision: PrecisionPolicy = field(default_factory=PrecisionPolicy)
    stream_aware: bool = True


@dataclass(frozen=True)
class KernelCapability:
    op: str
    device: str
    dtypes: tuple[DType, ...]
    forward: str
    backward: str

    def to_dict(self) -> dict[str, str | list[str]]:
        return {
            "op": self.op,
            "device": self.device,
            "dtypes": [d.value for d in self.dtypes],
            "forward": self.forward,
            "backward": self.backward,
        }


@dataclass(frozen=True)
class CudaDeviceInfo:
    index: int
    name: str
    memory_total_bytes: int
    memory_free_bytes: int
    driver_version: str

    def to_dict(self) -> dict[str, int | str]:
        return {
            "index": self.index,
            "name": self.name,
            "memory_total_bytes": self.memory_total_bytes,
            "memory_free_bytes": self.memory_free_bytes,
            "driver_version": self.driver_version,
        }


_SMI_FIELDS = "index,name,memory.total,memory.free,driver_version"


def is_available() -> bool:
    return which("nvidia-smi") is not None


def device_count() -> int:
    return len(devices())


def devices() -> list[CudaDeviceInfo]:
    if not is_available():
        return []
    proc = run(["nvidia-smi", f"--query-gpu={_SMI_FIELDS}", "--format=csv,noheader,nounits"],
               capture_output=True, text=True, check=False)
    return [] if proc.returncode else _parse_nvidia_smi_devices(proc.stdout)


def _parse_nvidia_smi_devices(output: str) -> list[CudaDeviceInfo]:
    out: list[CudaDeviceInfo] = []
    for line in output.splitlines():
        fields = [f.strip() for f in line.split(",")]
        if len(fields) != 5 or not line.strip():
            continue
        try:
            idx, name, total, free, drv = fields
            out.append(CudaDeviceInfo(int(idx), name, int(float(total) * 2**20), int(float(free) * 2**20), drv))
        except ValueError:
            continue
    return out


def _available_ram_bytes() -> int | None:
    """MemAvailable from /proc/meminfo (Linux) or GlobalMemoryStatusEx (Windows)."""
    try:
        with open("/proc/meminfo", encoding="ascii") as fh:
            for line in fh:
                if line.startswith("MemAvailable:"):
                    return int(line.split()[1]) * 1024
    except OSError:
        pass
    if os.name == "nt":  # pragma: no cover - not exercised on Linux hosts
        import ctypes

        class _Status(ctypes.Structure):
            _fields_ = [("dwLength", ctypes.c_ulong), ("dwMemoryLoad", ctypes.c_ulong),
                        ("ullTotalPhys", ctypes.c_ulonglong), ("ullAvailPhys", ctypes.c_ulonglong),
                        ("ullTotalPageFile", ctypes.c_ulonglong), ("ullAvailPageFile", ctypes.c_ulonglong),
                        ("ullTotalVirtual", ctypes.c_ulonglong), ("ullAvailVirtual", ctypes.c_ulonglong),
                        ("ullAvailExtendedVirtual", ctypes.c_ulonglong)]

        st = _Status()
        st.dwLength = ctypes.sizeof(_Status)
        if ctypes.windll.kernel32.GlobalMemoryStatusEx(ctypes.byref(st)):
            return int(st.ullAvailPhys)
    return None


def memory_budgets(vram_fraction: float = 0.9) -> dict[MemoryTier, int]:
    if not 0.0 < vram_fraction <= 1.0:
        raise ValueError("vram_fraction must be in the range (0, 1]")
    budgets: dict[MemoryTier, int] = {}
    gpus = devices()
    if gpus:
        budgets[MemoryTier.VRAM] = int(sum(d.memory_free_bytes for d in gpus) * vram_fraction)
    ram = _available_ram_bytes()
    if ram is not None:
        budgets[MemoryTier.RAM] = int(ram * 0.8)
    return budgets


def require_cuda_toolkit() -> None:
    if which("nvcc") is None:
        raise RuntimeError("CUDA Toolkit nvcc was not found on PATH. Install CUDA Toolkit 12.9+ for sm_100a builds.")


_ALL = (DType.FP32, DType.FP16, DType.BF16, DType.FP8_E4M3, DType.FP8_E5M2, DType.INT8, DType.INT4)
_DEV = (DType.FP32, DType.FP16, DType.BF16)


def capability_matrix() -> list[KernelCapability]:
    """Kernels this build exposes.  Unsupported combinations are absent, so
    ``require_kernel`` fails loudly instead of silently falling back."""
    from underhfs_b200.native import status

    caps = [
        KernelCapability("add", "cpu", _ALL, "torch-cpu-fp64", "autograd"),
        KernelCapability("mul", "cpu", _ALL, "torch-cpu-fp64", "autograd"),
        KernelCapability("matmul", "cpu", (DType.FP32,), "torch-cpu-fp64", "autograd"),
        KernelCapability("sum", "cpu", _ALL, "torch-cpu-fp64", "autograd"),
    ]
    if status().cuda_enabled:
        caps += [
            KernelCapability("add", "cuda", _DEV, "sm100a-vectorized", "sm100a-vectorized"),
            KernelCapability("mul", "cuda", _DEV, "sm100a-vectorized", "sm100a-vectorized"),
            KernelCapability("sum", "cuda", (DType.FP32,), "sm100a-single-pass-reduce", "broadcast"),
            KernelCapability("matmul", "cuda", (DType.FP32,), "sm100a-fp32-fma", "sm100a-fp32-fma"),
            KernelCapability("matmul", "cuda", (DType.BF16,), "sm100a-tcgen05-tma", "sm100a-tcgen05-tma"),
            KernelCapability("linear", "cuda", (DType.BF16,), "tcgen05+bias/gelu/residual epilogue",
                             "tcgen05 dgrad(+dgelu) / split-K wgrad"),
            KernelCapability("attention", "cuda", (DType.FP32,), "native-cuda-attention", "row-softmax-kernels"),
            KernelCapability("attention", "cuda", (DType.BF16,), "sm100a-flash-attention", "sm100a-flash-attention"),
            KernelCapability("rms_norm", "cuda", _DEV, "sm100a-warp-per-row", "sm100a-fused-residual"),
            KernelCapability("gelu", "cuda", _DEV, "sm100a", "sm100a"),
            KernelCapability("embedding", "cuda", _DEV, "sm100a-gather", "sm100a-scatter-add-fp32"),
            KernelCapability("cross_entropy", "cuda", _DEV, "sm100a-fused-softmax-ce", "fused-in-forward"),
            KernelCapability("softmax", "cuda", _DEV, "sm100a-row-softmax", "sm100a-row-softmax"),
            KernelCapability("conv2d", "cuda", (DType.FP32,), "native-sm100a-conv", "native-sm100a-conv"),
            KernelCapability("fused_adamw", "cuda", _DEV, "sm100a-flat-fused-adamw", "optimizer-state-preserving"),
        ]
    return caps


def supports_kernel(op: str, *, device: str = "cpu", dtype: DType | str = DType.FP32) -> bool:
    want = DType(dtype)
    return any(c.op == op and c.device == device and want in c.dtypes for c in capability_matrix())


def require_kernel(op: str, *, device: str = "cpu", dtype: DType | str = DType.FP32) -> None:
    if supports_kernel(op, device=device, dtype=dtype):
        return
    variants = [c.to_dict() for c in capability_matrix() if c.op == op and c.device == device]
    raise RuntimeError(
        f"underHFS does not have a {device} {DType(dtype).value} kernel for {op}. "
        f"Supported variants: {variants or 'none'}"
    )


def _core_or_raise(what: str):
    from underhfs_b200.native import require_native, status

    core = require_native()
    if not status().cuda_enabled:
        raise RuntimeError(f"CUDA {what} is unavailable: no CUDA device is visible to this process")
    return core


def allocator_stats() -> dict[str, int]:
    return {str(k): int(v) for k, v in _core_or_raise("allocator stats").cuda_allocator_stats().items()}


def empty_cache() -> None:
    _core_or_raise("empty_cache").cuda_empty_cache()


def stream_stats() -> dict[str, int]:
    return {str(k): int(v) for k, v in _core_or_raise("stream stats").cuda_stream_stats().items()}


def synchronize() -> None:
    core = _core_or_raise("synchronize")
    core.cuda_synchronize()
    import torch

    torch.cuda.synchronize()
