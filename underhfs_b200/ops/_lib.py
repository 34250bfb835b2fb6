"""Access to the native core and small launch helpers.

Every CUDA op of the framework goes through :func:`core`, which imports the
in-tree ``underhfs_b200._core`` extension.  When a CUDA device is present and
the extension cannot be imported the error is raised, never hidden: there is
no silent PyTorch fallback for the kernels this package provides.
"""

from __future__ import annotations

import functools
import os

import torch

DT_F32, DT_F16, DT_BF16 = 0, 1, 2
_DT = {torch.float32: DT_F32, torch.float16: DT_F16, torch.bfloat16: DT_BF16}


class NativeCoreMissing(RuntimeError):
    pass


@functools.lru_cache(maxsize=1)
def _import_core():
    from underhfs_b200 import _core  # noqa: F401  (in-tree extension)

    return _core


def core():
    """Return the native module, building it in place if allowed and missing."""
    try:
        return _import_core()
    except ImportError as exc:
        if os.environ.get("UNDERHFS_AUTOBUILD", "1") == "1":
            from underhfs_b200 import _native_build

            _native_build.build()
            _import_core.cache_clear()
            return _import_core()
        raise NativeCoreMissing(f"underhfs_b200 native core is not built: {exc}") from exc


def dt(t: torch.Tensor) -> int:
    try:
        return _DT[t.dtype]
    except KeyError as exc:
        raise TypeError(f"unsupported dtype for native kernel: {t.dtype}") from exc


def stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def ptr(t: torch.Tensor | None) -> int:
    return 0 if t is None else t.data_ptr()


def cuda_ready() -> bool:
    return torch.cuda.is_available()
