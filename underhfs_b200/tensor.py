"""underHFS Tensor on top of PyTorch storage and autograd.

Keeps the reference Tensor's public contract (tensor.py:9-1088): the DType /
Layout / Device metadata enums, ``shape``/``strides``/``version``/``backend``,
views that share storage and version counters, the in-place guard message,
the dtype/device/layout mismatch messages, reverse-mode autograd with
``backward()``/``grad``, and the deterministic LCG initialisers.

Storage is a ``torch.Tensor``.  CPU tensors compute in float64, as the
reference's Python-float storage does (there fp16/bf16/fp8 are metadata on
the CPU); CUDA tensors hold their real dtype and route their hot ops
(add/mul/matmul/sum/softmax) to the sm_100a kernels of ``underhfs_b200._core``.
"""

from __future__ import annotations

from dataclasses import dataclass
from enum import Enum
from math import sqrt
from typing import Any, Sequence

import torch


class DType(str, Enum):
    FP32 = "fp32"
    FP16 = "fp16"
    BF16 = "bf16"
    FP8_E4M3 = "fp8_e4m3"
    FP8_E5M2 = "fp8_e5m2"
    INT8 = "int8"
    INT4 = "int4"


class Layout(str, Enum):
    DENSE = "dense"
    SPARSE = "sparse"
    QUANTIZED = "quantized"


@dataclass(frozen=True)
class Device:
    kind: str = "cpu"
    index: int | None = None

    @classmethod
    def parse(cls, value: "str | Device | torch.device") -> "Device":
        if isinstance(value, Device):
            return value
        if isinstance(value, torch.device):
            return cls(value.type, value.index if value.type == "cuda" else None)
        if ":" in value:
            kind, index = value.split(":", 1)
            return cls(kind, int(index))
        return cls(value, None)

    def __str__(self) -> str:
        return self.kind if self.index is None else f"{self.kind}:{self.index}"

    def torch(self) -> torch.device:
        if self.kind == "cuda":
            return torch.device("cuda", 0 if self.index is None else self.index)
        return torch.device(self.kind)


# Real device dtypes; the CPU keeps float64 like the reference's Python floats.
CUDA_TORCH_DTYPE = {
    DType.FP32: torch.float32,
    DType.FP16: torch.float16,
    DType.BF16: torch.bfloat16,
}


def torch_dtype_for(dtype: DType, device: Device) -> torch.dtype:
    if device.kind == "cuda":
        return CUDA_TORCH_DTYPE.get(dtype, torch.float32)
    return torch.float64


def dtype_from_torch(t: torch.dtype) -> DType:
    return {torch.float16: DType.FP16, torch.bfloat16: DType.BF16}.get(t, DType.FP32)


def _is_sequence(value: Any) -> bool:
    return isinstance(value, (list, tuple))


def _infer_shape(value: Any) -> tuple[int, ...]:
    if not _is_sequence(value):
        return ()
    if not value:
        return (0,)
    child = _infer_shape(value[0])
    for item in value:
        if _infer_shape(item) != child:
            raise ValueError("ragged tensors are not supported")
    return (len(value), *child)


def _flatten(value: Any) -> list[float]:
    if not _is_sequence(value):
        return [float(value)]
    out: list[float] = []
    for item in value:
        out.extend(_flatten(item))
    return out


def _prod(shape: Sequence[int]) -> int:
    n = 1
    for d in shape:
        n *= d
    return n


def _resolve_shape(shape: Sequence[int], numel: int) -> tuple[int, ...]:
    unknown = [i for i, d in enumerate(shape) if d == -1]
    if len(unknown) > 1:
        raise ValueError("only one inferred dimension is allowed")
    resolved = list(shape)
    if unknown:
        known = _prod([d for d in resolved if d != -1])
        if known == 0 or numel % known != 0:
            raise ValueError(f"cannot infer shape {tuple(shape)} for {numel} values")
        resolved[unknown[0]] = numel // known
    if any(d < 0 for d in resolved):
        raise ValueError(f"invalid shape {tuple(shape)}")
    return tuple(resolved)


def _contiguous_strides(shape: Sequence[int]) -> tuple[int, ...]:
    stride = 1
    out: list[int] = []
    for d in reversed(shape):
        out.append(stride)
        stride *= d
    return tuple(reversed(out))


def _native_status():
    from underhfs_b200.native import status

    return status()


class Tensor:
    """Eager tensor with reverse-mode autograd (PyTorch engine underneath)."""

    def __init__(
        self,
        data: Any = None,
        *,
        shape: Sequence[int] | None = None,
        requires_grad: bool = False,
        dtype: DType | str = DType.FP32,
        device: Device | str = Device(),
        layout: Layout | str = Layout.DENSE,
        _data: torch.Tensor | None = None,
        _backend: str = "python",
    ) -> None:
        self.dtype = DType(dtype)
        self.device = Device.parse(device)
        self.layout = Layout(layout)
        if _data is None:
            tdt = torch_dtype_for(self.dtype, self.device)
            if isinstance(data, torch.Tensor):
                t = data.detach().to(self.device.torch(), tdt)
                if shape is not None:
                    t = t.reshape(tuple(shape))
            elif isinstance(data, Tensor):
                t = data._data.detach().to(self.device.torch(), tdt).clone()
            else:
                inferred = _infer_shape(data) if shape is None else tuple(shape)
                flat = _flatten(data)
                if _prod(inferred) != len(flat):
                    raise ValueError(f"shape {inferred} expects {_prod(inferred)} values, got {len(flat)}")
                t = torch.tensor(flat, dtype=torch.float64).reshape(inferred).to(self.device.torch(), tdt)
            if requires_grad:
                t.requires_grad_(True)
            _data = t
        self._data = _data
        self.backend = _backend
        self._prev: tuple = ()
        self._op = ""

    # ------------------------------------------------------------ wrapping
    @classmethod
    def _wrap(cls, t: torch.Tensor, like: "Tensor | None" = None, backend: str = "python",
              dtype: DType | None = None, op: str = "", parents: tuple = ()) -> "Tensor":
        out = cls.__new__(Tensor)
        out._data = t
        out.dtype = dtype if dtype is not None else (like.dtype if like is not None else dtype_from_torch(t.dtype))
        out.device = Device.parse(t.device)
        out.layout = like.layout if like is not None else Layout.DENSE
        out.backend = backend
        # op tape used by the compile report (compile.py walks _prev like the reference)
        out._prev = tuple(p for p in parents if isinstance(p, Tensor))
        out._op = op
        return out

    # ------------------------------------------------------------ metadata
    @property
    def shape(self) -> tuple[int, ...]:
        return tuple(self._data.shape)

    @property
    def strides(self) -> tuple[int, ...]:
        return tuple(self._data.stride())

    @property
    def ndim(self) -> int:
        return self._data.dim()

    @property
    def version(self) -> int:
        return self._data._version

    @property
    def requires_grad(self) -> bool:
        return self._data.requires_grad

    @requires_grad.setter
    def requires_grad(self, value: bool) -> None:
        self._data.requires_grad_(bool(value))

    def numel(self) -> int:
        return self._data.numel()

    def is_contiguous(self) -> bool:
        return self._data.is_contiguous()

    def torch(self) -> torch.Tensor:
        """The underlying torch.Tensor (shares storage and autograd history)."""
        return self._data

    @property
    def _storage(self) -> list[float]:
        return [float(v) for v in self._data.detach().reshape(-1).cpu().tolist()]

    @_storage.setter
    def _storage(self, values: Sequence[float]) -> None:
        new = torch.tensor([float(v) for v in values], dtype=self._data.dtype).reshape(self._data.shape)
        self._data.data = new.to(self._data.device)

    # ------------------------------------------------------------- grads
    @property
    def grad(self) -> "Tensor | None":
        view = getattr(self, "_main_grad", None)
        if view is not None:
            return Tensor._wrap(view, like=self)
        g = self._data.grad
        return None if g is None else Tensor._wrap(g, like=self)

    @grad.setter
    def grad(self, value: "Tensor | None") -> None:
        view = getattr(self, "_main_grad", None)
        if view is not None:
            if value is None:
                view.zero_()
            else:
                view.copy_(value._data if isinstance(value, Tensor) else value)
            return
        if value is None:
            self._data.grad = None
        else:
            t = value._data if isinstance(value, Tensor) else value
            self._data.grad = t.detach().to(self._data.dtype)

    def zero_grad(self) -> None:
        self.grad = None

    def requires_grad_(self, requires_grad: bool = True) -> "Tensor":
        self._data.requires_grad_(requires_grad)
        return self

    def backward(self, grad: "Tensor | None" = None) -> None:
        if grad is None and self.numel() != 1:
            raise ValueError("grad must be provided for non-scalar tensors")
        g = None if grad is None else grad._data.to(self._data.dtype)
        if g is None:
            g = torch.ones_like(self._data)
        try:
            self._data.backward(g)
        except RuntimeError as exc:
            if "modified by an inplace operation" in str(exc):
                raise RuntimeError(
                    "autograd detected an in-place mutation before backward: "
                    f"{exc}. Use out-of-place ops, clone(), or detach() before mutating tensors "
                    "needed for gradients."
                ) from exc
            raise

    # ------------------------------------------------------------ copies
    def clone(self) -> "Tensor":
        t = self._data.detach().clone()
        if self.requires_grad:
            t.requires_grad_(True)
        return Tensor._wrap(t, like=self)

    def detach(self) -> "Tensor":
        return Tensor._wrap(self._data.detach().clone(), like=self)

    def to(self, device: "Device | str | None" = None, dtype: "DType | str | None" = None,
           layout: "Layout | str | None" = None) -> "Tensor":
        target = self.device if device is None else Device.parse(device)
        if target.kind == "cuda":
            native = _native_status()
            if not native.available:
                raise RuntimeError(
                    f"cannot move tensor to CUDA because the native core is unavailable: {native.reason}"
                )
            if not native.cuda_enabled:
                raise RuntimeError(
                    "cannot move tensor to CUDA because the native core is unavailable: "
                    f"{native.reason or 'no CUDA device is visible'} (built without CUDA support for this host)"
                )
        new_dtype = self.dtype if dtype is None else DType(dtype)
        t = self._data.detach().to(target.torch(), torch_dtype_for(new_dtype, target)).clone()
        if self.requires_grad:
            t.requires_grad_(True)
        out = Tensor._wrap(t, dtype=new_dtype, backend="native_cuda" if target.kind == "cuda" else "python")
        out.layout = self.layout if layout is None else Layout(layout)
        return out

    def cpu(self) -> "Tensor":
        return self.to("cpu")

    def cuda(self, index: int = 0) -> "Tensor":
        return self.to(Device("cuda", index))

    def tolist(self) -> Any:
        v = self._data.detach().cpu()
        if v.dtype in (torch.float16, torch.bfloat16):
            v = v.float()
        return v.double().tolist() if v.dim() else float(v.item())

    def item(self) -> float:
        if self.numel() != 1:
            raise ValueError("item() is only valid for single-value tensors")
        return float(self._data.detach().reshape(-1)[0].item())

    def argmax(self) -> int:
        if self.numel() == 0:
            raise ValueError("argmax() is not valid for empty tensors")
        return int(torch.argmax(self._data.detach().reshape(-1)).item())

    # ------------------------------------------------------------ checks
    def _ensure(self, other: Any) -> "Tensor | float":
        if isinstance(other, Tensor):
            return other
        if isinstance(other, (int, float)):
            return float(other)
        return tensor(other, dtype=self.dtype, device=self.device, layout=self.layout)

    def _check_compatible(self, other: "Tensor", op: str) -> None:
        if self.device != other.device:
            raise RuntimeError(
                f"{op} received tensors on different devices: {self.device} and {other.device}. "
                "Move tensors explicitly with .to(...), .cpu(), or .cuda()."
            )
        if self.layout != other.layout:
            raise RuntimeError(
                f"{op} received tensors with different layouts: {self.layout.value} and "
                f"{other.layout.value}. Convert layout explicitly before the operation."
            )
        if self.dtype != other.dtype and self.shape != () and other.shape != ():
            raise RuntimeError(
                f"{op} received tensors with different dtypes: {self.dtype.value} and "
                f"{other.dtype.value}. Cast explicitly with .to(dtype=...)."
            )

    def _native_cpu_eligible(self) -> bool:
        return (
            self.device.kind == "cpu"
            and self.layout is Layout.DENSE
            and self.dtype is DType.FP32
            and self._data.is_contiguous()
            and _native_status().available
        )

    def _native_cuda_eligible(self) -> bool:
        return (
            self.device.kind == "cuda"
            and self.layout is Layout.DENSE
            and self.dtype in CUDA_TORCH_DTYPE
            and self._data.is_contiguous()
        )

    # ------------------------------------------------------------ binary
    def _binary(self, other: Any, op: str) -> "Tensor":
        rhs = self._ensure(other)
        if isinstance(rhs, Tensor):
            self._check_compatible(rhs, op)
            if (
                op in ("add", "mul")
                and self.shape == rhs.shape
                and self.dtype == rhs.dtype
                and self._native_cuda_eligible()
                and rhs._native_cuda_eligible()
            ):
                from underhfs_b200.ops import functions as OF

                return Tensor._wrap(OF.ew(op, self._data, rhs._data), like=self, backend="native_cuda", op=op,
                                    parents=(self, rhs))
            a, b = self._data, rhs._data
            if b.dtype != a.dtype:
                b = b.to(a.dtype)
        else:
            a, b = self._data, rhs
        fn = {"add": torch.add, "sub": torch.sub, "mul": torch.mul, "div": torch.div}[op]
        backend = "python"
        if (
            op in ("add", "mul")
            and isinstance(rhs, Tensor)
            and self.shape == rhs.shape
            and self._native_cpu_eligible()
            and rhs._native_cpu_eligible()
        ):
            backend = "native_cpu"
        return Tensor._wrap(fn(a, b), like=self, backend=backend, op=op, parents=(self, rhs))

    def __add__(self, other: Any) -> "Tensor":
        return self._binary(other, "add")

    def __radd__(self, other: Any) -> "Tensor":
        return self._binary(other, "add")

    def __sub__(self, other: Any) -> "Tensor":
        return self._binary(other, "sub")

    def __rsub__(self, other: Any) -> "Tensor":
        return tensor(other, dtype=self.dtype, device=self.device, layout=self.layout) - self

    def __mul__(self, other: Any) -> "Tensor":
        return self._binary(other, "mul")

    def __rmul__(self, other: Any) -> "Tensor":
        return self._binary(other, "mul")

    def __truediv__(self, other: Any) -> "Tensor":
        return self._binary(other, "div")

    def __rtruediv__(self, other: Any) -> "Tensor":
        return tensor(other, dtype=self.dtype, device=self.device, layout=self.layout) / self

    def __neg__(self) -> "Tensor":
        return self * -1.0

    def __pow__(self, power: float) -> "Tensor":
        return Tensor._wrap(self._data ** power, like=self, op="pow", parents=(self,))

    def __matmul__(self, other: Any) -> "Tensor":
        rhs = self._ensure(other)
        if not isinstance(rhs, Tensor):
            raise TypeError("matmul requires a tensor operand")
        self._check_compatible(rhs, "matmul")
        if self.ndim != 2 or rhs.ndim != 2:
            raise ValueError("matmul supports 2D tensors")
        (m, k), (k2, n) = self.shape, rhs.shape
        if k != k2:
            raise ValueError(f"matmul shape mismatch: {self.shape} @ {rhs.shape}")
        if self.device.kind == "cuda" and self.dtype in CUDA_TORCH_DTYPE:
            from underhfs_b200.ops import functions as OF

            return Tensor._wrap(OF.matmul(self._data, rhs._data), like=self, backend="native_cuda", op="matmul",
                                parents=(self, rhs))
        backend = "native_cpu" if (self._native_cpu_eligible() and rhs._native_cpu_eligible()) else "python"
        return Tensor._wrap(self._data @ rhs._data, like=self, backend=backend, op="matmul", parents=(self, rhs))

    def add_(self, other: Any) -> "Tensor":
        rhs = self._ensure(other)
        if isinstance(rhs, Tensor):
            self._check_compatible(rhs, "add_")
            value = rhs._data.to(self._data.dtype)
            out_shape = torch.broadcast_shapes(self.shape, rhs.shape)
            if tuple(out_shape) != self.shape:
                raise RuntimeError(f"in-place add cannot change tensor shape from {self.shape} to {tuple(out_shape)}")
        else:
            value = rhs
        with torch.no_grad():
            self._data.add_(value)
        if self.device.kind == "cuda":
            self.backend = "native_cuda"
        return self

    # -------------------------------------------------------- reductions
    def sum(self) -> "Tensor":
        if self.device.kind == "cuda" and self.dtype is DType.FP32 and self._data.is_contiguous():
            from underhfs_b200.ops import functions as OF

            return Tensor._wrap(OF.sum_all(self._data), like=self, backend="native_cuda", op="sum", parents=(self,))
        backend = "native_cpu" if self._native_cpu_eligible() else "python"
        return Tensor._wrap(self._data.sum(), like=self, backend=backend, op="sum", parents=(self,))

    def mean(self) -> "Tensor":
        return self.sum() / max(1, self.numel())

    # ---------------------------------------------------------- unary
    def relu(self) -> "Tensor":
        return Tensor._wrap(torch.relu(self._data), like=self, op="relu", parents=(self,))

    def tanh(self) -> "Tensor":
        return Tensor._wrap(torch.tanh(self._data), like=self, op="tanh", parents=(self,))

    def exp(self) -> "Tensor":
        return Tensor._wrap(torch.exp(self._data), like=self, op="exp", parents=(self,))

    def log(self) -> "Tensor":
        return Tensor._wrap(torch.log(self._data), like=self, op="log", parents=(self,))

    def sqrt(self) -> "Tensor":
        return self ** 0.5

    def softmax(self) -> "Tensor":
        if self.ndim not in (1, 2):
            raise ValueError("softmax supports 1D or 2D tensors")
        if self.device.kind == "cuda" and self.dtype in CUDA_TORCH_DTYPE:
            from underhfs_b200.ops import functions as OF

            return Tensor._wrap(OF.softmax(self._data), like=self, backend="native_cuda", op="softmax",
                                parents=(self,))
        return Tensor._wrap(torch.softmax(self._data, dim=-1), like=self, op="softmax", parents=(self,))

    # ---------------------------------------------------------- views
    def transpose(self) -> "Tensor":
        if self.ndim != 2:
            raise ValueError("transpose supports 2D tensors")
        return Tensor._wrap(self._data.t(), like=self, op="transpose", parents=(self,))

    @property
    def T(self) -> "Tensor":
        return self.transpose()

    def view(self, *shape: int) -> "Tensor":
        if len(shape) == 1 and isinstance(shape[0], (tuple, list)):
            shape = tuple(shape[0])
        actual = _resolve_shape(shape, self.numel())
        if not self._data.is_contiguous():
            raise ValueError("view requires a contiguous tensor; call reshape() for a copied fallback")
        if _prod(actual) != self.numel():
            raise ValueError(f"cannot view {self.shape} as {actual}")
        return Tensor._wrap(self._data.view(actual), like=self, backend=self.backend, op="view", parents=(self,))

    def flatten(self) -> "Tensor":
        return self.view(self.numel())

    def reshape(self, *shape: int) -> "Tensor":
        if len(shape) == 1 and isinstance(shape[0], (tuple, list)):
            shape = tuple(shape[0])
        actual = _resolve_shape(shape, self.numel())
        if _prod(actual) != self.numel():
            raise ValueError(f"cannot reshape {self.shape} to {actual}")
        if self._data.is_contiguous():
            return self.view(*actual)
        return Tensor._wrap(self._data.reshape(actual), like=self, op="reshape", parents=(self,))

    def __getitem__(self, key: Any) -> "Tensor":
        if not isinstance(key, tuple):
            key = (key,)
        if any(item is Ellipsis for item in key):
            raise IndexError("ellipsis indexing is not supported yet")
        if len(key) > self.ndim:
            raise IndexError(f"too many indices for tensor of dimension {self.ndim}")
        for axis, item in enumerate(key):
            if isinstance(item, int):
                dim = self.shape[axis]
                actual = item + dim if item < 0 else item
                if actual < 0 or actual >= dim:
                    raise IndexError(f"index {item} is out of bounds for axis {axis} with size {dim}")
            elif not isinstance(item, slice):
                raise IndexError("tensor indices must be integers or slices")
        return Tensor._wrap(self._data[key], like=self, op="slice", parents=(self,))

    def __len__(self) -> int:
        return self.shape[0] if self.shape else 0

    def __repr__(self) -> str:
        return (
            f"Tensor(data={self.tolist()!r}, shape={self.shape}, dtype={self.dtype.value}, "
            f"device={self.device}, requires_grad={self.requires_grad})"
        )


def tensor(data: Any, **kwargs: Any) -> Tensor:
    return Tensor(data, **kwargs)


def zeros(shape: int | Sequence[int], **kwargs: Any) -> Tensor:
    actual = (shape,) if isinstance(shape, int) else tuple(shape)
    dev = Device.parse(kwargs.get("device", Device()))
    dt = DType(kwargs.get("dtype", DType.FP32))
    return Tensor(torch.zeros(actual, dtype=torch_dtype_for(dt, dev)), **kwargs)


def ones(shape: int | Sequence[int], **kwargs: Any) -> Tensor:
    actual = (shape,) if isinstance(shape, int) else tuple(shape)
    dev = Device.parse(kwargs.get("device", Device()))
    dt = DType(kwargs.get("dtype", DType.FP32))
    return Tensor(torch.ones(actual, dtype=torch_dtype_for(dt, dev)), **kwargs)


def arange(stop: int, **kwargs: Any) -> Tensor:
    return Tensor(torch.arange(stop, dtype=torch.float64), **kwargs)


def lcg_values(n: int) -> torch.Tensor:
    """((i * 1103515245 + 12345) % 10000) / 5000 - 1 for i in [0, n) -- the
    reference's deterministic initialiser (tensor.py:1076-1088), vectorised."""
    i = torch.arange(n, dtype=torch.int64)
    return ((i * 1103515245 + 12345) % 10000).to(torch.float64) / 5000.0 - 1.0


def kaiming_uniform(rows: int, cols: int) -> Tensor:
    bound = sqrt(6.0 / max(1, rows + cols))
    return Tensor(lcg_values(rows * cols).reshape(rows, cols) * bound, requires_grad=True)


def uniform(shape: Sequence[int], bound: float, *, requires_grad: bool = False) -> Tensor:
    total = _prod(shape)
    return Tensor(lcg_values(total).reshape(tuple(shape)) * bound, requires_grad=requires_grad)
