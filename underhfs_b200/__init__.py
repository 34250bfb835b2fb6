"""underhfs_b200: a Blackwell (sm_100a) native framework with the underHFS API.

Public API (reference src/underhfs/__init__.py): Tensor, DType, Layout,
Device and the tensor factories.  Submodules: nn, optim, functional,
autograd, distributed, cuda, runtime, compile, serialization, serve, cli,
benchmarks, diagnostics, data, datasets, text, testing, config, train.
"""

from underhfs_b200.tensor import Device, DType, Layout, Tensor, arange, ones, tensor, zeros

__all__ = ["Device", "DType", "Layout", "Tensor", "arange", "ones", "tensor", "zeros"]

__version__ = "0.2.0"
