"""``import underhfs`` compatibility name for underhfs_b200.

Code written against the reference package (``from underhfs.nn import ...``)
runs unchanged: every public submodule of underhfs_b200 is registered here
under the ``underhfs.`` prefix.  Package attributes that name both a
submodule and a function (``tensor``) resolve to the function, as in the
reference package.
"""

import importlib
import sys

import underhfs_b200 as _impl
from underhfs_b200 import *  # noqa: F401,F403
from underhfs_b200 import __all__, __version__  # noqa: F401

_SUBMODULES = (
    "tensor", "autograd", "functional", "nn", "optim", "data", "datasets", "text", "testing", "cuda", "runtime",
    "compile", "config", "serialization", "serve", "cli", "benchmarks", "diagnostics", "native", "distributed",
    "train",
)

_this = sys.modules[__name__]
for _name in _SUBMODULES:
    _mod = importlib.import_module(f"underhfs_b200.{_name}")
    sys.modules[f"{__name__}.{_name}"] = _mod
    if not hasattr(_this, _name):
        setattr(_this, _name, _mod)
_this.tensor = _impl.tensor


def __getattr__(name):
    if name == "_core":
        from underhfs_b200.ops._lib import core

        return core()
    return getattr(_impl, name)
