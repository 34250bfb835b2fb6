"""Packaging hook: the wheel carries the native core built for sm_100a.

``pip install --no-build-isolation .`` runs ``build_py`` below, which first
builds ``underhfs_b200/_core*.so`` and the native serving executable with the
in-tree ninja driver (``underhfs_b200/_native_build.py``), then copies them
as package data.  Build options are environment variables with the names of
the reference's CMake options: ``UNDERHFS_WITH_CUDA`` (OFF: pure-Python
install), ``UNDERHFS_WITH_NCCL`` and ``UNDERHFS_WITH_CUDNN``; all default ON.
"""

import importlib.util
from pathlib import Path

from setuptools import setup
from setuptools.command.build_py import build_py

ROOT = Path(__file__).resolve().parent


def _native_build_module():
    # load the build driver by path: importing the package would import torch
    # and the (not yet built) extension
    spec = importlib.util.spec_from_file_location("_uhfs_native_build", ROOT / "underhfs_b200" / "_native_build.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


class BuildWithNative(build_py):
    def run(self):
        nb = _native_build_module()
        out = nb.build()
        self.announce(f"native core: {out if out is not None else 'not built (UNDERHFS_WITH_CUDA=OFF)'}", level=2)
        super().run()


setup(cmdclass={"build_py": BuildWithNative})
