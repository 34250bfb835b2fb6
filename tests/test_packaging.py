"""Packaging surface: the console script, the package data and the build
options (named like the reference's CMake options, pyproject.toml:22-23 and
CMakeLists.txt:4-6 of the reference)."""

import tomllib
from pathlib import Path

from underhfs_b200 import _native_build

ROOT = Path(__file__).resolve().parents[1]


def test_console_script_and_package_data():
    cfg = tomllib.loads((ROOT / "pyproject.toml").read_text())
    assert cfg["project"]["scripts"]["underhfs"] == "underhfs_b200.cli:main"
    data = cfg["tool"]["setuptools"]["package-data"]["underhfs_b200"]
    assert "_core*.so" in data and "bin/underhfs_cpp_serve" in data


def test_build_options(monkeypatch):
    for name in ("UNDERHFS_WITH_CUDA", "UNDERHFS_WITH_NCCL", "UNDERHFS_WITH_CUDNN"):
        monkeypatch.delenv(name, raising=False)
    assert _native_build.options() == {"cuda": True, "nccl": True, "cudnn": True}
    assert _native_build._option_flags() == ""
    monkeypatch.setenv("UNDERHFS_WITH_NCCL", "OFF")
    monkeypatch.setenv("UNDERHFS_WITH_CUDNN", "off")
    assert "-DUHFS_NO_NCCL" in _native_build._option_flags()
    assert "-DUHFS_NO_CONV" in _native_build._option_flags()
    ninja = _native_build._ninja_file()
    assert "libnccl" not in ninja.split("ldflags = ", 1)[1].splitlines()[0]
    monkeypatch.setenv("UNDERHFS_WITH_CUDA", "OFF")
    assert _native_build.build() is None  # pure-Python install: nothing is built
