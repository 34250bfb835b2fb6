"""Build the native core ``underhfs_b200._core`` for sm_100a.

Replaces the reference's CMake build (CMakeLists.txt:1-57, default
``CMAKE_CUDA_ARCHITECTURES 89``).  This driver writes a ninja file and builds
every translation unit under ``csrc/`` in parallel:

* ``.cu`` files with ``nvcc -gencode arch=compute_100a,code=sm_100a -lineinfo``
  (CUDA runtime linked statically, so the extension does not depend on the
  CUDA runtime version PyTorch ships);
* ``.cpp`` files (pybind11 bindings) with the host C++ compiler;
* one shared object placed next to this file, so it travels with the source
  tree and is the module every ``import underhfs_b200`` loads.

Usage: ``python -m underhfs_b200._native_build [--verbose] [--clean]``.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = ROOT / "csrc"
BUILD = ROOT / "build" / "native"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _on(name: str, default: str = "ON") -> bool:
    """Build option from the environment: ON/1/TRUE/YES (any case) is on."""
    return os.environ.get(name, default).strip().upper() in ("ON", "1", "TRUE", "YES")


def options() -> dict[str, bool]:
    """The build options, named like the reference's CMake options
    (CMakeLists.txt:4-6) but on by default, since this framework exists for
    the GPU:

    * ``UNDERHFS_WITH_CUDA`` -- build the native core at all (OFF: a pure
      Python install whose CPU paths run on torch; ``native.probe()``
      reports the core as unavailable);
    * ``UNDERHFS_WITH_NCCL`` -- link NCCL for ``NcclProcessGroup`` (OFF: the
      class raises, ``nccl_enabled`` is False; the NVLink comm kernels do not
      need NCCL and stay);
    * ``UNDERHFS_WITH_CUDNN`` -- expose the conv2d entry points (this
      framework's own implicit-GEMM kernels, not cuDNN; the name is kept for
      build-script compatibility).  OFF: ``cudnn_enabled`` is False.
    """
    return {"cuda": _on("UNDERHFS_WITH_CUDA"), "nccl": _on("UNDERHFS_WITH_NCCL"), "cudnn": _on("UNDERHFS_WITH_CUDNN")}


def _option_flags() -> str:
    opt = options()
    return ("" if opt["nccl"] else "-DUHFS_NO_NCCL ") + ("" if opt["cudnn"] else "-DUHFS_NO_CONV ")


def _check_flags() -> str:
    """Optional debug builds.  UNDERHFS_KERNEL_CHECKS=1 compiles the kernels' debug index checks in
    (UHFS_CHECK in csrc/kernels/common.cuh); a failed check is reported in the
    device status word and the access is skipped, never a trap."""
    flags = "-DUHFS_KERNEL_CHECKS " if os.environ.get("UNDERHFS_KERNEL_CHECKS", "0") == "1" else ""
    # UNDERHFS_ATTN_TRACE=1: per-step clock64 stamps in the attention kernels
    # (kernel_cases attn_fwd / attn_bwd --trace); never in the product build
    if os.environ.get("UNDERHFS_ATTN_TRACE", "0") == "1":
        flags += "-DUHFS_ATTN_TRACE "
    # UNDERHFS_GEMM_TRACE=1: per-unit clock64 stamps in the single-CTA GEMM
    # (kernel_cases <gemm case> --trace); never in the product build
    if os.environ.get("UNDERHFS_GEMM_TRACE", "0") == "1":
        flags += "-DUHFS_GEMM_TRACE "
    return flags + _option_flags()


def _pybind11_include() -> str:
    import pybind11

    return pybind11.get_include()


def _nccl_paths() -> tuple[str, str]:
    """Return (include_dir, lib_dir) of the NCCL that PyTorch loads at runtime."""
    try:
        import nvidia.nccl  # type: ignore

        base = Path(list(nvidia.nccl.__path__)[0])
        inc, lib = base / "include", base / "lib"
        if (lib / "libnccl.so.2").exists():
            return (str(inc) if (inc / "nccl.h").exists() else "/usr/include"), str(lib)
    except Exception:
        pass
    return "/usr/include", "/usr/lib/x86_64-linux-gnu"


def output_path() -> Path:
    return PKG / ("_core" + sysconfig.get_config_var("EXT_SUFFIX"))


def sources() -> list[Path]:
    out = sorted((CSRC / "kernels").glob("*.cu")) + sorted((CSRC / "runtime").glob("*.cu"))
    out += sorted((CSRC / "runtime").glob("*.cpp")) + [CSRC / "bindings.cpp"]
    return out


def _ninja_file() -> str:
    py_inc = sysconfig.get_paths()["include"]
    nccl_inc, nccl_lib = _nccl_paths()
    incs = f"-I{CSRC} -I{CUDA_HOME / 'include'} -I{py_inc} -I{_pybind11_include()} -I{nccl_inc}"
    nvcc = CUDA_HOME / "bin" / "nvcc"
    cxx = os.environ.get("CXX", "g++")
    lines = [
        "ninja_required_version = 1.3",
        f"nvcc = {nvcc}",
        f"cxx = {cxx}",
        f"nvflags = {' '.join(ARCH_FLAGS)} -lineinfo -O3 -std=c++17 --expt-relaxed-constexpr {_check_flags()}"
        f"-Xcompiler -fPIC -Xcompiler -fvisibility=hidden -DNDEBUG {incs}",
        f"cxxflags = -O2 -std=c++17 -fPIC -fvisibility=hidden -DNDEBUG {_option_flags()}{incs}",
        f"ldflags = -shared {' '.join(ARCH_FLAGS)} "
        + (f"-L{nccl_lib} -l:libnccl.so.2 -Xlinker -rpath,{nccl_lib} " if options()["nccl"] else "")
        + "-lpthread",
        "rule nvcc",
        "  command = $nvcc $nvflags -MD -MF $out.d -c $in -o $out",
        "  depfile = $out.d",
        "  deps = gcc",
        "  description = NVCC $in",
        "rule cxx",
        "  command = $cxx $cxxflags -MD -MF $out.d -c $in -o $out",
        "  depfile = $out.d",
        "  deps = gcc",
        "  description = CXX $in",
        "rule link",
        "  command = $nvcc $in -o $out $ldflags",
        "  description = LINK $out",
    ]
    objs = []
    for src in sources():
        rel = src.relative_to(CSRC)
        obj = BUILD / (str(rel).replace("/", "__") + ".o")
        rule = "nvcc" if src.suffix == ".cu" else "cxx"
        lines.append(f"build {obj}: {rule} {src}")
        objs.append(str(obj))
    lines.append(f"build {output_path()}: link {' '.join(objs)}")
    # native JSON-lines server (serve.CppJsonPredictServer)
    lines += [
        "rule cxxexe",
        "  command = $cxx -O2 -std=c++17 $in -o $out",
        "  description = CXX-EXE $out",
        f"build {serve_exe_path()}: cxxexe {CSRC / 'serve' / 'serve_main.cpp'}",
    ]
    lines.append(f"default {output_path()} {serve_exe_path()}")
    return "\n".join(lines) + "\n"


def serve_exe_path() -> Path:
    return PKG / "bin" / "underhfs_cpp_serve"


def build(verbose: bool = False, jobs: int | None = None) -> Path | None:
    """Compile and link the native core; returns the path of the built module
    (None with UNDERHFS_WITH_CUDA=OFF, which builds nothing)."""
    if not options()["cuda"]:
        return None
    BUILD.mkdir(parents=True, exist_ok=True)
    ninja_path = BUILD / "build.ninja"
    content = _ninja_file()
    if not ninja_path.exists() or ninja_path.read_text() != content:
        ninja_path.write_text(content)
    ninja = shutil.which("ninja")
    if ninja is None:
        try:
            import ninja as _ninja  # type: ignore

            ninja = str(Path(_ninja.BIN_DIR) / "ninja")
        except Exception as exc:  # pragma: no cover - environment dependent
            raise RuntimeError("ninja is required to build the native core") from exc
    cmd = [ninja, "-C", str(BUILD), "-f", "build.ninja"]
    if jobs:
        cmd += ["-j", str(jobs)]
    if verbose:
        cmd.append("-v")
    proc = subprocess.run(cmd, capture_output=not verbose, text=True)
    if proc.returncode != 0:
        out = (proc.stdout or "") + (proc.stderr or "")
        raise RuntimeError(f"native build failed:\n{out[-20000:]}")
    return output_path()


def clean() -> None:
    if BUILD.exists():
        shutil.rmtree(BUILD)
    out = output_path()
    if out.exists():
        out.unlink()


if __name__ == "__main__":
    if "--clean" in sys.argv:
        clean()
    path = build(verbose="--verbose" in sys.argv)
    print(path)
