"""In-tree build of the native library and its torch shim.

Produces, next to this file:

* ``libbysj_b200.so`` -- every CUDA kernel plus the C ABI declared in
  ``include/bysj_b200.h``; compiled by nvcc for sm_100a only
  (``-gencode arch=compute_100a,code=sm_100a -lineinfo``), with the CUDA
  runtime linked statically so the library has no dependency on a particular
  ``libcudart`` and loads on a host without a GPU.
* ``_C<ext-suffix>`` -- the pybind11 torch extension (``torch_bindings.cpp``)
  that keeps the Python names of the reference's ``kernels._C`` module and
  links against ``libbysj_b200.so`` through ``$ORIGIN``.

Run ``python -m bysj_b200._build`` (or ``__graft_entry__.build()``).  Object
files go to ``_build/`` at the repository root; rebuilding is incremental on
source timestamps.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
import sysconfig
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent
CSRC = PACKAGE / "csrc"
INCLUDE = ROOT / "include"
BUILD = ROOT / "_build"
LIBRARY = PACKAGE / "libbysj_b200.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
]
CU_SOURCES = [
    "runtime.cu",
    "offsets.cu",
    "group.cu",
    "segment_sum.cu",
    "segment_softmax.cu",
    "segment_attention.cu",
    "force_assembly.cu",
    "rmsnorm.cu",
    "gie.cu",
    "rotate_aggregate.cu",
    "edge_chain.cu",
    "checks.cu",
]
HEADERS = ["common.cuh", "launch.cuh"]


def _nvcc() -> str:
    home = os.environ.get("CUDA_HOME") or "/usr/local/cuda"
    candidate = Path(home) / "bin" / "nvcc"
    if candidate.exists():
        return str(candidate)
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found: set CUDA_HOME or put nvcc on PATH")
    return found


def _cuda_include() -> str:
    return str(Path(_nvcc()).resolve().parent.parent / "include")


def extension_path() -> Path:
    return PACKAGE / ("_C" + sysconfig.get_config_var("EXT_SUFFIX"))


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(Path(d).stat().st_mtime > t for d in deps)


def _run(cmd, verbose):
    if verbose:
        print("[build] " + " ".join(str(c) for c in cmd), flush=True)
    proc = subprocess.run([str(c) for c in cmd], capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(
            f"command failed ({proc.returncode}): {' '.join(map(str, cmd))}\n"
            f"{proc.stdout}\n{proc.stderr}"
        )
    return proc


def _headers():
    return [CSRC / h for h in HEADERS] + [INCLUDE / "bysj_b200.h"]


def build_library(verbose: bool = True) -> Path:
    """Compile every .cu file for sm_100a and link libbysj_b200.so."""
    BUILD.mkdir(exist_ok=True)
    nvcc = _nvcc()
    objects = []
    jobs = []
    for name in CU_SOURCES:
        src = CSRC / name
        obj = BUILD / (name + ".o")
        objects.append(obj)
        if _stale(obj, [src, *_headers()]):
            jobs.append([nvcc, *ARCH_FLAGS, *NVCC_FLAGS, "-I", INCLUDE, "-c", src, "-o", obj])
    if jobs:
        with ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as pool:
            list(pool.map(lambda c: _run(c, verbose), jobs))
    if jobs or _stale(LIBRARY, objects):
        _run(
            [nvcc, *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", LIBRARY, *objects],
            verbose,
        )
    return LIBRARY


def build_extension(verbose: bool = True) -> Path:
    """Compile the pybind11 shim against torch and link it to the library."""
    import torch
    from torch.utils import cpp_extension

    target = extension_path()
    src = CSRC / "torch_bindings.cpp"
    if not _stale(target, [src, LIBRARY, INCLUDE / "bysj_b200.h"]):
        return target
    includes = cpp_extension.include_paths() + [
        sysconfig.get_paths()["include"],
        _cuda_include(),
    ]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    libdirs = cpp_extension.library_paths()
    cmd = [
        os.environ.get("CXX", "g++"),
        "-O2",
        "-std=c++17",
        "-fPIC",
        "-shared",
        f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
        "-DTORCH_EXTENSION_NAME=_C",
        "-DTORCH_API_INCLUDE_EXTENSION_H",
        *[f"-I{p}" for p in includes],
        str(src),
        "-o",
        str(target),
        *[f"-L{p}" for p in libdirs],
        "-lc10",
        "-lc10_cuda",
        "-ltorch",
        "-ltorch_cpu",
        "-ltorch_cuda",
        "-ltorch_python",
        f"-L{PACKAGE}",
        "-lbysj_b200",
        "-Wl,-rpath,$ORIGIN",
        *[f"-Wl,-rpath,{p}" for p in libdirs],
    ]
    _run(cmd, verbose)
    return target


def build(verbose: bool = True) -> None:
    build_library(verbose)
    build_extension(verbose)


def clean() -> None:
    for path in (LIBRARY, extension_path()):
        if path.exists():
            path.unlink()
    if BUILD.exists():
        shutil.rmtree(BUILD)


if __name__ == "__main__":
    if "--clean" in sys.argv:
        clean()
    build(verbose="-q" not in sys.argv)
