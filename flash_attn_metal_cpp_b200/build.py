"""Ahead-of-time build of the B200 attention library.

Produces, inside this package directory:
  libfa_b200.so                     C ABI (include/fa_b200.h): kernels + host dispatcher
  _flash_attn_metal.<abi>.so        pybind11 module over that C ABI

Every CUDA translation unit is compiled for sm_100a only
(-gencode arch=compute_100a,code=sm_100a). Objects are compiled in
parallel into _build/ and relinked only when a source is newer than the
library. Run as `python flash_attn_metal_cpp_b200/build.py [--force]`.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys
import sysconfig

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
OBJDIR = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libfa_b200.so")
EXT = os.path.join(PKG, "_flash_attn_metal" + sysconfig.get_config_var("EXT_SUFFIX"))

CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr"] + ARCH

CU_SOURCES = [
    "fa_api.cu",
    "fa_aux.cu",
    "fa_host.cu",
    "fa_fwd_simt.cu",
    "fa_fwd_sm100.cu",
    "fa_fwd_sm100_d64_causal.cu",
    "fa_fwd_sm100_d64_full.cu",
    "fa_fwd_sm100_d128_causal.cu",
    "fa_fwd_sm100_d128_full.cu",
]
HEADERS = ["fa_internal.h", "fa_ptx.cuh", "fa_fwd_sm100.cuh", "fa_host.h"]


def _mtime(path: str) -> float:
    return os.path.getmtime(path) if os.path.exists(path) else -1.0


def _run(cmd: list[str]) -> None:
    proc = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"build step failed: {' '.join(cmd)}\n{proc.stdout}")


def _header_mtime() -> float:
    hs = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(INCLUDE, "fa_b200.h")]
    return max(_mtime(h) for h in hs)


def _compile(src: str, force: bool) -> str:
    obj = os.path.join(OBJDIR, os.path.splitext(src)[0] + ".o")
    path = os.path.join(CSRC, src)
    if force or _mtime(obj) < max(_mtime(path), _header_mtime()):
        _run([NVCC, *NVCC_FLAGS, "-I", INCLUDE, "-c", path, "-o", obj])
    return obj


def build(force: bool = False, jobs: int | None = None) -> tuple[str, str]:
    """Compile the CUDA library and the Python extension; return their paths."""
    if not os.path.exists(NVCC):
        raise RuntimeError(f"nvcc not found at {NVCC}")
    os.makedirs(OBJDIR, exist_ok=True)
    jobs = jobs or max(1, min(len(CU_SOURCES), os.cpu_count() or 1))
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        objs = list(ex.map(lambda s: _compile(s, force), CU_SOURCES))
    if force or _mtime(LIB) < max(_mtime(o) for o in objs):
        _run([NVCC, *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", LIB, *objs])

    bsrc = os.path.join(CSRC, "bindings.cpp")
    if force or _mtime(EXT) < max(_mtime(bsrc), _mtime(LIB), _mtime(os.path.join(INCLUDE, "fa_b200.h"))):
        import pybind11

        py_inc = sysconfig.get_paths()["include"]
        _run([
            "g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-fvisibility=hidden",
            "-I", pybind11.get_include(), "-I", py_inc, "-I", INCLUDE,
            bsrc, "-o", EXT, "-L", PKG, "-l:libfa_b200.so", "-Wl,-rpath,$ORIGIN",
        ])
    return LIB, EXT


if __name__ == "__main__":
    lib, ext = build(force="--force" in sys.argv)
    print(lib)
    print(ext)
