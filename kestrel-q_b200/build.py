"""Builds the B200 C-ABI library ``kestrel-q_b200/lib/libkqb200.so``.

Every translation unit is compiled by nvcc for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``); host files are compiled as CUDA
too so they can share the device headers.  Host code is built with
``-ffp-contract=off`` so the RoPE table it computes uses the same rounding as
the reference's scalar C.  The CUDA runtime is linked statically and its
symbols are kept private to the library: only ``kq_*`` is exported
(csrc/exports.map).

Usage: python kestrel-q_b200/build.py [--force]
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parent
CSRC = HERE / "csrc"
BUILD = HERE / "_build"
LIB = HERE / "lib" / "libkqb200.so"

SOURCES = [
    "kernels_proj.cu",
    "kernels_gdn.cu",
    "kernels_gdn_chunk.cu",
    "kernels_qsa.cu",
    "kernels_umma.cu",
    "kernels_moe.cu",
    "kernels_layer.cu",
    "runtime.cpp",
    "api_basic.cpp",
    "api_provider.cpp",
    "api_gdn.cpp",
    "api_qsa.cpp",
    "api_moe.cpp",
    "api_layer.cpp",
    "api_static.cu",
]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-ffp-contract=off",
    f"-I{REPO / 'include'}", f"-I{CSRC}",
]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: the B200 library has no CPU build")
    return cand


def _compile(src: str, force: bool) -> Path:
    obj = BUILD / (src + ".o")
    path = CSRC / src
    deps = [path] + list(CSRC.glob("*.hpp")) + list(CSRC.glob("*.cuh")) + list((REPO / "include").glob("*.h"))
    if not force and obj.exists() and obj.stat().st_mtime >= max(d.stat().st_mtime for d in deps):
        return obj
    cmd = [nvcc(), *ARCH, *COMMON, "-x", "cu", "-c", str(path), "-o", str(obj)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{res.stdout}\n{res.stderr}")
    return obj


def build(force: bool = False) -> Path:
    BUILD.mkdir(parents=True, exist_ok=True)
    LIB.parent.mkdir(parents=True, exist_ok=True)
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as pool:
        objs = list(pool.map(lambda s: _compile(s, force), SOURCES))
    if force or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(LIB), *map(str, objs),
               "-Xlinker", "--exclude-libs,ALL", "-Xlinker", f"--version-script={CSRC / 'exports.map'}",
               "-Xcompiler", "-fPIC"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
