"""Build libapk.so (in-tree) for sm_100a with nvcc.

    python -m apk_b200.build            # incremental
    python -m apk_b200.build --force

Every CUDA translation unit is compiled with
``-gencode arch=compute_100a,code=sm_100a -lineinfo``; the shared library
links the CUDA runtime statically, and reaches the driver API
(cuTensorMapEncodeTiled) through cudaGetDriverEntryPointByVersion, so it
loads on a machine without a GPU driver (symbol checks run there).
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libapk.so")

SOURCES = ["sgemm_f32.cu", "sgemm_f32_ws.cu", "gemm_bf16.cu", "gemm_bf16_pair.cu", "visibility.cu", "runtime.cu",
           "datagen.cpp"]
HEADERS = ["common.cuh", "proto.h", "tcgen05.cuh"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _host_compiler() -> list[str]:
    # the image exports CC/CXX pointing at a gcc without libgomp; nvcc picks
    # the first g++ on PATH, pin the system one when it exists
    return ["-ccbin", "/usr/bin/g++"] if os.path.exists("/usr/bin/g++") else []


def _deps_mtime() -> float:
    paths = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(ROOT, "include", "apk.h")]
    return max((os.path.getmtime(p) for p in paths if os.path.exists(p)), default=0.0)


def _compile(src: str, force: bool) -> str:
    obj = os.path.join(BUILD, src + ".o")
    sp = os.path.join(CSRC, src)
    if not force and os.path.exists(obj):
        if os.path.getmtime(obj) >= max(os.path.getmtime(sp), _deps_mtime()):
            return obj
    cmd = [nvcc(), *_host_compiler(), "-std=c++17", "-O3", "-lineinfo", *ARCH,
           "-Xcompiler", "-fPIC", "-Xcompiler", "-ffp-contract=off",
           "-I", os.path.join(ROOT, "include"), "-c", sp, "-o", obj]
    if src.endswith(".cu"):
        cmd[1:1] = ["-x", "cu"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return obj


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    with cf.ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        objs = list(ex.map(lambda s: _compile(s, force), SOURCES))
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= max(os.path.getmtime(o) for o in objs):
        return LIB
    tmp = LIB + ".tmp"
    cmd = [nvcc(), *_host_compiler(), *ARCH, "-shared", "-cudart", "static", "-o", tmp, *objs,
           "-lpthread", "-ldl", "-lrt"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    if verbose:
        print(f"built {LIB}")
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
