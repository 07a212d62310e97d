"""Builds the in-tree C-ABI library ``sglite_b200/lib/libawqb200.so`` with nvcc.

Every CUDA source is compiled for sm_100a only (``-gencode
arch=compute_100a,code=sm_100a``); object files go to ``_build/`` at the repo
root and are relinked when a source or header changes.
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
import sysconfig

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
INCLUDE = os.path.join(REPO_DIR, "include")
BUILD_DIR = os.path.join(REPO_DIR, "_build")
LIB_DIR = os.path.join(PKG_DIR, "lib")
LIB_PATH = os.path.join(LIB_DIR, "libawqb200.so")

SOURCES = [
    "awqb_common.cpp",
    "awqb_repack.cu",
    "awqb_gemm.cu",
    "awqb_moe.cu",
    "awqb_norm.cu",
    "awqb_nccl.cpp",
]

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3", "-I", INCLUDE, "-I", CSRC]


def _nccl_dirs() -> tuple[str, str]:
    """Include and library directory of the NCCL that torch loads (same soname)."""
    site = sysconfig.get_paths()["purelib"]
    base = os.path.join(site, "nvidia", "nccl")
    if os.path.isfile(os.path.join(base, "include", "nccl.h")):
        return os.path.join(base, "include"), os.path.join(base, "lib")
    return "/usr/include", "/usr/lib/x86_64-linux-gnu"


def _nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the sm_100a library cannot be built")


def _headers() -> list[str]:
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hs.append(os.path.join(INCLUDE, "awqb200.h"))
    return hs


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def _compile(src: str, obj: str, nccl_inc: str) -> None:
    cmd = [_nvcc(), *ARCH_FLAGS, *NVCC_FLAGS, "-I", nccl_inc, "-c", src, "-o", obj]
    if src.endswith(".cpp"):
        cmd = [_nvcc(), "-x", "cu", *cmd[1:]]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{res.stderr}")


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile stale objects and relink the library; returns its path."""
    os.makedirs(BUILD_DIR, exist_ok=True)
    os.makedirs(LIB_DIR, exist_ok=True)
    nccl_inc, nccl_lib = _nccl_dirs()
    headers = _headers()
    jobs = []
    objs = []
    for name in SOURCES:
        src = os.path.join(CSRC, name)
        obj = os.path.join(BUILD_DIR, name + ".o")
        objs.append(obj)
        if force or _stale(obj, [src, *headers, __file__]):
            jobs.append((src, obj))
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            futs = [ex.submit(_compile, s, o, nccl_inc) for s, o in jobs]
            for f in futs:
                f.result()
    if force or jobs or _stale(LIB_PATH, objs):
        cmd = [
            _nvcc(), *ARCH_FLAGS, "-shared", "-cudart", "shared", "-o", LIB_PATH, *objs,
            "-L", nccl_lib, "-l:libnccl.so.2", "-Xlinker", f"-rpath,{nccl_lib}",
        ]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stderr}")
        if verbose:
            print("linked", LIB_PATH, file=sys.stderr)
    return LIB_PATH


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
