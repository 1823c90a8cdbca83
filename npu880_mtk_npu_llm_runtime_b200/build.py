"""Build libkq.so (the C ABI of include/kq.h) in-tree with nvcc for sm_100a.

The library is plain CUDA C++ with the CUDA runtime linked statically; it has no dependency
on PyTorch.  Each source compiles to its own object (in parallel, into _build/, reused while
it is newer than the sources and headers), then nvcc links the shared library.
Usage:  python -m npu880_mtk_npu_llm_runtime_b200.build  [--force]
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIB = os.path.join(PKG, "libkq.so")
OBJ_DIR = os.path.join(ROOT, "_build", "kq")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo", *ARCH,
    "-Xcompiler", "-fPIC",
    "--expt-relaxed-constexpr",
    "-I", os.path.join(ROOT, "include"),
]


def nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def headers() -> list[str]:
    return (glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h"))
            + [os.path.join(ROOT, "include", "kq.h")])


def _obj(src: str) -> str:
    return os.path.join(OBJ_DIR, os.path.basename(src)[:-3] + ".o")


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def needs_build() -> bool:
    return _stale(LIB, sources() + headers())


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not needs_build():
        return LIB
    os.makedirs(OBJ_DIR, exist_ok=True)
    hdr = headers()
    todo = [s for s in sources() if force or _stale(_obj(s), [s, *hdr])]

    def compile_one(src: str):
        cmd = [nvcc(), *NVCC_FLAGS, "-c", "-o", _obj(src) + ".tmp", src]
        if verbose:
            print(" ".join(cmd), flush=True)
        out = subprocess.run(cmd, capture_output=True, text=True)
        if out.returncode != 0:
            return src, out.stdout + out.stderr
        os.replace(_obj(src) + ".tmp", _obj(src))
        return src, None

    with ThreadPoolExecutor(max_workers=max(1, min(len(todo), os.cpu_count() or 4))) as ex:
        errors = [(s, e) for s, e in ex.map(compile_one, todo) if e]
    if errors:
        raise RuntimeError("nvcc failed:\n" + "\n".join(f"{s}:\n{e}" for s, e in errors))
    tmp = LIB + ".tmp"
    cmd = [nvcc(), *ARCH, "-shared", "-o", tmp, *[_obj(s) for s in sources()]]
    if verbose:
        print(" ".join(cmd), flush=True)
    out = subprocess.run(cmd, capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError("nvcc link failed:\n" + out.stdout + out.stderr)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
