"""Build the in-tree CUDA library ``fxpr_vllm/_lib/libfxpr_b200.so`` for sm_100a.

Plain nvcc (no torch headers): the library is a C ABI (``include/fxpr_b200.h``)
loaded with ctypes. Objects are compiled in parallel and cached by source
hash under ``_build/``; the shared object is only relinked when an object
changed.

    python fixed-point-reductions-for-vllm_b200/build.py [--force]
"""

from __future__ import annotations

import concurrent.futures as cf
import hashlib
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(HERE, "_build")
OUT_DIR = os.path.join(HERE, "fxpr_vllm", "_lib")
LIB = os.path.join(OUT_DIR, "libfxpr_b200.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-std=c++17", "-lineinfo",
    "--fmad=false",  # no contraction of separately rounded multiply/add
    "-Xcompiler", "-fPIC",
]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found")
    return cand


def _sources() -> list[str]:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _digest(src: str) -> str:
    h = hashlib.sha256()
    h.update(" ".join(NVCC_FLAGS).encode())
    for f in [src] + sorted(
        os.path.join(d, f) for d in (CSRC, INCLUDE) for f in os.listdir(d)
        if f.endswith((".cuh", ".h"))
    ):
        with open(f, "rb") as fh:
            h.update(fh.read())
    return h.hexdigest()[:16]


def _compile(src: str) -> tuple[str, bool]:
    base = os.path.splitext(os.path.basename(src))[0]
    obj = os.path.join(BUILD, f"{base}.{_digest(src)}.o")
    if os.path.exists(obj):
        return obj, False
    for f in os.listdir(BUILD):  # drop stale objects of this source
        if f.startswith(base + ".") and f.endswith(".o"):
            os.remove(os.path.join(BUILD, f))
    cmd = [_nvcc(), *NVCC_FLAGS, "-I", INCLUDE, "-c", src, "-o", obj + ".tmp"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    os.replace(obj + ".tmp", obj)
    return obj, True


def build(force: bool = False, verbose: bool = True) -> str:
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(OUT_DIR, exist_ok=True)
    if force:
        for f in os.listdir(BUILD):
            os.remove(os.path.join(BUILD, f))
    srcs = _sources()
    with cf.ThreadPoolExecutor(max_workers=min(len(srcs), os.cpu_count() or 4)) as ex:
        results = list(ex.map(_compile, srcs))
    objs = [o for o, _ in results]
    changed = any(c for _, c in results)
    if changed or not os.path.exists(LIB):
        cmd = [_nvcc(), "-shared", "-o", LIB + ".tmp", *objs, "-lcudart"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(LIB + ".tmp", LIB)
        if verbose:
            print(f"built {LIB}")
    elif verbose:
        print(f"up to date: {LIB}")
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv)
