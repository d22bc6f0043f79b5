"""Build libalb_cuda.so in-tree with nvcc for sm_100a (no GPU needed).

    python -m arclight_b200.build          # incremental
    python -m arclight_b200.build --clean
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
OBJ = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libalb_cuda.so")
NVCC = os.environ.get("NVCC", shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-I" + os.path.join(ROOT, "include"), "-I" + CSRC]


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cpp")))


def headers_mtime():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hs += [os.path.join(ROOT, "include", f) for f in os.listdir(os.path.join(ROOT, "include"))]
    return max(os.path.getmtime(h) for h in hs)


def compile_one(src: str, hdr_t: float) -> str:
    obj = os.path.join(OBJ, os.path.basename(src) + ".o")
    if os.path.exists(obj) and os.path.getmtime(obj) > max(os.path.getmtime(src), hdr_t):
        return obj
    cmd = [NVCC, *ARCH, *FLAGS, "-c", src, "-o", obj]
    if src.endswith(".cpp"):
        cmd = [NVCC, "-x", "cu", *ARCH, *FLAGS, "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{r.stderr}")
    return obj


def build(verbose: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    hdr_t = headers_mtime()
    srcs = sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: compile_one(s, hdr_t), srcs))
    if os.path.exists(LIB) and os.path.getmtime(LIB) > max(os.path.getmtime(o) for o in objs):
        return LIB
    cmd = [NVCC, *ARCH, "-shared", "-o", LIB, *objs, "-lcuda", "-ldl", "-lpthread"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("link failed:\n" + r.stderr)
    if verbose:
        print("built", LIB)
    return LIB


if __name__ == "__main__":
    if "--clean" in sys.argv:
        shutil.rmtree(OBJ, ignore_errors=True)
        if os.path.exists(LIB):
            os.remove(LIB)
    build(verbose=True)
