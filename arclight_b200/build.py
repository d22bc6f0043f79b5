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
APPS = os.path.join(PKG, "apps")
SHIM = os.path.join(PKG, "libalb_nnml_ops.so")      # nnml-shaped operator shim over the C ABI
AL_BENCH = os.path.join(PKG, "al_bench")            # C++ driver of the engine (al-gen's flow)
CXX = os.environ.get("CXX", shutil.which("g++") or "g++")
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
    if not (os.path.exists(LIB) and os.path.getmtime(LIB) > max(os.path.getmtime(o) for o in objs)):
        cmd = [NVCC, *ARCH, "-shared", "-o", LIB, *objs, "-lcuda", "-ldl", "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n" + r.stderr)
        if verbose:
            print("built", LIB)
    build_apps(verbose)
    return LIB


def _stale(out: str, deps) -> bool:
    return not os.path.exists(out) or os.path.getmtime(out) < max(os.path.getmtime(d) for d in deps)


def build_apps(verbose: bool = False) -> None:
    """Host C++ on top of the C ABI: the nnml operator shim (a shared library)
    and the al_bench driver, both linked against the in-tree libalb_cuda.so."""
    inc = ["-I" + os.path.join(ROOT, "include"), "-I" + APPS]
    link = ["-L" + PKG, "-lalb_cuda", "-Wl,-rpath,$ORIGIN"]
    hdr = os.path.join(ROOT, "include", "alb_cuda.h")
    shim_src = [os.path.join(APPS, "nnml_gpu_ops.cpp"), os.path.join(APPS, "nnml_gpu_ops.h")]
    if _stale(SHIM, shim_src + [hdr, LIB]):
        cmd = [CXX, "-O2", "-std=c++17", "-fPIC", "-shared", "-fvisibility=hidden", *inc, shim_src[0], "-o", SHIM, *link]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("nnml shim build failed:\n" + r.stderr)
        if verbose:
            print("built", SHIM)
    bench_src = os.path.join(APPS, "al_bench.cpp")
    if _stale(AL_BENCH, [bench_src, hdr, LIB]):
        cmd = [CXX, "-O2", "-std=c++17", "-pthread", *inc, bench_src, "-o", AL_BENCH, *link]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("al_bench build failed:\n" + r.stderr)
        if verbose:
            print("built", AL_BENCH)


if __name__ == "__main__":
    if "--clean" in sys.argv:
        shutil.rmtree(OBJ, ignore_errors=True)
        for f in (LIB, SHIM, AL_BENCH):
            if os.path.exists(f):
                os.remove(f)
    build(verbose=True)
