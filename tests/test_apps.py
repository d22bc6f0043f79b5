"""The host C++ on top of the C ABI, without a GPU: the nnml operator shim
(libalb_nnml_ops.so) loads and exports its operators and rejects bad calls
before touching the device; the al_bench driver parses its arguments and
reports a missing device instead of running."""
import ctypes as C
import os
import subprocess

import pytest

import arclight_b200 as A
from arclight_b200 import build as B

SHIM_OPS = ["nnml_gpu_forward_mul_mat", "nnml_gpu_forward_rms_norm_mul", "nnml_gpu_forward_get_rows",
            "nnml_gpu_forward_set_rows",
            "nnml_gpu_forward_swiglu", "nnml_gpu_forward_flash_attn_ext", "nnml_gpu_sample_greedy"]


class Tensor(C.Structure):
    pass


Tensor._fields_ = [("ne", C.c_int64 * 4), ("nb", C.c_size_t * 4), ("data", C.c_void_p),
                   ("op_params", C.c_int32 * 16), ("src", C.POINTER(Tensor) * 4)]


class State(C.Structure):
    _fields_ = [("ith", C.c_int32), ("nth", C.c_int32), ("stream", C.c_void_p), ("xq", C.c_void_p),
                ("xq_bytes", C.c_size_t), ("attn_ws", C.c_void_p), ("attn_ws_bytes", C.c_size_t)]


def shim():
    A.lib()   # the shim links against libalb_cuda.so next to it
    return C.CDLL(B.SHIM)


def test_apps_are_built():
    B.build()
    assert os.path.exists(B.SHIM) and os.path.exists(B.AL_BENCH)


def test_shim_exports_and_rejects_bad_calls():
    L = shim()
    for name in SHIM_OPS:
        f = getattr(L, name)
        f.restype = C.c_int
        f.argtypes = [C.c_void_p, C.c_void_p]
        assert f(None, None) == -1, name                       # ALB_ERR_INVALID
        t = Tensor()
        st = State(ith=1, nth=8)
        assert f(C.byref(st), C.byref(t)) == 0, name           # not thread 0: nothing to do
        st0 = State(ith=0, nth=8)
        assert f(C.byref(st0), C.byref(t)) == -1, name         # thread 0, no operands: rejected on the host


def test_al_bench_arguments():
    r = subprocess.run([B.AL_BENCH, "--bogus"], capture_output=True, text=True)
    assert r.returncode == 2 and "usage" in r.stderr
    r = subprocess.run([B.AL_BENCH, "--model", "nope"], capture_output=True, text=True)
    assert r.returncode == 2


def test_al_bench_rejects_bad_gguf(tmp_path):
    # the file is read before any device is touched
    r = subprocess.run([B.AL_BENCH, "--gguf", str(tmp_path / "missing.gguf")], capture_output=True, text=True)
    assert r.returncode == 1 and "cannot open" in r.stderr
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"NOPE" + bytes(64))
    r = subprocess.run([B.AL_BENCH, "--gguf", str(bad)], capture_output=True, text=True)
    assert r.returncode == 1 and "not a GGUF file" in r.stderr


def test_al_bench_reports_missing_device():
    if A.lib().alb_device_check(0) == 0:
        pytest.skip("a B200 is present (the GPU tests run the driver)")
    r = subprocess.run([B.AL_BENCH, "--model", "tiny", "--prompt", "8", "--max_gen", "2"], capture_output=True,
                       text=True)
    assert r.returncode == 1 and "device 0" in r.stderr
