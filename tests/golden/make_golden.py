"""Generate the golden fixtures that pin oracle/oracle.c to the reference.

Runs the reference's OWN portable nnml code -- types.cpp, ops.cpp, binary.cpp,
common.cpp, tensor.cpp, memory.cpp compiled with an x86 shim by
``make -C oracle ref`` into ``oracle/_ref/libalref.so`` -- on seeded inputs, and
writes inputs + reference outputs to ``tests/golden/*.npz``.  The reference tree
is needed only here; the committed fixtures travel, the reference does not.

    make -C oracle ref && python tests/golden/make_golden.py
"""
import ctypes as C
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from oracle import lib as O  # noqa: E402


def p(a):
    return a.ctypes.data_as(C.c_void_p)


def main():
    R = O.ref_lib()
    if R is None:
        raise SystemExit("oracle/_ref/libalref.so missing: run `make -C oracle ref` where the reference exists")
    rng = np.random.default_rng(20240611)
    out = {}

    # fp16 conversions (ops.h:276-324): special values + random magnitudes
    f = np.concatenate([np.array([0.0, -0.0, 1.0, -1.0, 65504.0, 65520.0, 1e-8, 5.96e-8, 6.1e-5, 3.14159, np.inf, -np.inf],
                                 np.float32),
                        (rng.standard_normal(4000) * np.exp2(rng.integers(-26, 17, 4000))).astype(np.float32)])
    out["fp16_in"] = f
    out["fp16_out"] = np.array([R.ref_fp32_to_fp16(float(v)) for v in f], np.uint16)

    # Q4_0 quantize / dequantize (types.cpp:337-378); includes an all-zero block,
    # a negative-max block and exact-tie blocks
    x = (rng.standard_normal((16, 256)) * 0.02).astype(np.float32)
    x[0, :32] = 0.0
    x[1, :32] = -np.abs(x[1, :32]); x[1, 5] = -0.1
    x[2, :32] = np.arange(-16, 16, dtype=np.float32) / 8.0
    x[3, :32] = np.float32(0.5) * np.arange(32, dtype=np.float32) - 8.0
    q4 = np.empty(16 * 8, O.Q4_DTYPE)
    R.ref_quantize_row_q4_0(p(x), p(q4), x.size)
    dq4 = np.empty_like(x)
    R.ref_dequantize_row_q4_0(p(q4), p(dq4), x.size)
    out["q4_in"], out["q4_out"], out["q4_deq"] = x, q4.view(np.uint8), dq4

    # Q8_0 reference quantizer (types.cpp:494-514): ties, zero block, exact +/-127
    x8 = rng.standard_normal((8, 256)).astype(np.float32)
    x8[0, :32] = 0.0
    x8[1, :32] = np.arange(32, dtype=np.float32) - 16.0
    x8[2, :32] = (np.arange(32, dtype=np.float32) - 16.0) * np.float32(127.0 / 16.0)
    x8[3, :32] = np.linspace(-127, 127, 32).astype(np.float32) * np.float32(0.25)
    q8 = np.empty(8 * 8, O.Q8_DTYPE)
    R.ref_quantize_row_q8_0_ref(p(x8), p(q8), x8.size)
    dq8 = np.empty_like(x8)
    R.ref_dequantize_row_q8_0(p(q8), p(dq8), x8.size)
    out["q8_in"], out["q8_out"], out["q8_deq"] = x8, q8.view(np.uint8), dq8

    # repack<block_q4_0,4,4> (types.cpp:133-201)
    w = (rng.standard_normal((8, 128)) * 0.02).astype(np.float32)
    wq = np.empty(8 * 4, O.Q4_DTYPE)
    R.ref_quantize_row_q4_0(p(w), p(wq), w.size)
    rp = np.empty(8 * 4 * 18, np.uint8)
    assert R.ref_repack_q4_0_4x4(p(wq), p(rp), 8, 128) == 0
    out["repack_in"], out["repack_out"] = wq.view(np.uint8), rp

    # RMS_NORM + MUL (ops.cpp:680-724, binary.cpp): hidden rows and per-head rows
    xr = (rng.standard_normal((3, 2560)) * 3).astype(np.float32)
    wr = (1 + 0.01 * rng.standard_normal(2560)).astype(np.float32)
    yr = np.empty_like(xr)
    R.ref_rms_norm_mul(p(xr), p(wr), p(yr), 3, 2560, C.c_float(1e-6))
    xh = rng.standard_normal((40, 128)).astype(np.float32)
    wh = (1 + 0.01 * rng.standard_normal(128)).astype(np.float32)
    yh = np.empty_like(xh)
    R.ref_rms_norm_mul(p(xh), p(wh), p(yh), 40, 128, C.c_float(1e-6))
    out.update(rms_x=xr, rms_w=wr, rms_y=yr, rmsh_x=xh, rmsh_w=wh, rmsh_y=yh)

    # ROPE NEOX theta 1e6 (ops.cpp:747-961) at several positions incl. 32767
    pos = np.array([0, 1, 2, 17, 255, 1000, 4095, 32767], np.int32)
    xq = rng.standard_normal((pos.size, 4, 128)).astype(np.float32)
    yq = np.empty_like(xq)
    R.ref_rope_neox(p(xq), p(yq), 4, 128, pos.size, p(pos), C.c_float(1e6))
    out.update(rope_pos=pos, rope_x=xq, rope_y=yq)

    # GET_ROWS Q4_0 (ops.cpp:12-52)
    tab = np.empty(50 * 8, O.Q4_DTYPE)
    tw = (rng.standard_normal((50, 256)) * 0.02).astype(np.float32)
    R.ref_quantize_row_q4_0(p(tw), p(tab), tw.size)
    ids = np.array([0, 7, 49, 7, 23], np.int32)
    gr = np.empty((ids.size, 256), np.float32)
    R.ref_get_rows_q4_0(p(tab), 50, 256, p(ids), ids.size, p(gr))
    out.update(getrows_table=tab.view(np.uint8), getrows_ids=ids, getrows_out=gr)

    # SET_ROWS fp32 -> fp16 (ops.cpp:135-181)
    cache = np.zeros((16, 256), np.uint16)
    src = (rng.standard_normal((3, 256)) * 4).astype(np.float32)
    idx = np.array([5, 0, 15], np.int64)
    R.ref_set_rows_f16(p(cache), 16, 256, p(src), p(idx), 3)
    out.update(setrows_src=src, setrows_idx=idx, setrows_cache=cache)

    # ADD (binary.cpp)
    a = rng.standard_normal(1000).astype(np.float32)
    b = rng.standard_normal(1000).astype(np.float32)
    y = np.empty_like(a)
    R.ref_add_f32(p(a), p(b), p(y), 1000)
    out.update(add_a=a, add_b=b, add_y=y)

    path = os.path.join(HERE, "nnml_ref_ops.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()
