"""Pin the oracle (oracle/oracle.c) against the reference's own nnml code.

tests/golden/nnml_ref_ops.npz holds outputs of the reference's portable sources
(types.cpp, ops.cpp, binary.cpp, common.cpp, tensor.cpp, memory.cpp) compiled
unmodified by oracle/Makefile and driven by oracle/ref_driver.cpp
(tests/golden/make_golden.py).  Every comparison here is bit-exact.
"""
import os

import numpy as np
import pytest

from oracle import lib as O

G = np.load(os.path.join(os.path.dirname(__file__), "golden", "nnml_ref_ops.npz"))


def test_fp16_conversion_matches_reference():
    f = G["fp16_in"]
    got = np.array([O.lib().orc_fp32_to_fp16(float(v)) for v in f], np.uint16)
    np.testing.assert_array_equal(got, G["fp16_out"])
    back = np.array([O.lib().orc_fp16_to_fp32(int(h)) for h in got], np.float32)
    ok = np.isfinite(back)
    np.testing.assert_array_equal(back[ok], G["fp16_out"][ok].view(np.float16).astype(np.float32))


def test_q4_0_quantize_dequantize_match_reference():
    q = O.quantize_q4_0(G["q4_in"])
    np.testing.assert_array_equal(q.reshape(-1).view(np.uint8), G["q4_out"])
    np.testing.assert_array_equal(O.dequantize_q4_0(q), G["q4_deq"])


def test_q8_0_ref_quantize_matches_reference():
    q = O.quantize_q8_0(G["q8_in"], ref_rounding=True)
    np.testing.assert_array_equal(q.reshape(-1).view(np.uint8), G["q8_out"])
    np.testing.assert_array_equal(O.dequantize_q8_0(q), G["q8_deq"])


def test_repack_4x4_matches_reference():
    w = G["repack_in"].view(O.Q4_DTYPE).reshape(8, 4)
    np.testing.assert_array_equal(O.repack_q4_0_4x4(w), G["repack_out"])


@pytest.mark.parametrize("pre", ["rms", "rmsh"])
def test_rms_norm_mul_matches_reference(pre):
    np.testing.assert_array_equal(O.rms_norm(G[pre + "_x"], G[pre + "_w"]), G[pre + "_y"])


def test_rope_neox_matches_reference():
    for i, pos in enumerate(G["rope_pos"]):
        np.testing.assert_array_equal(O.rope_neox(G["rope_x"][i], int(pos)), G["rope_y"][i], err_msg=f"pos {pos}")


def test_get_rows_matches_reference():
    tab = G["getrows_table"].view(O.Q4_DTYPE).reshape(50, 8)
    got = np.stack([O.dequantize_q4_0(tab[i]) for i in G["getrows_ids"]])
    np.testing.assert_array_equal(got, G["getrows_out"])


def test_set_rows_f16_matches_reference():
    cache = np.zeros((16, 256), np.uint16)
    for r, i in enumerate(G["setrows_idx"]):
        cache[i] = O.fp32_to_fp16(G["setrows_src"][r])
    np.testing.assert_array_equal(cache, G["setrows_cache"])


def test_gather_add_matches_reference():
    np.testing.assert_array_equal(G["add_a"] + G["add_b"], G["add_y"])


# ---- known-answer tests derived from the reference code (no fixture needed) ----
def test_kat_xor_nibble_trick():
    # types.cpp:140-149 / gemm.cpp:115-117: after XOR 0x88, (int8)(b<<4) == 16*(q-8)
    for q in range(16):
        b = (q ^ 0x8) & 0xF
        v = np.array([b << 4], np.uint8).view(np.int8)[0]
        assert int(v) == 16 * (q - 8)


def test_kat_zero_block():
    # types.cpp:366-373: all-zero block -> d = 0/-8 = -0.0 (fp16 0x8000), id = 0, every nibble = 8
    q = O.quantize_q4_0(np.zeros(32, np.float32))
    assert q["d"][0] == 0x8000
    assert all(int(b) == 0x88 for b in q["qs"][0])
    q8 = O.quantize_q8_0(np.zeros(32, np.float32))
    assert q8["d"][0] == 0 and not q8["qs"].any()


def test_kat_q8_exact_127():
    # arm.cpp:1836-1841: max-abs 127*2^k quantizes to exact +/-127
    x = np.linspace(-1, 1, 32).astype(np.float32) * np.float32(127 * 2.0 ** -3)
    q = O.quantize_q8_0(x)
    assert q["qs"][0].max() == 127 and q["qs"][0].min() == -127


def test_q8_runtime_rounding_is_rne():
    # arm.cpp:1841 vcvtnq: ties to even, unlike the _ref's roundf
    x = np.zeros(32, np.float32)
    x[0] = 127.0
    x[1] = 2.5
    x[2] = -2.5
    x[3] = 3.5
    q = O.quantize_q8_0(x)["qs"][0]
    qr = O.quantize_q8_0(x, ref_rounding=True)["qs"][0]
    assert (q[1], q[2], q[3]) == (2, -2, 4)
    assert (qr[1], qr[2], qr[3]) == (3, -3, 4)
