"""ctypes front-end of the ArcLight hot-path ORACLE (test infrastructure only).

Loads ``oracle/liboracle.so`` (built from ``oracle/oracle.c`` by
``oracle/Makefile``), the CPU restatement of the reference's nnml arithmetic.
Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s ``cpu_baseline``
and ``--impl reference`` legs import this module, as the checker or as the
timed CPU baseline.  The CUDA product in ``arclight_b200`` never imports it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
REF_PATH = os.path.join(HERE, "_ref", "libalref.so")

Q4_BYTES = 18   # block_q4_0 (nnml.h:646-651)
Q8_BYTES = 34   # block_q8_0 (nnml.h:695-700)

Q4_DTYPE = np.dtype([("d", "<u2"), ("qs", "u1", (16,))])
Q8_DTYPE = np.dtype([("d", "<u2"), ("qs", "i1", (32,))])
assert Q4_DTYPE.itemsize == Q4_BYTES and Q8_DTYPE.itemsize == Q8_BYTES

# tensor kinds (oracle.h)
T_TOK_EMBD, T_OUTPUT, T_OUTPUT_NORM = 0, 1, 2
T_ATTN_NORM, T_WQ, T_WK, T_WV, T_WO, T_Q_NORM, T_K_NORM, T_FFN_NORM, T_GATE, T_UP, T_DOWN = range(3, 14)


class Qwen3Config(C.Structure):
    _fields_ = [("n_layer", C.c_int32), ("n_embd", C.c_int32), ("n_head", C.c_int32),
                ("n_head_kv", C.c_int32), ("head_dim", C.c_int32), ("n_ff", C.c_int32),
                ("n_vocab", C.c_int32), ("tied", C.c_int32), ("eps", C.c_float),
                ("freq_base", C.c_float)]


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def build(quiet: bool = True) -> None:
    """Compile liboracle.so (gcc, no GPU needed)."""
    out = subprocess.run(["make", "-C", HERE, "all"], capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + out.stdout + out.stderr)


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(os.path.join(HERE, "oracle.c")):
            build()
        L = C.CDLL(LIB_PATH)
        vp, i64, i32, f32, u64 = C.c_void_p, C.c_int64, C.c_int32, C.c_float, C.c_uint64
        sig = {
            "orc_fp32_to_fp16": (C.c_uint16, [f32]),
            "orc_fp16_to_fp32": (f32, [C.c_uint16]),
            "orc_splitmix64": (u64, [u64]),
            "orc_normal_table": (None, [vp]),
            "orc_normal": (f32, [vp, u64, u64]),
            "orc_tensor_seed": (u64, [u64, C.c_int, C.c_int]),
            "orc_quantize_row_q4_0": (None, [vp, vp, i64]),
            "orc_dequantize_row_q4_0": (None, [vp, vp, i64]),
            "orc_quantize_row_q8_0": (None, [vp, vp, i64]),
            "orc_quantize_row_q8_0_ref": (None, [vp, vp, i64]),
            "orc_dequantize_row_q8_0": (None, [vp, vp, i64]),
            "orc_repack_q4_0_4x4": (C.c_int, [vp, vp, i64, i64]),
            "orc_gemv_q4_0_q8_0": (None, [vp, vp, vp, i64, i64, vp, C.c_int]),
            "orc_gemv_q4_0_q8_0_exact": (None, [vp, vp, vp, i64, i64, C.c_int]),
            "orc_neon_expf": (f32, [f32]),
            "orc_model_set_exact": (None, [vp, C.c_int]),
            "orc_model_set_tp": (None, [vp, C.c_int]),
            "orc_gemv_q4_0_q8_0_exact_tp": (None, [vp, vp, vp, C.c_int64, C.c_int64, C.c_int, C.c_int]),
            "orc_gemv_q4_0_q8_0_tp": (None, [vp, vp, vp, C.c_int64, C.c_int64, C.c_int, C.c_int]),
            "orc_vec_dot_q4_0_q8_0": (f32, [vp, vp, i64]),
            "orc_mul_mat_generic": (None, [vp, vp, vp, i64, i64, C.c_int]),
            "orc_rms_norm": (None, [vp, vp, vp, i64, i64, f32]),
            "orc_rope_cache": (None, [i32, i64, f32, vp]),
            "orc_rope_neox": (None, [vp, vp, i64, i64, i32, f32]),
            "orc_swiglu": (None, [vp, vp, vp, i64]),
            "orc_gather_sum": (None, [vp, C.c_int, vp, i64]),
            "orc_flash_attn": (None, [vp, vp, vp, vp, i64, i64, i64, i64, f32, C.c_int, vp]),
            "orc_model_create": (vp, [vp, u64, i32, C.c_int]),
            "orc_model_free": (None, [vp]),
            "orc_model_q4_tensor": (vp, [vp, C.c_int, C.c_int, vp, vp]),
            "orc_model_f32_tensor": (vp, [vp, C.c_int, C.c_int, vp]),
            "orc_model_forward": (C.c_int, [vp, vp, i32, i32, C.c_int, vp, vp]),
            "orc_model_reset": (None, [vp]),
            "orc_model_fill_kv": (None, [vp, i32, C.c_uint64]),
            "orc_argmax": (i32, [vp, i64]),
        }
        for name, (res, args) in sig.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


# ----------------------------------------------------------------- helpers
def fp32_to_fp16(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, np.float32).astype(np.float16).view(np.uint16)


def normal_table() -> np.ndarray:
    t = np.empty(65537, np.float32)
    lib().orc_normal_table(_ptr(t))
    return t


def quantize_q4_0(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty(x.size // 32, Q4_DTYPE)
    lib().orc_quantize_row_q4_0(_ptr(x), _ptr(y), x.size)
    return y.reshape(x.shape[:-1] + (x.shape[-1] // 32,))


def dequantize_q4_0(q: np.ndarray) -> np.ndarray:
    q = np.ascontiguousarray(q)
    y = np.empty(q.size * 32, np.float32)
    lib().orc_dequantize_row_q4_0(_ptr(q), _ptr(y), q.size * 32)
    return y.reshape(q.shape[:-1] + (q.shape[-1] * 32,))


def quantize_q8_0(x: np.ndarray, ref_rounding: bool = False) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty(x.size // 32, Q8_DTYPE)
    fn = lib().orc_quantize_row_q8_0_ref if ref_rounding else lib().orc_quantize_row_q8_0
    fn(_ptr(x), _ptr(y), x.size)
    return y.reshape(x.shape[:-1] + (x.shape[-1] // 32,))


def dequantize_q8_0(q: np.ndarray) -> np.ndarray:
    q = np.ascontiguousarray(q)
    y = np.empty(q.size * 32, np.float32)
    lib().orc_dequantize_row_q8_0(_ptr(q), _ptr(y), q.size * 32)
    return y.reshape(q.shape[:-1] + (q.shape[-1] * 32,))


def repack_q4_0_4x4(w: np.ndarray) -> np.ndarray:
    w = np.ascontiguousarray(w)
    n, nb = w.shape
    out = np.empty(n * nb * 18, np.uint8)
    rc = lib().orc_repack_q4_0_4x4(_ptr(w), _ptr(out), n, nb * 32)
    if rc != 0:
        raise ValueError("repack requires rows % 4 == 0")
    return out


def gemv(w: np.ndarray, xq: np.ndarray, threads: int = 8):
    """y[N] and block dots I[N][K/32] of a Q4_0 [N][K/32] x Q8_0 [K/32] mat-vec."""
    w = np.ascontiguousarray(w)
    xq = np.ascontiguousarray(xq)
    n, nb = w.shape
    y = np.empty(n, np.float32)
    dots = np.empty((n, nb), np.int32)
    lib().orc_gemv_q4_0_q8_0(_ptr(w), _ptr(xq), _ptr(y), n, nb * 32, _ptr(dots), threads)
    return y, dots


def gemv_exact(w: np.ndarray, xq: np.ndarray, threads: int = 8) -> np.ndarray:
    """Exactly rounded mat-vec (block terms summed exactly in double)."""
    w = np.ascontiguousarray(w)
    xq = np.ascontiguousarray(xq)
    n, nb = w.shape
    y = np.empty(n, np.float32)
    lib().orc_gemv_q4_0_q8_0_exact(_ptr(w), _ptr(xq), _ptr(y), n, nb * 32, threads)
    return y


def gemv_tp(w: np.ndarray, xq: np.ndarray, tp: int, threads: int = 8) -> np.ndarray:
    """The reference's TP mat-vec of a column-split matrix: node chains over K/tp
    slices, partials added in node order."""
    w = np.ascontiguousarray(w)
    xq = np.ascontiguousarray(xq)
    n, nb = w.shape
    y = np.empty(n, np.float32)
    lib().orc_gemv_q4_0_q8_0_tp(_ptr(w), _ptr(xq), _ptr(y), n, nb * 32, tp, threads)
    return y


def mul_mat_generic(w: np.ndarray, xq: np.ndarray, threads: int = 8) -> np.ndarray:
    w = np.ascontiguousarray(w)
    xq = np.ascontiguousarray(xq)
    n, nb = w.shape
    y = np.empty(n, np.float32)
    lib().orc_mul_mat_generic(_ptr(w), _ptr(xq), _ptr(y), n, nb * 32, threads)
    return y


def rms_norm(x: np.ndarray, w, eps: float = 1e-6) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    n = x.shape[-1]
    y = np.empty_like(x)
    wp = None if w is None else _ptr(np.ascontiguousarray(w, np.float32))
    lib().orc_rms_norm(_ptr(x), wp, _ptr(y), x.size // n, n, eps)
    return y


def rope_neox(x: np.ndarray, pos: int, freq_base: float = 1e6) -> np.ndarray:
    """x: [n_heads][head_dim] of one token."""
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    lib().orc_rope_neox(_ptr(x), _ptr(y), x.shape[0], x.shape[1], int(pos), freq_base)
    return y


def swiglu(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    g = np.ascontiguousarray(g, np.float32)
    u = np.ascontiguousarray(u, np.float32)
    y = np.empty_like(g)
    lib().orc_swiglu(_ptr(g), _ptr(u), _ptr(y), g.size)
    return y


def flash_attn(q, k, v, kv_len, scale, mode=0):
    """q [T][H][D] f32, k/v [cells][Hkv][D] fp16 bits (uint16), kv_len [T] int32.
    mode 0: fp32 scores / double sums (the CUDA semantics); 1: the reference's
    fp16-accumulating NEON loop; 2: fp64 attention (the yardstick)."""
    q = np.ascontiguousarray(q, np.float32)
    k = np.ascontiguousarray(k, np.uint16)
    v = np.ascontiguousarray(v, np.uint16)
    kv_len = np.ascontiguousarray(kv_len, np.int32)
    T, H, D = q.shape
    Hkv = k.shape[1]
    out = np.empty_like(q)
    lib().orc_flash_attn(_ptr(q), _ptr(k), _ptr(v), _ptr(kv_len), T, H, Hkv, D, scale, mode, _ptr(out))
    return out


class Model:
    """Synthetic seeded Qwen3 model on the CPU (qwen3.cpp:174-275 restated)."""

    def __init__(self, cfg: dict, seed: int, max_ctx: int, threads: int = 8):
        self.cfg = cfg
        c = Qwen3Config(cfg["n_layer"], cfg["n_embd"], cfg["n_head"], cfg["n_head_kv"], cfg["head_dim"],
                        cfg["n_ff"], cfg["n_vocab"], int(cfg.get("tied", 1)), cfg.get("eps", 1e-6),
                        cfg.get("freq_base", 1e6))
        self._c = c
        self.h = lib().orc_model_create(C.byref(c), seed, max_ctx, threads)
        if not self.h:
            raise MemoryError("orc_model_create failed")

    def close(self):
        if self.h:
            lib().orc_model_free(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def q4_tensor(self, layer: int, kind: int) -> np.ndarray:
        rows, cols = C.c_int64(), C.c_int64()
        p = lib().orc_model_q4_tensor(self.h, layer, kind, C.byref(rows), C.byref(cols))
        nb = cols.value // 32
        buf = (C.c_uint8 * (rows.value * nb * Q4_BYTES)).from_address(p)
        return np.frombuffer(buf, Q4_DTYPE).reshape(rows.value, nb).copy()

    def f32_tensor(self, layer: int, kind: int) -> np.ndarray:
        n = C.c_int64()
        p = lib().orc_model_f32_tensor(self.h, layer, kind, C.byref(n))
        return np.ctypeslib.as_array((C.c_float * n.value).from_address(p)).copy()

    def forward(self, tokens, pos0: int, fa_mode: int = 0):
        toks = np.ascontiguousarray(tokens, np.int32)
        logits = np.empty(self.cfg["n_vocab"], np.float32)
        hidden = np.empty(self.cfg["n_embd"], np.float32)
        rc = lib().orc_model_forward(self.h, _ptr(toks), toks.size, pos0, fa_mode, _ptr(logits), _ptr(hidden))
        if rc != 0:
            raise ValueError(f"orc_model_forward failed ({rc})")
        return logits, hidden

    def reset(self):
        lib().orc_model_reset(self.h)

    def fill_kv(self, n_pos: int, seed: int):
        """K/V of positions [0, n_pos) := fp16 N(0,1), the long-context benchmark's pre-fill."""
        lib().orc_model_fill_kv(self.h, int(n_pos), int(seed))

    def set_exact(self, exact: bool):
        """False (default): the reference's NEON fp32 chains; True: exactly rounded mat-vecs."""
        lib().orc_model_set_exact(self.h, 1 if exact else 0)

    def set_tp(self, tp: int):
        """tp > 1: O and down projections as tp node partials added in node order
        (the reference's tensor-parallel GATHER)."""
        lib().orc_model_set_tp(self.h, int(tp))


def argmax(x: np.ndarray) -> int:
    x = np.ascontiguousarray(x, np.float32)
    return int(lib().orc_argmax(_ptr(x), x.size))


def ref_lib():
    """The reference's own portable nnml code compiled by ``make -C oracle ref``
    (only where the reference sources are present)."""
    if not os.path.exists(REF_PATH):
        return None
    L = C.CDLL(REF_PATH)
    vp, i64, f32 = C.c_void_p, C.c_int64, C.c_float
    sig = {
        "ref_quantize_row_q4_0": (None, [vp, vp, i64]),
        "ref_dequantize_row_q4_0": (None, [vp, vp, i64]),
        "ref_quantize_row_q8_0_ref": (None, [vp, vp, i64]),
        "ref_dequantize_row_q8_0": (None, [vp, vp, i64]),
        "ref_fp32_to_fp16": (C.c_uint16, [f32]),
        "ref_fp16_to_fp32": (f32, [C.c_uint16]),
        "ref_repack_q4_0_4x4": (C.c_int, [vp, vp, i64, i64]),
        "ref_rms_norm_mul": (None, [vp, vp, vp, i64, i64, f32]),
        "ref_rope_neox": (None, [vp, vp, i64, i64, i64, vp, f32]),
        "ref_get_rows_q4_0": (None, [vp, i64, i64, vp, i64, vp]),
        "ref_set_rows_f16": (None, [vp, i64, i64, vp, vp, i64]),
        "ref_add_f32": (None, [vp, vp, vp, i64]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    return L
