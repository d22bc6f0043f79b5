"""arclight_b200 -- B200-native (sm_100a) ArcLight Qwen3 Q4_0 decode/prefill hot path.

The product is ``libalb_cuda.so`` (CUDA kernels + the C ABI declared in
``include/alb_cuda.h``).  This module only loads it with ctypes and declares
argument types; there is no Python or CPU fallback: if the library is missing
or fails to load, every call raises.
"""
from __future__ import annotations

import ctypes as C
import os
import re

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
LIB_PATH = os.path.join(PKG, "libalb_cuda.so")
HEADER = os.path.join(ROOT, "include", "alb_cuda.h")

ALB_OK = 0
ALB_ERR_INVALID = -1
ALB_ERR_NO_SLOT = -7
ALB_FLASH_ATTN_STATIC_BYTES = 4 << 20   # include/alb_cuda.h
_lib = None


class AlbError(RuntimeError):
    pass


def header_symbols(path: str | None = None) -> list[str]:
    """Every function the C ABI headers declare (include/*.h, or one header)."""
    inc = os.path.join(ROOT, "include")
    paths = [path] if path else sorted(os.path.join(inc, f) for f in os.listdir(inc) if f.endswith(".h"))
    names = set()
    for p in paths:
        src = re.sub(r"/\*.*?\*/", "", open(p).read(), flags=re.S)
        names.update(re.findall(r"\b(alb_[a-z0-9_]+)\s*\(", src))
    return sorted(names)


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise AlbError(f"{LIB_PATH} is not built (run `python -m arclight_b200.build`); "
                           "there is no fallback path")
        _lib = C.CDLL(LIB_PATH)
        _declare(_lib)
    return _lib


def check(rc: int, what: str = "") -> None:
    if rc != ALB_OK:
        msg = lib().alb_last_error().decode(errors="replace")
        raise AlbError(f"{what or 'alb call'} failed with status {rc}: {msg}")


def _declare(L: C.CDLL) -> None:
    vp, i64, i32, f32, sz = C.c_void_p, C.c_int64, C.c_int32, C.c_float, C.c_size_t
    ci = C.c_int
    sigs = {
        "alb_version": (ci, []),
        "alb_last_error": (C.c_char_p, []),
        "alb_device_check": (ci, [ci]),
        "alb_device_error": (ci, [ci]),
        "alb_q4_0_gpu_bytes": (sz, [i64, i64]),
        "alb_q4_0_row_bytes": (sz, [i64]),
        "alb_repack_q4_0": (ci, [vp, vp, i64, i64, vp]),
        "alb_unpack_q4_0": (ci, [vp, vp, i64, i64, vp]),
        "alb_quantize_q8_0": (ci, [vp, vp, i64, i64, vp]),
        "alb_gemv_q4_0_q8_0": (ci, [vp, vp, vp, i64, i64, vp, vp]),
        "alb_gemv_q4_0_q8_0_block_dots": (ci, [vp, vp, vp, i64, i64, vp]),
        "alb_mul_mat_q4_0_q8_0": (ci, [vp, vp, vp, i64, i64, vp]),
        "alb_rms_norm": (ci, [vp, vp, vp, i64, i64, f32, vp]),
        "alb_swiglu": (ci, [vp, vp, vp, i64, vp]),
        "alb_rms_norm_q8": (ci, [vp, vp, vp, vp, i64, i64, f32, vp]),
        "alb_swiglu_q8": (ci, [vp, vp, vp, vp, i64, vp]),
        "alb_comm_create": (ci, [vp, C.c_int32, C.c_int32, C.c_int32, vp]),
        "alb_comm_destroy": (ci, [vp]),
        "alb_allreduce_sum_f32": (ci, [vp, vp, vp, i64, vp]),
        "alb_allgather_f32": (ci, [vp, vp, vp, i64, vp]),
        "alb_get_rows_q4_0": (ci, [vp, i64, i64, vp, i64, vp, vp]),
        "alb_set_rows_f16": (ci, [vp, i64, i64, vp, vp, i64, vp]),
        "alb_get_rows_f16": (ci, [vp, i64, i64, vp, i64, vp, vp]),
        "alb_kv_visible_cells": (ci, [vp, i32, i32, C.c_uint32, vp, vp]),
        "alb_rope_table": (ci, [vp, i32, i32, f32]),
        "alb_qk_norm_rope_kv": (ci, [vp, i64, i32, i32, vp, vp, f32, vp, i32, vp, vp, vp, vp]),
        "alb_qk_norm_rope_kv_cells": (ci, [vp, i64, i32, i32, vp, vp, f32, vp, i32, vp, vp, i64, vp, vp, vp, vp]),
        "alb_flash_attn_workspace_bytes": (sz, [i32, i32, i64, i32, i32]),
        "alb_flash_attn": (ci, [vp, vp, vp, i64, i32, i32, i32, f32, i32, vp, vp, vp]),
        "alb_gemm_workspace_bytes": (C.c_size_t, [i64, i64]),
        "alb_gemm_q4_0_q8_0": (ci, [vp, vp, vp, i64, i64, i64, vp, vp, vp]),
        "alb_engine_time_prefill_gemm": (ci, [vp, i32, C.POINTER(C.c_float), C.POINTER(C.c_double)]),
        "alb_flash_attn_static": (ci, [vp, vp, vp, i64, i32, i32, i32, f32, i32, vp, vp]),
        "alb_argmax": (ci, [vp, i64, vp, vp, vp]),
        "alb_nccl_unique_id": (ci, [vp]),
        "alb_engine_create": (ci, [vp, C.c_uint64, i32, i32, i32, i32, vp, i32, vp]),
        "alb_engine_destroy": (ci, [vp]),
        "alb_engine_device_bytes": (sz, [vp]),
        "alb_engine_reset": (ci, [vp]),
        "alb_engine_prefill": (ci, [vp, vp, i32, i32, vp]),
        "alb_engine_decode": (ci, [vp, i32, i32, vp]),
        "alb_engine_decode_loop": (ci, [vp, i32, i32, i32, vp, i32]),
        "alb_engine_logits": (ci, [vp, vp, i64]),
        "alb_engine_hidden": (ci, [vp, vp, i64]),
        "alb_engine_info": (ci, [vp, vp, i32]),
        "alb_engine_stream": (vp, [vp]),
        "alb_engine_weight_blocks": (ci, [vp, i32, i32, vp, vp, vp]),
        "alb_engine_norm_weights": (ci, [vp, i32, i32, vp, i64]),
        "alb_engine_set_weight_blocks": (ci, [vp, i32, i32, vp, i64, i64]),
        "alb_engine_set_norm_weights": (ci, [vp, i32, i32, vp, i64]),
        "alb_engine_fill_kv": (ci, [vp, i32, C.c_uint64]),
        "alb_engine_time_gemv": (ci, [vp, i32, vp, vp]),
        "alb_kv_create": (ci, [C.c_uint32, C.c_uint32, i32, C.c_uint32, vp]),
        "alb_kv_destroy": (ci, [vp]),
        "alb_kv_clear": (ci, [vp]),
        "alb_kv_find_slot": (ci, [vp, vp, vp, i32, i32, vp]),
        "alb_kv_prepare": (ci, [vp, vp, i32, vp, vp, vp]),
        "alb_kv_apply": (ci, [vp, vp, vp, i32, vp, vp]),
        "alb_kv_seq_rm": (ci, [vp, i32, i32, i32]),
        "alb_kv_seq_add": (ci, [vp, i32, i32, i32, i32]),
        "alb_kv_seq_pos_range": (ci, [vp, i32, vp, vp]),
        "alb_kv_mask": (ci, [vp, vp, vp, i32, i32, C.c_uint32, vp]),
        "alb_kv_cell": (ci, [vp, C.c_uint32, C.c_uint32, vp, vp, vp]),
        "alb_kv_info": (ci, [vp, C.c_uint32, vp, i32]),
    }
    for name, (res, args) in sigs.items():
        if hasattr(L, name):
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
