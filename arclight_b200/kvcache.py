"""KV-cache cell manager: the reference's ``llm_kv_cache`` slot interface over
the ``alb_kv_*`` C ABI (``include/alb_kvcache.h``, ``csrc/alb_kvcache.cpp``).

Method names follow ``llm_kv_cache`` (nnml/include/cgraph.h:249-374): ``prepare``
(cgraph.cpp:1263-1315), ``find_slot`` (:1317-1418), ``apply`` with the ubatch
(:1420-1492), ``seq_rm`` (:1535-1592), ``seq_add`` (:1501-1533),
``seq_pos_min`` / ``seq_pos_max`` (:1008-1018), ``set_inputs_attn_mask``
(:1224-1261) and ``clear`` (:988-993).  A ubatch is (positions, sequence ids),
one sequence per token; cell indices are flat ``stream * kv_size + cell``.
``prepare`` returns None where the reference returns an empty slot list
(no room), and ``find_slot`` likewise.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import ALB_ERR_NO_SLOT, check, lib

MAX_SEQ = 64
MASK_PAD = 64


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.int32).reshape(-1))


class KVCache:
    """Cells of a KV cache of ``kv_size`` cells per stream (one stream, or one
    per sequence when ``unified`` is False); ``kv_size % n_pad == 0``."""

    def __init__(self, kv_size: int, n_seq_max: int = 1, unified: bool = True, n_pad: int = 32):
        self._L = lib()
        h = C.c_void_p()
        check(self._L.alb_kv_create(kv_size, n_seq_max, 1 if unified else 0, n_pad, C.byref(h)), "alb_kv_create")
        self._h = h
        self.kv_size, self.n_pad = kv_size, n_pad
        self.n_stream = 1 if unified else n_seq_max
        self.n_kv = 0

    def close(self) -> None:
        if self._h:
            self._L.alb_kv_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def clear(self) -> None:
        check(self._L.alb_kv_clear(self._h), "alb_kv_clear")
        self.n_kv = 0

    def find_slot(self, pos, seq, cont: bool = False) -> np.ndarray | None:
        p, s = _i32(pos), _i32(seq)
        out = np.zeros(len(p), dtype=np.int64)
        rc = self._L.alb_kv_find_slot(self._h, p.ctypes.data, s.ctypes.data, len(p), int(cont), out.ctypes.data)
        if rc == ALB_ERR_NO_SLOT:
            return None
        check(rc, "alb_kv_find_slot")
        return out

    def prepare(self, ubatches) -> list[np.ndarray] | None:
        """Cells for each (pos, seq) ubatch placed in turn; the cells are left as
        they were.  None if some ubatch does not fit."""
        ps = [(_i32(p), _i32(s)) for p, s in ubatches]
        sizes = _i32([len(p) for p, _ in ps])
        pos = _i32(np.concatenate([p for p, _ in ps]))
        seq = _i32(np.concatenate([s for _, s in ps]))
        out = np.zeros(len(pos), dtype=np.int64)
        rc = self._L.alb_kv_prepare(self._h, sizes.ctypes.data, len(sizes), pos.ctypes.data, seq.ctypes.data,
                                    out.ctypes.data)
        if rc == ALB_ERR_NO_SLOT:
            return None
        check(rc, "alb_kv_prepare")
        return list(np.split(out, np.cumsum(sizes)[:-1]))

    def apply(self, pos, seq, idxs) -> int:
        """Place the ubatch in cells ``idxs``; returns (and keeps) n_kv."""
        p, s = _i32(pos), _i32(seq)
        ix = np.ascontiguousarray(np.asarray(idxs, dtype=np.int64))
        n_kv = C.c_uint32()
        check(self._L.alb_kv_apply(self._h, p.ctypes.data, s.ctypes.data, len(p), ix.ctypes.data, C.byref(n_kv)),
              "alb_kv_apply")
        self.n_kv = n_kv.value
        return self.n_kv

    def seq_rm(self, seq_id: int, p0: int, p1: int) -> None:
        check(self._L.alb_kv_seq_rm(self._h, seq_id, p0, p1), "alb_kv_seq_rm")

    def seq_add(self, seq_id: int, p0: int, p1: int, shift: int) -> None:
        check(self._L.alb_kv_seq_add(self._h, seq_id, p0, p1, shift), "alb_kv_seq_add")

    def _range(self, seq_id: int) -> tuple[int, int]:
        lo, hi = C.c_int32(), C.c_int32()
        check(self._L.alb_kv_seq_pos_range(self._h, seq_id, C.byref(lo), C.byref(hi)), "alb_kv_seq_pos_range")
        return lo.value, hi.value

    def seq_pos_min(self, seq_id: int) -> int:
        return self._range(seq_id)[0]

    def seq_pos_max(self, seq_id: int) -> int:
        return self._range(seq_id)[1]

    def set_inputs_attn_mask(self, pos, seq, n_stream_ub: int = 1, n_kv: int | None = None) -> np.ndarray:
        """The ubatch's mask [n_stream_ub, pad(n_tokens / n_stream_ub, 64), n_kv]
        (fp32: 0 visible, -inf hidden), over the current n_kv by default."""
        p, s = _i32(pos), _i32(seq)
        n_kv = self.n_kv if n_kv is None else n_kv
        n_tps = len(p) // n_stream_ub
        rows = (n_tps + MASK_PAD - 1) // MASK_PAD * MASK_PAD
        out = np.empty((n_stream_ub, rows, n_kv), dtype=np.float32)
        check(self._L.alb_kv_mask(self._h, p.ctypes.data, s.ctypes.data, len(p), n_stream_ub, n_kv,
                                  out.ctypes.data), "alb_kv_mask")
        return out

    def visible_cells(self, seq_id: int, pos: int, n_kv: int | None = None) -> np.ndarray:
        """Flat indices of the cells (seq_id, pos) may see among the first n_kv,
        ascending: one mask row as a list (the rows to gather for attention)."""
        n_kv = self.n_kv if n_kv is None else n_kv
        out = np.zeros(max(n_kv, 1), dtype=np.int64)
        n = C.c_int32()
        check(self._L.alb_kv_visible_cells(self._h, seq_id, pos, n_kv, out.ctypes.data, C.byref(n)),
              "alb_kv_visible_cells")
        return out[:n.value].copy()

    def cell(self, stream: int, idx: int) -> tuple[int, int, int]:
        """(position or -1, sequence bit set, accumulated shift) of one cell."""
        p, q, sh = C.c_int32(), C.c_uint64(), C.c_int32()
        check(self._L.alb_kv_cell(self._h, stream, idx, C.byref(p), C.byref(q), C.byref(sh)), "alb_kv_cell")
        return p.value, q.value, sh.value

    def info(self, stream: int = 0) -> dict:
        v = np.zeros(6, dtype=np.int64)
        check(self._L.alb_kv_info(self._h, stream, v.ctypes.data, 6), "alb_kv_info")
        keys = ("kv_size", "n_stream", "n_pad", "used", "head", "used_max_p1")
        return dict(zip(keys, (int(x) for x in v)))
