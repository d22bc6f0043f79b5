"""Python handle on the C-ABI Qwen3 engine (alb_engine_* in include/alb_cuda.h)."""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import AlbError, check, lib

Q4_DTYPE = np.dtype([("d", "<u2"), ("qs", "u1", (16,))])


class Qwen3Config(C.Structure):
    _fields_ = [("n_layer", C.c_int32), ("n_embd", C.c_int32), ("n_head", C.c_int32),
                ("n_head_kv", C.c_int32), ("head_dim", C.c_int32), ("n_ff", C.c_int32),
                ("n_vocab", C.c_int32), ("tied", C.c_int32), ("eps", C.c_float), ("freq_base", C.c_float)]

    @classmethod
    def from_dict(cls, d):
        return cls(d["n_layer"], d["n_embd"], d["n_head"], d["n_head_kv"], d["head_dim"], d["n_ff"],
                   d["n_vocab"], int(d.get("tied", 1)), d.get("eps", 1e-6), d.get("freq_base", 1e6))


def nccl_unique_id() -> bytes:
    buf = (C.c_uint8 * 128)()
    check(lib().alb_nccl_unique_id(buf), "alb_nccl_unique_id")
    return bytes(buf)


class Engine:
    def __init__(self, cfg: dict, seed: int, max_ctx: int, max_ubatch: int = 256, tp_rank: int = 0,
                 tp_size: int = 1, nccl_id: bytes | None = None, device: int = 0):
        self.cfg = dict(cfg)
        self._c = Qwen3Config.from_dict(cfg)
        self.h = C.c_void_p()
        idb = None
        if tp_size > 1:
            if nccl_id is None or len(nccl_id) != 128:
                raise AlbError("tensor parallel engine needs a 128-byte NCCL unique id")
            idb = (C.c_uint8 * 128).from_buffer_copy(nccl_id)
        check(lib().alb_engine_create(C.byref(self._c), seed, max_ctx, max_ubatch, tp_rank, tp_size, idb, device,
                                      C.byref(self.h)), "alb_engine_create")
        info = (C.c_int64 * 8)()
        check(lib().alb_engine_info(self.h, info, 8))
        self.vocab_local, self.vocab_offset = int(info[0]), int(info[1])
        self.max_ctx = max_ctx

    def info(self) -> dict:
        info = (C.c_int64 * 8)()
        check(lib().alb_engine_info(self.h, info, 8))
        keys = ["vocab_local", "vocab_offset", "n_head_local", "n_head_kv_local", "n_ff_local",
                "launches_per_step", "device_bytes", "attn_splits"]
        return dict(zip(keys, [int(v) for v in info]))

    def close(self):
        if self.h:
            lib().alb_engine_destroy(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def reset(self):
        check(lib().alb_engine_reset(self.h), "alb_engine_reset")

    def prefill(self, tokens, pos0: int = 0) -> int:
        t = np.ascontiguousarray(tokens, np.int32)
        out = C.c_int32()
        check(lib().alb_engine_prefill(self.h, t.ctypes.data_as(C.c_void_p), t.size, pos0, C.byref(out)),
              "alb_engine_prefill")
        return int(out.value)

    def decode(self, token: int, pos: int) -> int:
        out = C.c_int32()
        check(lib().alb_engine_decode(self.h, int(token), int(pos), C.byref(out)), "alb_engine_decode")
        return int(out.value)

    def decode_loop(self, token: int, pos: int, n_steps: int, want_tokens: bool = True, sync: bool = True):
        buf = np.empty(n_steps, np.int32) if want_tokens else None
        check(lib().alb_engine_decode_loop(self.h, int(token), int(pos), int(n_steps),
                                           buf.ctypes.data_as(C.c_void_p) if buf is not None else None,
                                           1 if sync else 0), "alb_engine_decode_loop")
        return buf

    def logits(self) -> np.ndarray:
        out = np.empty(self.vocab_local, np.float32)
        check(lib().alb_engine_logits(self.h, out.ctypes.data_as(C.c_void_p), out.size), "alb_engine_logits")
        return out

    def hidden(self, rows: int) -> np.ndarray:
        """Residual stream of the last forward pass, rows [0, rows) of its ubatch."""
        out = np.empty((rows, self.cfg["n_embd"]), np.float32)
        check(lib().alb_engine_hidden(self.h, out.ctypes.data_as(C.c_void_p), rows), "alb_engine_hidden")
        return out

    def stream(self) -> int:
        return lib().alb_engine_stream(self.h) or 0

    def weight_blocks(self, layer: int, kind: int) -> np.ndarray:
        rows, cols = C.c_int64(), C.c_int64()
        check(lib().alb_engine_weight_blocks(self.h, layer, kind, None, C.byref(rows), C.byref(cols)))
        out = np.empty((rows.value, cols.value // 32), Q4_DTYPE)
        check(lib().alb_engine_weight_blocks(self.h, layer, kind, out.ctypes.data_as(C.c_void_p), C.byref(rows),
                                             C.byref(cols)), "alb_engine_weight_blocks")
        return out

    def norm_weights(self, layer: int, kind: int, n: int) -> np.ndarray:
        out = np.empty(n, np.float32)
        check(lib().alb_engine_norm_weights(self.h, layer, kind, out.ctypes.data_as(C.c_void_p), n))
        return out

    def fill_kv(self, n_pos: int, seed: int):
        check(lib().alb_engine_fill_kv(self.h, n_pos, seed), "alb_engine_fill_kv")
