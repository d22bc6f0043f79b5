"""GGUF model files for the engine: read a Qwen3 Q4_0 model and upload it.

The reference loads a model in llm_model::load_model / load_all_tensors
(src/model.cpp:130-335 header, key/values and tensor infos, :355-474 tensor
data) with the Qwen3 keys and tensor names of models/qwen3.cpp:7-45.  Format
(little-endian): magic "GGUF", u32 version, u64 tensor count, u64 key/value
count; each key/value = string key, u32 type, value (strings are u64 length +
bytes, arrays are u32 element type + u64 count + elements); each tensor info =
string name, u32 n_dims, u64 ne[n_dims] (ne[0] innermost), u32 type, u64 offset
relative to the data section, which starts at the first multiple of the
alignment (key general.alignment, default 32) after the tensor infos
(model.cpp:149, 334-335).  Tensor types used here: F32 (0), F16 (1) and Q4_0
(2: 18-byte blocks of 32 values, the block_q4_0 of the C ABI).

`load_qwen3(path, ...)` returns an Engine holding the file's weights: the
configuration comes from the qwen3.* keys (n_vocab from token_embd), each Q4_0
matrix goes through alb_engine_set_weight_blocks (which keeps this rank's
tensor-parallel shard and repacks it on the device) and each norm through
alb_engine_set_norm_weights.  `write_gguf` writes files of the same format
(tests build models with it; no checkpoint is needed).
"""
from __future__ import annotations

import ctypes as C
import struct
from dataclasses import dataclass

import numpy as np

GGUF_MAGIC = b"GGUF"
DEFAULT_ALIGNMENT = 32

# value types (gguf.cpp: GGUF_TYPE_*)
T_UINT8, T_INT8, T_UINT16, T_INT16, T_UINT32, T_INT32, T_FLOAT32, T_BOOL, T_STRING, T_ARRAY, \
    T_UINT64, T_INT64, T_FLOAT64 = range(13)
_SCALAR = {T_UINT8: "<B", T_INT8: "<b", T_UINT16: "<H", T_INT16: "<h", T_UINT32: "<I", T_INT32: "<i",
           T_FLOAT32: "<f", T_BOOL: "<B", T_UINT64: "<Q", T_INT64: "<q", T_FLOAT64: "<d"}

# tensor types: (block size in values, bytes per block)
GGML_F32, GGML_F16, GGML_Q4_0 = 0, 1, 2
_TENSOR_TYPES = {GGML_F32: (1, 4), GGML_F16: (1, 2), GGML_Q4_0: (32, 18)}

# engine tensor kinds (oracle.h ORC_T_*, the C ABI's kinds)
K_TOK_EMBD, K_OUTPUT, K_OUTPUT_NORM, K_ATTN_NORM, K_WQ, K_WK, K_WV, K_WO, K_Q_NORM, K_K_NORM, K_FFN_NORM, \
    K_GATE, K_UP, K_DOWN = range(14)
# per-layer tensor names (models/qwen3.cpp:35-45) -> kind
LAYER_TENSORS = {"attn_norm.weight": K_ATTN_NORM, "attn_q.weight": K_WQ, "attn_k.weight": K_WK,
                 "attn_v.weight": K_WV, "attn_output.weight": K_WO, "attn_q_norm.weight": K_Q_NORM,
                 "attn_k_norm.weight": K_K_NORM, "ffn_norm.weight": K_FFN_NORM, "ffn_gate.weight": K_GATE,
                 "ffn_up.weight": K_UP, "ffn_down.weight": K_DOWN}
NORM_KINDS = {K_ATTN_NORM, K_Q_NORM, K_K_NORM, K_FFN_NORM, K_OUTPUT_NORM}


class GGUFError(ValueError):
    pass


@dataclass
class TensorInfo:
    name: str
    ne: tuple          # ne[0] innermost (columns of a matrix)
    ttype: int
    offset: int        # absolute file offset of the data
    nbytes: int

    @property
    def shape(self):   # numpy order: rows first
        return tuple(reversed(self.ne))


class _Cursor:
    def __init__(self, buf: memoryview):
        self.buf, self.pos = buf, 0

    def take(self, n: int) -> bytes:
        if self.pos + n > len(self.buf):
            raise GGUFError("truncated file")
        b = bytes(self.buf[self.pos:self.pos + n])
        self.pos += n
        return b

    def scalar(self, t: int):
        fmt = _SCALAR[t]
        (v,) = struct.unpack(fmt, self.take(struct.calcsize(fmt)))
        return bool(v) if t == T_BOOL else v

    def string(self) -> str:
        n = self.scalar(T_UINT64)
        return self.take(n).decode("utf-8", errors="replace")

    def value(self, t: int):
        if t == T_STRING:
            return self.string()
        if t == T_ARRAY:
            et = self.scalar(T_UINT32)
            n = self.scalar(T_UINT64)
            if et == T_ARRAY:
                raise GGUFError("nested arrays are not supported")
            return [self.value(et) for _ in range(n)]
        if t not in _SCALAR:
            raise GGUFError(f"unknown value type {t}")
        return self.scalar(t)


class GGUFReader:
    """Header, key/values and tensor infos of a GGUF file; tensor data mapped lazily."""

    def __init__(self, path: str):
        self.path = path
        self._map = np.memmap(path, dtype=np.uint8, mode="r")
        cur = _Cursor(memoryview(self._map))
        if cur.take(4) != GGUF_MAGIC:
            raise GGUFError(f"{path}: not a GGUF file")
        self.version = cur.scalar(T_UINT32)
        if self.version not in (2, 3):
            raise GGUFError(f"{path}: unsupported GGUF version {self.version}")
        n_tensors = cur.scalar(T_UINT64)
        n_kv = cur.scalar(T_UINT64)
        self.kv = {}
        for _ in range(n_kv):
            key = cur.string()
            self.kv[key] = cur.value(cur.scalar(T_UINT32))
        align = int(self.kv.get("general.alignment", DEFAULT_ALIGNMENT))
        if align <= 0 or align & (align - 1):
            raise GGUFError(f"{path}: bad alignment {align}")
        infos = []
        for _ in range(n_tensors):
            name = cur.string()
            nd = cur.scalar(T_UINT32)
            ne = tuple(cur.scalar(T_UINT64) for _ in range(nd))
            tt = cur.scalar(T_UINT32)
            off = cur.scalar(T_UINT64)
            infos.append((name, ne, tt, off))
        base = (cur.pos + align - 1) // align * align
        self.tensors = {}
        for name, ne, tt, off in infos:
            if tt not in _TENSOR_TYPES:
                raise GGUFError(f"{path}: tensor {name} has unsupported type {tt}")
            bs, bb = _TENSOR_TYPES[tt]
            count = int(np.prod(ne)) if ne else 1
            if ne and ne[0] % bs:
                raise GGUFError(f"{path}: tensor {name}: {ne[0]} values per row is not a multiple of {bs}")
            nbytes = count // bs * bb
            if base + off + nbytes > len(self._map):
                raise GGUFError(f"{path}: tensor {name} runs past the end of the file")
            self.tensors[name] = TensorInfo(name, ne, tt, base + off, nbytes)

    def raw(self, name: str) -> np.ndarray:
        t = self.tensors[name]
        return self._map[t.offset:t.offset + t.nbytes]

    def f32(self, name: str) -> np.ndarray:
        """A float tensor (F32 or F16) as fp32, numpy shape (rows first)."""
        t = self.tensors[name]
        if t.ttype == GGML_F32:
            return np.frombuffer(self.raw(name), dtype="<f4").reshape(t.shape)
        if t.ttype == GGML_F16:
            return np.frombuffer(self.raw(name), dtype="<f2").astype(np.float32).reshape(t.shape)
        raise GGUFError(f"tensor {name} is not a float tensor")

    def q4_0(self, name: str) -> np.ndarray:
        """A Q4_0 matrix as its block_q4_0 bytes, shape [rows][cols / 32 * 18]."""
        t = self.tensors[name]
        if t.ttype != GGML_Q4_0 or len(t.ne) != 2:
            raise GGUFError(f"tensor {name} is not a Q4_0 matrix")
        return self.raw(name).reshape(t.ne[1], t.ne[0] // 32 * 18)


def qwen3_config(r: GGUFReader) -> dict:
    """Engine configuration from the qwen3.* keys (models/qwen3.cpp:7-16)."""
    kv = r.kv
    arch = kv.get("general.architecture", "qwen3")
    if arch != "qwen3":
        raise GGUFError(f"architecture {arch!r} is not qwen3")

    def need(key):
        if key not in kv:
            raise GGUFError(f"missing key {key}")
        return kv[key]
    n_head = int(need("qwen3.attention.head_count"))
    n_embd = int(need("qwen3.embedding_length"))
    head_dim = int(kv.get("qwen3.attention.key_length", n_embd // n_head))
    if "token_embd.weight" not in r.tensors:
        raise GGUFError("missing tensor token_embd.weight")
    return dict(n_layer=int(need("qwen3.block_count")), n_embd=n_embd, n_head=n_head,
                n_head_kv=int(need("qwen3.attention.head_count_kv")), head_dim=head_dim,
                n_ff=int(need("qwen3.feed_forward_length")),
                n_vocab=int(r.tensors["token_embd.weight"].ne[1]),
                tied="output.weight" not in r.tensors,
                eps=float(kv.get("qwen3.attention.layer_norm_rms_epsilon", 1e-6)),
                freq_base=float(kv.get("qwen3.rope.freq_base", 1e6)))


def tensor_plan(cfg: dict):
    """(gguf name, layer, kind) of every tensor the engine takes."""
    plan = [("token_embd.weight", -1, K_TOK_EMBD), ("output_norm.weight", -1, K_OUTPUT_NORM)]
    if not cfg["tied"]:
        plan.append(("output.weight", -1, K_OUTPUT))
    for il in range(cfg["n_layer"]):
        for suffix, kind in LAYER_TENSORS.items():
            plan.append((f"blk.{il}.{suffix}", il, kind))
    return plan


def upload(engine, r: GGUFReader, cfg: dict) -> int:
    """Every tensor of the plan into `engine` (its weights are replaced)."""
    import arclight_b200 as A
    L = A.lib()
    n = 0
    for name, layer, kind in tensor_plan(cfg):
        if name not in r.tensors:
            raise GGUFError(f"missing tensor {name}")
        if kind in NORM_KINDS:
            w = np.ascontiguousarray(r.f32(name), dtype=np.float32).reshape(-1)
            A.check(L.alb_engine_set_norm_weights(engine.h, layer, kind, w.ctypes.data_as(C.c_void_p), w.size),
                    f"set_norm_weights({name})")
        else:
            t = r.tensors[name]
            b = np.ascontiguousarray(r.q4_0(name))
            A.check(L.alb_engine_set_weight_blocks(engine.h, layer, kind, b.ctypes.data_as(C.c_void_p),
                                                   int(t.ne[1]), int(t.ne[0])), f"set_weight_blocks({name})")
        n += 1
    return n


def engine_to_gguf(engine, path: str) -> None:
    """The weights of a single-GPU engine as a Qwen3 Q4_0 GGUF file (the
    reference's tensor names and keys; norms as F32)."""
    cfg = engine.cfg
    tensors = []
    for name, layer, kind in tensor_plan(cfg):
        if kind in NORM_KINDS:
            n = cfg["head_dim"] if kind in (K_Q_NORM, K_K_NORM) else cfg["n_embd"]
            w = np.ascontiguousarray(engine.norm_weights(layer, kind, n), dtype="<f4")
            tensors.append((name, GGML_F32, (n,), w.tobytes()))
        else:
            b = np.ascontiguousarray(engine.weight_blocks(layer, kind))
            rows, nblk = b.shape[0], b.shape[1]
            tensors.append((name, GGML_Q4_0, (nblk * 32, rows), b.tobytes()))
    write_gguf(path, qwen3_kv(cfg), tensors)


def load_qwen3(path: str, max_ctx: int, max_ubatch: int = 256, tp_rank: int = 0, tp_size: int = 1,
               nccl_id=None, device: int = 0):
    """An Engine holding the Qwen3 Q4_0 model of a GGUF file."""
    from arclight_b200.engine import Engine
    r = GGUFReader(path)
    cfg = qwen3_config(r)
    e = Engine(cfg, 0, max_ctx, max_ubatch, tp_rank, tp_size, nccl_id, device)
    upload(e, r, cfg)
    return e


# ------------------------------------------------------------------ writer
def _pack_value(v):
    if isinstance(v, bool):
        return struct.pack("<I", T_BOOL) + struct.pack("<B", int(v))
    if isinstance(v, int):
        return struct.pack("<I", T_UINT32) + struct.pack("<I", v) if 0 <= v < 2 ** 32 else \
            struct.pack("<I", T_INT64) + struct.pack("<q", v)
    if isinstance(v, float):
        return struct.pack("<I", T_FLOAT32) + struct.pack("<f", v)
    if isinstance(v, str):
        b = v.encode()
        return struct.pack("<I", T_STRING) + struct.pack("<Q", len(b)) + b
    if isinstance(v, (list, tuple)):
        if not v:
            return struct.pack("<I", T_ARRAY) + struct.pack("<IQ", T_INT32, 0)
        inner = [_pack_value(x) for x in v]
        et = struct.unpack("<I", inner[0][:4])[0]
        return struct.pack("<I", T_ARRAY) + struct.pack("<IQ", et, len(v)) + b"".join(x[4:] for x in inner)
    raise GGUFError(f"cannot write value {v!r}")


def _pack_string(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def write_gguf(path: str, kv: dict, tensors: list, alignment: int = DEFAULT_ALIGNMENT, version: int = 3):
    """tensors: (name, ttype, ne, data bytes); ne[0] innermost."""
    head = bytearray(GGUF_MAGIC + struct.pack("<IQQ", version, len(tensors), len(kv)))
    for k, v in kv.items():
        head += _pack_string(k) + _pack_value(v)
    offs, off = [], 0
    for name, tt, ne, data in tensors:
        bs, bb = _TENSOR_TYPES[tt]
        if len(data) != int(np.prod(ne)) // bs * bb:
            raise GGUFError(f"tensor {name}: {len(data)} bytes for ne {ne}")
        offs.append(off)
        off = (off + len(data) + alignment - 1) // alignment * alignment
    for (name, tt, ne, _), o in zip(tensors, offs):
        head += _pack_string(name) + struct.pack("<I", len(ne)) + b"".join(struct.pack("<Q", x) for x in ne)
        head += struct.pack("<IQ", tt, o)
    base = (len(head) + alignment - 1) // alignment * alignment
    with open(path, "wb") as f:
        f.write(head)
        f.write(b"\0" * (base - len(head)))
        pos = 0
        for (name, tt, ne, data), o in zip(tensors, offs):
            f.write(b"\0" * (o - pos))
            f.write(bytes(data))
            pos = o + len(data)


def qwen3_kv(cfg: dict) -> dict:
    """The qwen3.* keys of a configuration (for write_gguf)."""
    return {"general.architecture": "qwen3", "general.alignment": DEFAULT_ALIGNMENT,
            "qwen3.block_count": cfg["n_layer"], "qwen3.embedding_length": cfg["n_embd"],
            "qwen3.feed_forward_length": cfg["n_ff"], "qwen3.attention.head_count": cfg["n_head"],
            "qwen3.attention.head_count_kv": cfg["n_head_kv"], "qwen3.attention.key_length": cfg["head_dim"],
            "qwen3.attention.value_length": cfg["head_dim"], "qwen3.rope.freq_base": float(cfg.get("freq_base", 1e6)),
            "qwen3.attention.layer_norm_rms_epsilon": float(cfg.get("eps", 1e-6))}
