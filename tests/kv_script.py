"""Seeded operation scripts for the KV-cache cell manager, run against either
the product (``arclight_b200.kvcache.KVCache`` over ``alb_kv_*``) or the
reference's own ``llm_kv_cache`` (``oracle/_ref/libalref.so``, built from the
reference sources by ``oracle/Makefile``).  A script is the sequence of calls
the reference's decode loop makes (context.cpp:85-129 and 211-236: prepare
the ubatches, then apply each and build its mask), with sequence removals,
position shifts, contiguous slot searches and position queries in between.
Recorded scripts (arguments and outputs) are the golden fixtures."""
from __future__ import annotations

import ctypes as C
import hashlib
import os

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_LIB = os.path.join(ROOT, "oracle", "_ref", "libalref.so")
NO_SLOT = -7

# (kv_size, n_seq_max, unified, n_pad): one sequence as al-gen runs it
# (al-gen.cpp:114-116), several sequences in one stream, one stream per sequence
CONFIGS = [(64, 1, True, 32), (128, 4, True, 32), (96, 3, False, 32), (256, 2, True, 256)]


def mask_digest(m: np.ndarray) -> tuple[str, int]:
    """(sha256 of the visible-cell bits, visible cells); every entry must be 0 or -inf."""
    vis = m == 0.0
    assert np.all(vis | np.isneginf(m)), "mask values other than 0 and -inf"
    return hashlib.sha256(np.packbits(vis.reshape(-1)).tobytes()).hexdigest()[:32], int(vis.sum())


class ProductBackend:
    def __init__(self, cfg):
        from arclight_b200.kvcache import KVCache
        kv_size, n_seq_max, unified, n_pad = cfg
        self.kv = KVCache(kv_size, n_seq_max, unified, n_pad)

    def prepare(self, ubs):
        r = self.kv.prepare(ubs)
        return None if r is None else [x.tolist() for x in r]

    def find_slot(self, pos, seq, cont):
        r = self.kv.find_slot(pos, seq, cont)
        return None if r is None else r.tolist()

    def apply(self, pos, seq, idxs):
        return self.kv.apply(pos, seq, idxs)

    def mask(self, pos, seq, n_stream_ub, n_kv):
        return self.kv.set_inputs_attn_mask(pos, seq, n_stream_ub, n_kv)

    def seq_rm(self, s, p0, p1):
        self.kv.seq_rm(s, p0, p1)

    def seq_add(self, s, p0, p1, d):
        self.kv.seq_add(s, p0, p1, d)

    def pos_range(self, s):
        return [self.kv.seq_pos_min(s), self.kv.seq_pos_max(s)]


class RefBackend:
    """The reference's llm_kv_cache through oracle/ref_kv_driver.cpp (checker only)."""
    _L = None

    @classmethod
    def available(cls) -> bool:
        return os.path.exists(REF_LIB)

    @classmethod
    def lib(cls):
        if cls._L is None:
            L = C.CDLL(REF_LIB)
            vp, i32, u32 = C.c_void_p, C.c_int32, C.c_uint32
            L.refkv_create.restype = vp
            L.refkv_create.argtypes = [u32, u32, C.c_int, u32]
            L.refkv_destroy.argtypes = [vp]
            L.refkv_find_slot.argtypes = [vp, vp, vp, C.c_int, C.c_int, vp]
            L.refkv_prepare.argtypes = [vp, vp, C.c_int, vp, vp, vp]
            L.refkv_apply.argtypes = [vp, vp, vp, C.c_int, vp, vp]
            L.refkv_seq_rm.argtypes = [vp, C.c_int, C.c_int, C.c_int]
            L.refkv_seq_add.argtypes = [vp, C.c_int, C.c_int, C.c_int, C.c_int]
            L.refkv_seq_pos_range.argtypes = [vp, C.c_int, vp, vp]
            L.refkv_mask.argtypes = [vp, vp, vp, C.c_int, C.c_int, u32, vp]
            cls._L = L
        return cls._L

    def __init__(self, cfg):
        kv_size, n_seq_max, unified, n_pad = cfg
        self.L = self.lib()
        self.h = self.L.refkv_create(kv_size, n_seq_max, int(unified), n_pad)
        self.kv_size = kv_size

    def __del__(self):
        if getattr(self, "h", None):
            self.L.refkv_destroy(self.h)

    @staticmethod
    def _a(x, dt=np.int32):
        return np.ascontiguousarray(np.asarray(x, dtype=dt).reshape(-1))

    def prepare(self, ubs):
        sizes = self._a([len(p) for p, _ in ubs])
        pos = self._a(np.concatenate([p for p, _ in ubs]))
        seq = self._a(np.concatenate([s for _, s in ubs]))
        out = np.zeros(len(pos), dtype=np.int64)
        rc = self.L.refkv_prepare(self.h, sizes.ctypes.data, len(sizes), pos.ctypes.data, seq.ctypes.data,
                                  out.ctypes.data)
        if rc == NO_SLOT:
            return None
        return [x.tolist() for x in np.split(out, np.cumsum(sizes)[:-1])]

    def find_slot(self, pos, seq, cont):
        p, s = self._a(pos), self._a(seq)
        out = np.zeros(len(p), dtype=np.int64)
        rc = self.L.refkv_find_slot(self.h, p.ctypes.data, s.ctypes.data, len(p), int(cont), out.ctypes.data)
        return None if rc == NO_SLOT else out.tolist()

    def apply(self, pos, seq, idxs):
        p, s, ix = self._a(pos), self._a(seq), self._a(idxs, np.int64)
        n_kv = C.c_uint32()
        self.L.refkv_apply(self.h, p.ctypes.data, s.ctypes.data, len(p), ix.ctypes.data, C.byref(n_kv))
        return n_kv.value

    def mask(self, pos, seq, n_stream_ub, n_kv):
        p, s = self._a(pos), self._a(seq)
        rows = (len(p) // n_stream_ub + 63) // 64 * 64
        out = np.empty((n_stream_ub, rows, n_kv), dtype=np.float32)
        self.L.refkv_mask(self.h, p.ctypes.data, s.ctypes.data, len(p), n_stream_ub, n_kv, out.ctypes.data)
        return out

    def seq_rm(self, s, p0, p1):
        self.L.refkv_seq_rm(self.h, s, p0, p1)

    def seq_add(self, s, p0, p1, d):
        self.L.refkv_seq_add(self.h, s, p0, p1, d)

    def pos_range(self, s):
        lo, hi = C.c_int32(), C.c_int32()
        self.L.refkv_seq_pos_range(self.h, s, C.byref(lo), C.byref(hi))
        return [lo.value, hi.value]


def _ubatch(rng, cfg, nxt):
    """One ubatch: (pos list, seq list, streams in the ubatch).  Positions
    continue each sequence from nxt[s] (its last position + 1)."""
    kv_size, n_seq_max, unified, _ = cfg
    k = int(rng.integers(1, n_seq_max + 1))
    seqs = sorted(rng.choice(n_seq_max, size=k, replace=False).tolist())
    if unified:
        pos, seq = [], []
        for s in seqs:
            n = int(rng.integers(1, max(2, kv_size // 6)))
            pos += list(range(nxt[s], nxt[s] + n))
            seq += [s] * n
            nxt[s] += n
        if rng.random() < 0.3:   # tokens of the sequences interleaved
            order = rng.permutation(len(pos))
            pos, seq = [pos[i] for i in order], [seq[i] for i in order]
        return pos, seq, 1
    n = int(rng.integers(1, max(2, kv_size // 8)))   # equal runs, one per sequence
    pos, seq = [], []
    for s in seqs:
        pos += list(range(nxt[s], nxt[s] + n))
        seq += [s] * n
        nxt[s] += n
    return pos, seq, len(seqs)


def record(cfg, seed: int, n_ops: int, backend) -> list[dict]:
    """Run a seeded script on `backend`, recording every call and its result."""
    rng = np.random.default_rng(seed)
    n_seq_max = cfg[1]
    ops = []
    full = False
    used = set()   # flat cells some apply has written
    kv_size = cfg[0]
    for _ in range(n_ops):
        nxt = [max(backend.pos_range(s)[1] + 1, 0) for s in range(n_seq_max)]
        r = rng.random()
        if full and rng.random() < 0.7:
            # make room: drop a sequence's tail, or shift it as a context shift
            # does (drop its first k positions, move the rest down by k)
            s = int(rng.integers(0, n_seq_max))
            k = int(rng.integers(1, max(2, nxt[s])))
            if rng.random() < 0.5:
                backend.seq_rm(s, k, -1)
                ops.append({"op": "seq_rm", "args": [s, k, -1]})
            else:
                backend.seq_rm(s, 0, k)
                backend.seq_add(s, k, -1, -k)
                ops.append({"op": "seq_rm", "args": [s, 0, k]})
                ops.append({"op": "seq_add", "args": [s, k, -1, -k]})
            full = False
            continue
        if r < 0.5:
            ubs = [_ubatch(rng, cfg, nxt) for _ in range(int(rng.integers(1, 4)))]
            out = backend.prepare([(p, s) for p, s, _ in ubs])
            ops.append({"op": "prepare", "ubatches": [[p, s] for p, s, _ in ubs], "out": out})
            full = out is None
            if out is None:
                continue
            for (p, s, ns), idxs in zip(ubs, out):
                used.update(idxs)
                n_kv = backend.apply(p, s, idxs)
                dig = mask_digest(backend.mask(p, s, ns, n_kv))
                ops.append({"op": "apply", "pos": p, "seq": s, "idxs": idxs, "n_kv": n_kv,
                            "n_stream_ub": ns, "mask": list(dig)})
        elif r < 0.56 and used:
            # a ubatch of one sequence written over cells used before (apply
            # without prepare): the overwritten sequences lose those positions
            # and every earlier one (apply_ubatch's purge)
            s = int(rng.integers(0, n_seq_max))
            pool = sorted(c for c in used if cfg[2] or c // kv_size == s)
            n = min(len(pool), int(rng.integers(1, 5)))
            if n == 0:
                continue
            idxs = sorted(int(c) for c in rng.choice(pool, size=n, replace=False))
            p = list(range(nxt[s], nxt[s] + n))
            n_kv = backend.apply(p, [s] * n, idxs)
            dig = mask_digest(backend.mask(p, [s] * n, 1, n_kv))
            ops.append({"op": "apply", "pos": p, "seq": [s] * n, "idxs": idxs, "n_kv": n_kv,
                        "n_stream_ub": 1, "mask": list(dig)})
        elif r < 0.65:
            s = int(rng.integers(-1, n_seq_max)) if rng.random() < 0.2 else int(rng.integers(0, n_seq_max))
            hi = max(nxt) + 2
            p0 = int(rng.integers(-1, hi))
            p1 = -1 if rng.random() < 0.5 else int(rng.integers(p0 + 1 if p0 >= 0 else 0, hi + 1))
            backend.seq_rm(s, p0, p1)
            ops.append({"op": "seq_rm", "args": [s, p0, p1]})
        elif r < 0.75:
            s = int(rng.integers(0, n_seq_max))
            hi = max(nxt) + 2
            p0 = int(rng.integers(-1, hi))
            p1 = -1 if rng.random() < 0.5 else int(rng.integers(max(p0, 0), hi + 1))
            d = int(rng.integers(-hi, hi // 2 + 2))
            backend.seq_add(s, p0, p1, d)
            ops.append({"op": "seq_add", "args": [s, p0, p1, d]})
        elif r < 0.85:
            p, s, _ = _ubatch(rng, cfg, list(nxt))
            ops.append({"op": "find_slot", "pos": p, "seq": s, "cont": 1,
                        "out": backend.find_slot(p, s, True)})
        else:
            ops.append({"op": "pos_range", "out": [backend.pos_range(s) for s in range(n_seq_max)]})
    return ops


def replay(ops: list[dict], backend) -> None:
    """Re-run recorded calls on `backend`; assert every result equals the record."""
    for i, o in enumerate(ops):
        k = o["op"]
        if k == "prepare":
            got = backend.prepare([(p, s) for p, s in o["ubatches"]])
            assert got == o["out"], f"op {i} prepare: {got} != {o['out']}"
        elif k == "apply":
            n_kv = backend.apply(o["pos"], o["seq"], o["idxs"])
            assert n_kv == o["n_kv"], f"op {i} apply n_kv {n_kv} != {o['n_kv']}"
            dig = list(mask_digest(backend.mask(o["pos"], o["seq"], o["n_stream_ub"], n_kv)))
            assert dig == o["mask"], f"op {i} mask differs ({dig[1]} vs {o['mask'][1]} visible)"
        elif k == "seq_rm":
            backend.seq_rm(*o["args"])
        elif k == "seq_add":
            backend.seq_add(*o["args"])
        elif k == "find_slot":
            got = backend.find_slot(o["pos"], o["seq"], bool(o["cont"]))
            assert got == o["out"], f"op {i} find_slot: {got} != {o['out']}"
        elif k == "pos_range":
            got = [backend.pos_range(s) for s in range(len(o["out"]))]
            assert got == o["out"], f"op {i} pos_range: {got} != {o['out']}"
