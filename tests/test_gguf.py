"""GGUF files on the CPU: the writer and reader agree, the Qwen3 configuration
and tensor plan follow the reference's keys and names (models/qwen3.cpp:7-45),
and malformed files are rejected (model.cpp:130-335 is the reference reader)."""
import struct

import numpy as np
import pytest

from arclight_b200 import gguf as G
from arclight_b200.configs import TINY, TINY_GQA


def _tiny_file(path, cfg, rng, alignment=32, extra_kv=None):
    kv = G.qwen3_kv(cfg)
    kv["general.alignment"] = alignment
    kv.update(extra_kv or {})
    tensors = []
    for name, layer, kind in G.tensor_plan(cfg):
        if kind in G.NORM_KINDS:
            n = cfg["head_dim"] if kind in (G.K_Q_NORM, G.K_K_NORM) else cfg["n_embd"]
            tensors.append((name, G.GGML_F32, (n,), rng.standard_normal(n).astype("<f4").tobytes()))
        else:
            rows, cols = {G.K_TOK_EMBD: (cfg["n_vocab"], cfg["n_embd"]), G.K_OUTPUT: (cfg["n_vocab"], cfg["n_embd"]),
                          G.K_WQ: (cfg["n_head"] * 128, cfg["n_embd"]), G.K_WK: (cfg["n_head_kv"] * 128, cfg["n_embd"]),
                          G.K_WV: (cfg["n_head_kv"] * 128, cfg["n_embd"]), G.K_WO: (cfg["n_embd"], cfg["n_head"] * 128),
                          G.K_GATE: (cfg["n_ff"], cfg["n_embd"]), G.K_UP: (cfg["n_ff"], cfg["n_embd"]),
                          G.K_DOWN: (cfg["n_embd"], cfg["n_ff"])}[kind]
            data = rng.integers(0, 256, rows * cols // 32 * 18, dtype=np.uint8).tobytes()
            tensors.append((name, G.GGML_Q4_0, (cols, rows), data))
    G.write_gguf(str(path), kv, tensors, alignment=alignment)
    return kv, tensors


@pytest.mark.parametrize("cfg,alignment", [(TINY, 32), (TINY_GQA, 64)])
def test_round_trip(tmp_path, cfg, alignment):
    rng = np.random.default_rng(3)
    p = tmp_path / "m.gguf"
    kv, tensors = _tiny_file(p, cfg, rng, alignment, {"test.list": [1, 2, 3], "test.flag": True, "test.name": "x"})
    r = G.GGUFReader(str(p))
    assert r.version == 3
    assert r.kv["test.list"] == [1, 2, 3] and r.kv["test.flag"] is True and r.kv["test.name"] == "x"
    assert set(r.tensors) == {t[0] for t in tensors}
    for name, tt, ne, data in tensors:
        t = r.tensors[name]
        assert t.ne == tuple(ne) and t.ttype == tt and t.offset % alignment == 0
        assert bytes(r.raw(name)) == data
    c = G.qwen3_config(r)
    for k in ("n_layer", "n_embd", "n_head", "n_head_kv", "head_dim", "n_ff", "n_vocab"):
        assert c[k] == cfg[k]
    assert c["tied"] == bool(cfg["tied"])
    name = "blk.1.ffn_down.weight"
    assert r.q4_0(name).shape == (cfg["n_embd"], cfg["n_ff"] // 32 * 18)
    assert r.f32("blk.0.attn_q_norm.weight").shape == (128,)


def test_tensor_plan_names():
    plan = G.tensor_plan(TINY_GQA)
    names = {n for n, _, _ in plan}
    assert {"token_embd.weight", "output.weight", "output_norm.weight", "blk.2.attn_k_norm.weight",
            "blk.0.ffn_gate.weight"} <= names
    assert len(plan) == 3 + 11 * TINY_GQA["n_layer"]
    assert "output.weight" not in {n for n, _, _ in G.tensor_plan(TINY)}   # tied embeddings


def test_rejects_malformed(tmp_path):
    rng = np.random.default_rng(4)
    p = tmp_path / "m.gguf"
    _tiny_file(p, TINY, rng)
    raw = p.read_bytes()
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGUX" + raw[4:])
    with pytest.raises(G.GGUFError, match="not a GGUF"):
        G.GGUFReader(str(bad))
    bad.write_bytes(raw[:4] + struct.pack("<I", 9) + raw[8:])
    with pytest.raises(G.GGUFError, match="version"):
        G.GGUFReader(str(bad))
    bad.write_bytes(raw[: len(raw) // 2])
    with pytest.raises(G.GGUFError):
        G.GGUFReader(str(bad))
    # a missing configuration key
    G.write_gguf(str(bad), {"general.architecture": "qwen3"}, [("token_embd.weight", G.GGML_F32, (4,), b"\0" * 16)])
    with pytest.raises(G.GGUFError, match="missing key"):
        G.qwen3_config(G.GGUFReader(str(bad)))
    # an unsupported tensor type (Q8_0 = 8)
    G.write_gguf(str(bad), {}, [("t", G.GGML_F32, (4,), b"\0" * 16)])
    data = bytearray(bad.read_bytes())
    i = data.index(b"t", 24)   # the tensor info: name, n_dims, ne, type
    struct.pack_into("<I", data, i + 1 + 4 + 8, 8)
    bad.write_bytes(bytes(data))
    with pytest.raises(G.GGUFError, match="unsupported type"):
        G.GGUFReader(str(bad))
