"""GGUF load path on the GPU: a seeded engine's weights written as a GGUF file
and loaded into an engine built from another seed give the same weights and
the same logits and greedy tokens, bit for bit."""
import numpy as np
import pytest

from arclight_b200 import gguf as G
from arclight_b200.configs import TINY, TINY_GQA

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("cfg", [TINY, TINY_GQA], ids=["tied", "untied_gqa"])
def test_gguf_round_trip_engine(tmp_path, cfg):
    from arclight_b200.engine import Engine
    a = Engine(cfg, 77, 96, 32)
    path = str(tmp_path / "m.gguf")
    G.engine_to_gguf(a, path)
    b = G.load_qwen3(path, 96, 32)
    assert b.cfg["n_vocab"] == cfg["n_vocab"] and bool(b.cfg["tied"]) == bool(cfg["tied"])
    for name, layer, kind in G.tensor_plan(b.cfg):
        if kind in G.NORM_KINDS:
            n = cfg["head_dim"] if kind in (G.K_Q_NORM, G.K_K_NORM) else cfg["n_embd"]
            np.testing.assert_array_equal(a.norm_weights(layer, kind, n), b.norm_weights(layer, kind, n), err_msg=name)
        else:
            assert a.weight_blocks(layer, kind).tobytes() == b.weight_blocks(layer, kind).tobytes(), name
    prompt = np.random.default_rng(5).integers(0, cfg["n_vocab"], 20).astype(np.int32)
    ta, tb = a.prefill(prompt, 0), b.prefill(prompt, 0)
    assert ta == tb
    np.testing.assert_array_equal(a.logits(), b.logits())
    ga = a.decode_loop(ta, 20, 12)
    gb = b.decode_loop(tb, 20, 12)
    np.testing.assert_array_equal(ga, gb)
    np.testing.assert_array_equal(a.logits(), b.logits())
