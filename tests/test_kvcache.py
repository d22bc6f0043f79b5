"""KV-cache cell manager (alb_kv_* over include/alb_kvcache.h) against the
reference's own llm_kv_cache: golden scripts recorded from it
(tests/golden/make_kv_golden.py), live scripts where oracle/_ref is built, and
the properties the engine relies on.  Host code only: no GPU."""
import gzip
import json
import os

import numpy as np
import pytest

import arclight_b200 as A
from arclight_b200.kvcache import KVCache
from tests.kv_script import CONFIGS, ProductBackend, RefBackend, record, replay

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "kv_cache_golden.json.gz")


def _golden():
    with gzip.open(GOLDEN, "rt") as f:
        return json.load(f)["scripts"]


@pytest.mark.parametrize("k", range(2 * len(CONFIGS)))
def test_golden_scripts_replay_identically(k):
    """Every slot, n_kv, mask, position range and no-slot answer equals the
    reference's on the recorded scripts."""
    sc = _golden()[k]
    ops = sc["ops"]
    assert any(o["op"] == "apply" for o in ops) and any(o["op"] == "prepare" and o["out"] is None for o in ops)
    replay(ops, ProductBackend(tuple(sc["config"])))


@pytest.mark.skipif(not RefBackend.available(), reason="oracle/_ref not built (needs the reference tree)")
@pytest.mark.parametrize("cfg", CONFIGS)
def test_live_scripts_match_reference(cfg):
    for seed in range(100, 104):
        replay(record(cfg, seed, 150, RefBackend(cfg)), ProductBackend(cfg))


def _n_kv(used_max_p1, size, n_pad):
    return min(size, max(n_pad, (used_max_p1 + n_pad - 1) // n_pad * n_pad))


def test_single_sequence_cell_is_position():
    """al-gen's use: one sequence, prompt in ubatches then one token per step,
    with truncations (seq_rm(0, p, -1)) refilled from p: every token lands in
    cell == its position, which is how the engine addresses its device cache."""
    size, n_pad, n_ub = 512, 32, 64
    kv = KVCache(size, 1, True, n_pad)
    rng = np.random.default_rng(0)
    n = 0
    for it in range(40):
        if it % 7 == 6 and n > 1:   # regenerate from an earlier position
            n = int(rng.integers(1, n))
            kv.seq_rm(0, n, -1)
        k = int(rng.integers(1, 3 * n_ub)) if it % 3 == 0 else 1
        k = min(k, size - n)
        if k <= 0:
            break
        pos = np.arange(n, n + k)
        ubs = [(pos[i:i + n_ub], np.zeros(len(pos[i:i + n_ub]), np.int32)) for i in range(0, k, n_ub)]
        slots = kv.prepare(ubs)
        assert slots is not None
        for (p, s), idx in zip(ubs, slots):
            assert np.array_equal(idx, p)
            assert kv.apply(p, s, idx) == _n_kv(int(p[-1]) + 1, size, n_pad)
        n += k
        assert (kv.seq_pos_min(0), kv.seq_pos_max(0)) == (0, n - 1)
    m = kv.set_inputs_attn_mask([n - 1], [0])
    assert m.shape == (1, 64, kv.n_kv)
    assert np.all(m[0, 0, :n] == 0) and np.all(np.isneginf(m[0, 0, n:])) and np.all(np.isneginf(m[0, 1:]))


def test_no_slot_leaves_the_cells_untouched():
    kv = KVCache(64, 2, True, 32)
    p = np.arange(40)
    (idx,) = kv.prepare([(p, np.zeros(40, np.int32))])
    kv.apply(p, np.zeros(40, np.int32), idx)
    before = [kv.cell(0, i) for i in range(64)], kv.info()
    # two ubatches that fit alone but not together: all or nothing
    assert kv.prepare([(np.arange(20), np.ones(20, np.int32)), (np.arange(20, 30), np.ones(10, np.int32))]) is None
    assert kv.find_slot(np.arange(25), np.ones(25, np.int32)) is None
    assert ([kv.cell(0, i) for i in range(64)], kv.info()) == before
    assert kv.prepare([(np.arange(24), np.ones(24, np.int32))]) is not None


def test_mask_of_interleaved_sequences():
    """Two sequences sharing one stream see only their own cells at positions
    <= their own (cgraph.cpp:1224-1261); padding rows are all -inf."""
    kv = KVCache(64, 2, True, 32)
    pos = np.array([0, 0, 1, 1, 2], np.int32)
    seq = np.array([0, 1, 0, 1, 0], np.int32)
    (idx,) = kv.prepare([(pos, seq)])
    assert idx.tolist() == [0, 1, 2, 3, 4]
    assert kv.apply(pos, seq, idx) == 32
    m = kv.set_inputs_attn_mask(pos, seq)
    vis = (m[0] == 0)
    want = np.zeros((64, 32), bool)
    want[0, [0]] = want[1, [1]] = True
    want[2, [0, 2]] = want[3, [1, 3]] = True
    want[4, [0, 2, 4]] = True
    assert np.array_equal(vis, want)


def test_context_shift_moves_positions_and_frees_cells():
    kv = KVCache(64, 1, True, 32)
    p = np.arange(20, dtype=np.int32)
    (idx,) = kv.prepare([(p, np.zeros(20, np.int32))])
    kv.apply(p, np.zeros(20, np.int32), idx)
    kv.seq_rm(0, 0, 5)            # drop the first 5 positions
    kv.seq_add(0, 5, -1, -5)      # and move the rest down
    assert (kv.seq_pos_min(0), kv.seq_pos_max(0)) == (0, 14)
    assert kv.cell(0, 5) == (0, 1, -5) and kv.cell(0, 0) == (-1, 0, 0)
    assert kv.info()["used"] == 15
    # the freed cells 0..4 are found first by the next search
    assert kv.find_slot([15, 16], [0, 0]).tolist() == [0, 1]
    # a shift below zero frees the cells it moves there
    kv.seq_add(0, 0, 3, -10)
    assert kv.seq_pos_min(0) == 3 and kv.info()["used"] == 12


def test_one_stream_per_sequence_layout():
    kv = KVCache(32, 3, False, 32)
    pos = np.array([0, 1, 0, 1], np.int32)
    seq = np.array([0, 0, 2, 2], np.int32)
    (idx,) = kv.prepare([(pos, seq)])
    assert idx.tolist() == [0, 1, 2 * 32 + 0, 2 * 32 + 1]   # flat stream * kv_size + cell
    kv.apply(pos, seq, idx)
    m = kv.set_inputs_attn_mask(pos, seq, n_stream_ub=2)
    assert m.shape == (2, 64, 32)
    assert (m[1, 1] == 0).sum() == 2 and (m[0, 0] == 0).sum() == 1


def test_invalid_arguments_are_errors():
    with pytest.raises(A.AlbError):
        KVCache(100, 1, True, 32)                      # kv_size % n_pad
    kv = KVCache(32, 2, False, 32)
    with pytest.raises(A.AlbError):
        kv.find_slot([0, 1, 2], [0, 0, 1])             # unequal runs with one stream per sequence
    with pytest.raises(A.AlbError):
        kv.find_slot([0], [5])                         # sequence id beyond the streams
    with pytest.raises(A.AlbError):
        kv.find_slot(np.arange(40), np.zeros(40))      # larger than the cache
    with pytest.raises(A.AlbError):
        kv.apply([0, 1], [0, 0], [3, 3])               # a cell given twice
    with pytest.raises(A.AlbError):
        kv.seq_rm(7, 0, -1)


def test_overwrite_purges_the_sequence_up_to_the_lost_position():
    """apply_ubatch (cgraph.cpp:1420-1468): writing over cell 3 (position 3 of
    sequence 0) drops position 3 and every earlier position of sequence 0."""
    kv = KVCache(64, 1, True, 32)
    p = np.arange(10, dtype=np.int32)
    (idx,) = kv.prepare([(p, np.zeros(10, np.int32))])
    kv.apply(p, np.zeros(10, np.int32), idx)
    kv.apply([10], [0], [3])
    assert (kv.seq_pos_min(0), kv.seq_pos_max(0)) == (4, 10)
    assert [kv.cell(0, i)[0] for i in range(11)] == [-1, -1, -1, 10, 4, 5, 6, 7, 8, 9, -1]
    assert kv.info()["used"] == 7 and kv.info()["head"] == 4


@pytest.mark.parametrize("cfg", CONFIGS)
def test_visible_cells_are_the_mask_rows(cfg):
    b = ProductBackend(cfg)
    record(cfg, 5, 80, b)
    kv = b.kv
    for s in range(cfg[1]):
        st = 0 if cfg[2] else s
        for p in (0, 7, 40, 500):
            row = kv.set_inputs_attn_mask([p], [s], 1, kv.kv_size)[0, 0]
            want = st * kv.kv_size + np.nonzero(row == 0)[0]
            assert np.array_equal(kv.visible_cells(s, p, kv.kv_size), want)
