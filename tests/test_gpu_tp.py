"""Tensor-parallel engine (one process per GPU) against the oracle run with the
reference's tensor-parallel semantics on the same seeded model.

The reference splits the O and down projections over the nodes by input
columns and adds the node partials in node order (GATHER, ops.cpp:1465-1511)
before the residual ADD; the GPU ranks all-gather their partials and add them
in rank order, so the result is the oracle's `set_tp(tp)` model bit for bit:
greedy tokens for 32 steps and the last logits are compared exactly.  (Against
the single-GPU model the partials' fp32 rounding moves logits by a few 1e-2,
the same order-sensitivity the reference's own TP has.)  Needs >= 2 GPUs.
"""
import multiprocessing as mp
import os

import numpy as np
import pytest

from arclight_b200.configs import QWEN3_0_6B, TINY_GQA
from oracle import lib as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

STEPS = 32


def _rank_main(cfg, seed, tp, rank, nid, prompt, q):
    try:
        from arclight_b200.engine import Engine
        e = Engine(cfg, seed, len(prompt) + STEPS + 8, 64, rank, tp, nid, rank)
        tok = e.prefill(prompt, 0)
        toks = [tok]
        for i in range(STEPS - 1):
            tok = e.decode(tok, len(prompt) + i)
            toks.append(tok)
        q.put((rank, toks, e.logits(), e.info()))
        e.close()
    except Exception as ex:   # reported to the parent, which fails the test
        q.put((rank, None, repr(ex), None))


def _run_tp(cfg, seed, tp, prompt):
    from arclight_b200.engine import nccl_unique_id
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    nid = nccl_unique_id()
    procs = [ctx.Process(target=_rank_main, args=(cfg, seed, tp, r, nid, prompt, q)) for r in range(tp)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(tp):
            r, toks, lg, info = q.get(timeout=600)
            assert toks is not None, f"rank {r}: {lg}"
            res[r] = (toks, lg, info)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    return res


@pytest.mark.parametrize("cfg,tp", [(TINY_GQA, 2), (QWEN3_0_6B, 2)], ids=["tiny_gqa_tp2", "qwen3_0.6b_tp2"])
def test_tp_matches_oracle_tp(cfg, tp):
    if torch.cuda.device_count() < tp:
        pytest.skip(f"needs {tp} GPUs")
    os.environ.setdefault("NCCL_DEBUG", "WARN")
    seed = 23
    prompt = np.random.default_rng(seed).integers(0, cfg["n_vocab"], 48).astype(np.int32)
    res = _run_tp(cfg, seed, tp, prompt)
    m = O.Model(cfg, seed, len(prompt) + STEPS + 8, os.cpu_count() or 8)
    try:
        m.set_tp(tp)
        lg, _ = m.forward(prompt, 0)
        ref = [O.argmax(lg)]
        for i in range(STEPS - 1):
            lg, _ = m.forward([ref[-1]], len(prompt) + i)
            ref.append(O.argmax(lg))
    finally:
        m.close()
    for r in range(tp):
        assert res[r][0] == ref, f"rank {r} tokens differ from the oracle"
    logits = np.concatenate([res[r][1] for r in range(tp)])   # vocabulary shards in rank order
    assert logits.shape == lg.shape
    np.testing.assert_array_equal(logits, lg)


def _comm_rank_main(rank, size, nid, q):
    try:
        import ctypes as C
        import torch as T
        import arclight_b200 as A
        L = A.lib()
        T.cuda.set_device(rank)
        comm = C.c_void_p()
        A.check(L.alb_comm_create(nid, rank, size, rank, C.byref(comm)), "alb_comm_create")
        n = 10240
        x = T.arange(n, dtype=T.float32, device="cuda") * (rank + 1) + 0.25
        red = T.empty_like(x)
        gat = T.empty(size * n, dtype=T.float32, device="cuda")
        s = T.cuda.current_stream().cuda_stream
        A.check(L.alb_allreduce_sum_f32(comm, x.data_ptr(), red.data_ptr(), n, s), "allreduce")
        A.check(L.alb_allgather_f32(comm, x.data_ptr(), gat.data_ptr(), n, s), "allgather")
        T.cuda.synchronize()
        q.put((rank, red.cpu().numpy(), gat.cpu().numpy()))
        A.check(L.alb_comm_destroy(comm), "alb_comm_destroy")
    except Exception as ex:
        q.put((rank, None, repr(ex)))


def test_comm_allreduce_and_allgather():
    """The op-level communicator ABI: sum all-reduce and rank-ordered all-gather."""
    size = 2
    if torch.cuda.device_count() < size:
        pytest.skip(f"needs {size} GPUs")
    from arclight_b200.engine import nccl_unique_id
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    nid = nccl_unique_id()
    procs = [ctx.Process(target=_comm_rank_main, args=(r, size, nid, q)) for r in range(size)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(size):
            r, red, gat = q.get(timeout=300)
            assert red is not None, f"rank {r}: {gat}"
            res[r] = (red, gat)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    n = 10240
    parts = [np.arange(n, dtype=np.float32) * (r + 1) + np.float32(0.25) for r in range(size)]
    for r in range(size):
        np.testing.assert_array_equal(res[r][0], parts[0] + parts[1])
        np.testing.assert_array_equal(res[r][1], np.concatenate(parts))
