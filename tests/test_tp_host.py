"""Host plumbing of the multi-GPU bench (gloo ranks on the CPU, world size 2):
the NCCL unique id travels from rank 0 to every rank, the timing is the max over
ranks, and a rank that stops taking part makes the others fail with an error instead of
waiting for ever (short process-group timeout)."""
import datetime
import multiprocessing as mp
import os
import socket

import pytest


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, mode, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    try:
        import torch.distributed as dist
        from arclight_b200 import bench_util as BU
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=5))
        if mode == "ok":
            obj = [bytes(range(128)) if rank == 0 else None]
            dist.broadcast_object_list(obj, src=0)        # how bench.py ships the NCCL unique id
            BU.barrier(world)
            m = BU.max_over_ranks(0.5 + rank, world)
            q.put((rank, "ok", obj[0] == bytes(range(128)), m))
        else:  # rank 1 never joins the collective; rank 0 must get an error after the timeout
            if rank == 1:
                q.put((rank, "left", None, None))
                import time
                time.sleep(12)
                os._exit(0)
            try:
                BU.barrier(world)
                q.put((rank, "no-error", None, None))
            except Exception as ex:
                q.put((rank, "error", type(ex).__name__, None))
        dist.destroy_process_group()
    except Exception as ex:
        q.put((rank, "exception", repr(ex), None))


def _spawn(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in range(2):
            r, status, a, b = q.get(timeout=60)
            out[r] = (status, a, b)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    return out


def test_id_broadcast_barrier_and_max_over_ranks():
    out = _spawn("ok")
    for r in range(2):
        status, id_ok, m = out[r]
        assert status == "ok", out[r]
        assert id_ok
        assert m == pytest.approx(1.5)


def test_rank_that_leaves_turns_into_an_error():
    out = _spawn("leave")
    assert out[1][0] == "left"
    assert out[0][0] == "error", out[0]
