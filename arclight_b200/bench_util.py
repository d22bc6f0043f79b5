"""Helpers for bench.py: device buffers, rank barriers and max-over-ranks timing."""
from __future__ import annotations

import numpy as np


def barrier(world: int) -> None:
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(v: float, world: int) -> float:
    if world <= 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def q4_0_blocks_from_normal(N: int, K: int, seed: int, std: float = 0.02) -> np.ndarray:
    """block_q4_0 bytes [N][K/32] of W ~ N(0, std) quantized with the llama.cpp rule
    (types.cpp:352-378), vectorised in numpy (same arithmetic as the reference)."""
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((N, K // 32, 32)) * std).astype(np.float32)
    aw = np.abs(w)
    idx = np.argmax(aw, axis=2)                       # first max-abs (strict < update)
    mx = np.take_along_axis(w, idx[..., None], axis=2)[..., 0]
    d = (mx / np.float32(-8)).astype(np.float32)
    with np.errstate(divide="ignore"):
        idv = np.where(d != 0, np.float32(1.0) / d, np.float32(0)).astype(np.float32)
    q = (w * idv[..., None]).astype(np.float32) + np.float32(8.5)
    qi = np.minimum(q.astype(np.int8), 15).astype(np.uint8)   # (int8) truncation, MIN(15)
    out = np.empty((N, K // 32), dtype=[("d", "<u2"), ("qs", "u1", (16,))])
    out["d"] = d.astype(np.float16).view(np.uint16)
    out["qs"] = qi[..., :16] | (qi[..., 16:] << 4)
    return out


def make_gemv_weights(n_copies: int, N: int, K: int, seed: int):
    import torch
    import arclight_b200 as A
    L = A.lib()
    blocks = q4_0_blocks_from_normal(N, K, seed)
    src = torch.from_numpy(blocks.view(np.uint8).reshape(-1).copy()).cuda()
    s = torch.cuda.current_stream().cuda_stream
    nbytes = L.alb_q4_0_gpu_bytes(N, K)
    Ws = []
    for _ in range(n_copies):
        W = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
        A.check(L.alb_repack_q4_0(W.data_ptr(), src.data_ptr(), N, K, s), "repack")
        Ws.append(W)
    rng = np.random.default_rng(seed + 1)
    x = torch.from_numpy(rng.standard_normal(K).astype(np.float32)).cuda()
    xq = torch.empty((K // 32) * 34, dtype=torch.uint8, device="cuda")
    A.check(L.alb_quantize_q8_0(x.data_ptr(), xq.data_ptr(), K, 1, s), "quantize")
    torch.cuda.synchronize()
    return Ws, xq


def time_decode_gemvs(engine, cfg, world, rank, reps=3):
    """Mean per-launch duration / achieved GB/s of the decode step's mat-vecs."""
    import ctypes as C
    import arclight_b200 as A
    us, by = C.c_float(), C.c_double()
    A.check(A.lib().alb_engine_time_gemv(engine.h, reps, C.byref(us), C.byref(by)), "alb_engine_time_gemv")
    u = max_over_ranks(float(us.value), world)
    return {"us_per_launch": u, "bytes_per_launch": float(by.value), "gbs": float(by.value) / (u * 1e-6) / 1e9}
