#!/usr/bin/env python3
"""ArcLight B200 hot-path benchmark (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload decode|gemv|prefill|long|attn] [--impl ours|reference]

Workloads:
  decode  config 3 (default): Qwen3-4B-shaped Q4_0 model, random init, 512-token
          uniform random prompt, then greedy batch-1 decode; a step is one token
          (one CUDA-graph replay).  N > 1: tensor parallel over N GPUs (NCCL).
  gemv    config 1: one Q4_0 x Q8_0 mat-vec, W [9728 x 2560]; a step is one
          launch over one of 24 distinct weight copies (336 MB > 126 MB L2).
  prefill config 4: the same model prefilling a 2048-token prompt from an empty
          cache; a step is one prompt (time to first token); the mat-muls run on
          the int8 tensor cores.
  long    config 5: Qwen3-8B shape, KV cache filled to 32768 positions, then
          batch-1 decode; a step is one token; N > 1: tensor parallel.
  attn    config 5's attention alone: split-K flash decode of one token over
          32768 fp16 cells (32 query / 8 KV heads); a step is one call.
Metric / value / roofline: value is whole-job tok/s with inputs resident; e2e goes through the C ABI with host buffers; roofline.achieved = algorithmic bytes per launch / CUDA-event launch time.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "src": "fallback"}


def host_cpu():
    """Model name, logical CPUs and NUMA nodes of the host (for cpu_baseline)."""
    model = None
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    try:
        numa = len([d for d in os.listdir("/sys/devices/system/node") if d.startswith("node") and d[4:].isdigit()])
    except OSError:
        numa = None
    return {"model": model, "logical_cpus": os.cpu_count(), "numa_nodes": numa}


DTYPE_DECODE = ("q4_0 weights x q8_0 activations: int32 block dots in the reference's fp32 chains; "
                "attention fp32 scores and chunk sums, fp64 chunk merge; fp16 KV")


# ----------------------------------------------------------------- clocks
class ClockSampler:
    """Samples nvidia-smi SM clocks and throttle reasons during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.samples = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                self.samples.append(parts)

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4) if s[5 + i].lower() == "active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples)}


# ----------------------------------------------------------------- GEMV (config 1)
GEMV_N, GEMV_K = 9728, 2560
GEMV_BYTES = GEMV_N * (GEMV_K // 32) * 18 + (GEMV_K // 32) * 34 + GEMV_N * 4  # 14 049 952
# DRAM bytes (read + write) of one config-1 launch from an ncu capture; None until captured
GEMV_TRAFFIC = None
GEMV_TRAFFIC_SRC = "ncu dram__bytes_read.sum + dram__bytes_write.sum of one k_mv launch (config 1)"


def cpu_gemv_baseline(seconds: float = 12.0):
    """The oracle mat-vec (reference semantics, all host threads) on a bounded sample."""
    from oracle import lib as O
    rng = np.random.default_rng(1)
    wq = O.quantize_q4_0((rng.standard_normal((GEMV_N, GEMV_K)) * 0.02).astype(np.float32))
    xq = O.quantize_q8_0(rng.standard_normal(GEMV_K).astype(np.float32))
    threads = os.cpu_count() or 1
    O.gemv(wq, xq, threads)
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        O.gemv(wq, xq, threads)
        n += 1
    dt = (time.perf_counter() - t0) / n
    return {"value": GEMV_BYTES / dt / 1e9, "unit": "GB/s", "cores": threads, "kind": "port", "cpu": host_cpu(),
            "sample": f"{n} mat-vecs of config 1 ({GEMV_N}x{GEMV_K}) in {seconds:.0f} s"}


def gemv_graph(L, A, Ws, xqs, y, n_copies):
    """One CUDA graph = one pass over the weight copies (n_copies launches, PDL edges)."""
    import torch
    g = torch.cuda.CUDAGraph()
    cap = torch.cuda.Stream()
    with torch.cuda.stream(cap):
        for i in range(n_copies):   # untimed eager pass (also sets kernel attributes)
            A.check(L.alb_gemv_q4_0_q8_0(Ws[i].data_ptr(), xqs.data_ptr(), y.data_ptr(), GEMV_N, GEMV_K, None,
                                         cap.cuda_stream))
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=cap):
            for i in range(n_copies):
                A.check(L.alb_gemv_q4_0_q8_0(Ws[i].data_ptr(), xqs.data_ptr(), y.data_ptr(), GEMV_N, GEMV_K,
                                             None, cap.cuda_stream))
    return g


def gemv_config1_record(reps: int = 40):
    """Config 1 (one Q4_0 x Q8_0 mat-vec, W 9728 x 2560) timed on this GPU: 24
    rotating weight copies (336 MB > L2) replayed from one CUDA graph; mean
    CUDA-event time per launch and algorithmic GB/s."""
    import torch
    import arclight_b200 as A
    from arclight_b200 import bench_util as BU
    L = A.lib()
    n_copies = 24
    Ws, xqs = BU.make_gemv_weights(n_copies, GEMV_N, GEMV_K, seed=1234)
    y = torch.empty(GEMV_N, dtype=torch.float32, device="cuda")
    g = gemv_graph(L, A, Ws, xqs, y, n_copies)
    s = torch.cuda.current_stream()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(reps):
        g.replay()
    e1.record(s)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (reps * n_copies)
    peaks = load_peaks()
    gbs = GEMV_BYTES / (us * 1e-6) / 1e9
    del Ws, g
    torch.cuda.empty_cache()
    return {"workload": "config1_gemv", "kernel": "k_mv (Q4_0 x Q8_0 mat-vec, W 9728x2560)", "us_per_launch": us,
            "algorithmic_bytes_per_launch": GEMV_BYTES, "achieved_gbs": gbs, "peak_gbs": peaks["hbm_gbs"],
            "frac": gbs / peaks["hbm_gbs"], "launches": reps * n_copies,
            "l2": "24 rotating weight copies (336 MB > 126 MB L2)"}


def run_gemv(args, rank, world):
    import torch
    import arclight_b200 as A
    from arclight_b200 import bench_util as BU
    L = A.lib()
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    A.check(L.alb_device_check(dev.index), "device check")
    s = torch.cuda.current_stream()
    n_copies = 24
    Ws, xqs = BU.make_gemv_weights(n_copies, GEMV_N, GEMV_K, seed=1234)
    y = torch.empty(GEMV_N, dtype=torch.float32, device=dev)

    g = gemv_graph(L, A, Ws, xqs, y, n_copies)
    reps = max(1, args.steps // n_copies)
    steps = reps * n_copies
    with ClockSampler(dev.index) as clk:
        t_end = time.time() + 0.6          # warm-up: >= W graph replays and >= 0.6 s under load
        w = 0
        while w < args.warmup or time.time() < t_end:
            g.replay()
            w += 1
        torch.cuda.synchronize()
        BU.barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.nvtx.range_push("timed")   # lets ncu --nvtx-include timed/ list exactly these launches
        e0.record(s)
        for _ in range(reps):
            g.replay()
        e1.record(s)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    ms = BU.max_over_ranks(ms, world)
    launch_us = ms * 1e3
    args.steps = steps

    # e2e through the C ABI with host buffers: H2D x, quantize, gemv, D2H y
    xh = torch.randn(GEMV_K, dtype=torch.float32).pin_memory()
    yh = torch.empty(GEMV_N, dtype=torch.float32).pin_memory()
    xd = torch.empty(GEMV_K, dtype=torch.float32, device=dev)
    xqd = torch.empty((GEMV_K // 32) * 34, dtype=torch.uint8, device=dev)

    def e2e_step(i):
        xd.copy_(xh, non_blocking=True)
        A.check(L.alb_quantize_q8_0(xd.data_ptr(), xqd.data_ptr(), GEMV_K, 1, s.cuda_stream))
        A.check(L.alb_gemv_q4_0_q8_0(Ws[i % n_copies].data_ptr(), xqd.data_ptr(), y.data_ptr(),
                                     GEMV_N, GEMV_K, None, s.cuda_stream))
        yh.copy_(y, non_blocking=True)

    for i in range(args.warmup):
        e2e_step(i)
    torch.cuda.synchronize()
    e0.record(s)
    for i in range(args.steps):
        e2e_step(i)
    e1.record(s)
    torch.cuda.synchronize()
    e2e_ms = BU.max_over_ranks(e0.elapsed_time(e1) / args.steps, world)

    peaks = load_peaks()
    achieved = GEMV_BYTES / (launch_us * 1e-6) / 1e9
    out = {
        "metric": "Q4_0xQ8_0 GEMV HBM GB/s (config 1, W 9728x2560)",
        "value": achieved * world, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "q4_0 x q8_0 -> int32 block dots, the reference's fp32 block chain",
        "data": "synthetic",
        "config": {"workload": "config1_gemv", "N": GEMV_N, "K": GEMV_K, "weight_copies": n_copies,
                   "l2": "inputs larger than L2: 24 rotating weight copies (336 MB)"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / peaks["hbm_gbs"], "traffic": GEMV_TRAFFIC, "traffic_src": GEMV_TRAFFIC_SRC,
                     "peak_src": peaks["src"], "kernel": "k_mv", "algorithmic_bytes_per_launch": GEMV_BYTES,
                     "avg_launch_us": launch_us},
        "e2e": {"value": GEMV_BYTES / (e2e_ms * 1e-3) / 1e9 * world, "unit": "GB/s",
                "h2d_bytes_per_step": GEMV_K * 4, "d2h_bytes_per_step": GEMV_N * 4},
        "gpu_launches": args.steps,
        "clocks": clk.summary(),
    }
    return out


# ----------------------------------------------------------------- decode (config 3)
def decode_bytes_per_token(cfg, pos_mean):
    """Algorithmic HBM bytes of one batch-1 decode step: every Q4_0 weight once
    (18 B per 32 values), the fp32 norm weights, and the fp16 K/V of the valid
    positions (pos + 1 cells per layer)."""
    E, F, L, V = cfg["n_embd"], cfg["n_ff"], cfg["n_layer"], cfg["n_vocab"]
    Dq, Dkv = cfg["n_head"] * cfg["head_dim"], cfg["n_head_kv"] * cfg["head_dim"]
    per_layer = (E * (Dq + 2 * Dkv) + Dq * E + 3 * E * F) * 18 // 32
    lm = V * E * 18 // 32
    norms = (L * (2 * E + 2 * cfg["head_dim"]) + E) * 4
    kv = L * 2 * Dkv * 2 * (pos_mean + 1)
    return L * per_layer + lm + norms + kv


DECODE_PROMPT = 512


def cpu_decode_baseline(cfg, seconds=20.0, pos0=DECODE_PROMPT):
    """The oracle (reference semantics, all host threads) decoding the same model
    at the GPU bench's positions: its KV cache holds pos0 cells (seeded N(0,1)
    fp16, standing in for the prompt's K/V: the same work per token) and a
    bounded sample of greedy steps runs from position pos0."""
    from oracle import lib as O
    threads = os.cpu_count() or 1
    t0 = time.perf_counter()
    m = O.Model(cfg, 1234, pos0 + 64, threads)
    m.fill_kv(pos0, 99)
    build_s = time.perf_counter() - t0
    n, tok, t0 = 0, 1, time.perf_counter()
    while n < 3 or (time.perf_counter() - t0 < seconds and n < 60):
        lg, _ = m.forward([tok], pos0 + n, 0)
        tok = O.argmax(lg)
        n += 1
    dt = (time.perf_counter() - t0) / n
    m.close()
    return {"value": 1.0 / dt, "unit": "tok/s", "cores": threads, "kind": "port", "cpu": host_cpu(),
            "sample": f"{n} greedy decode steps of the same model at positions {pos0}..{pos0 + n - 1} over a "
                      f"cache pre-filled to {pos0} cells (oracle/oracle.c, {threads} threads; weights and cache "
                      f"generated in {build_s:.0f} s)"}


def cpu_long_baseline(cfg, ctx, seconds=20.0):
    """Config 5 on the host cores: the oracle model with its KV cache pre-filled
    to ctx cells by the same seeded generator as the GPU engine, then greedy
    decode from position ctx for a bounded sample (at least one token)."""
    from oracle import lib as O
    threads = os.cpu_count() or 1
    t0 = time.perf_counter()
    m = O.Model(cfg, 1234, ctx + 64, threads)
    m.fill_kv(ctx, 99)
    setup_s = time.perf_counter() - t0
    n, tok, t0 = 0, 1, time.perf_counter()
    while n < 1 or (time.perf_counter() - t0 < seconds and n < 60):
        lg, _ = m.forward([tok], ctx + n, 0)
        tok = O.argmax(lg)
        n += 1
    dt = (time.perf_counter() - t0) / n
    m.close()
    return {"value": 1.0 / dt, "unit": "tok/s", "cores": threads, "kind": "port", "cpu": host_cpu(),
            "sample": f"{n} greedy decode step(s) of the same 8B model at positions {ctx}..{ctx + n - 1} over a "
                      f"cache pre-filled to {ctx} cells (oracle/oracle.c, {threads} threads; model and cache "
                      f"generated in {setup_s:.0f} s)"}


def cpu_prefill_baseline(cfg, n_tokens=48):
    """The oracle (reference semantics, all host threads) prefilling a bounded
    prompt of the same model from an empty cache: prompt tokens per second."""
    from oracle import lib as O
    threads = os.cpu_count() or 1
    m = O.Model(cfg, 1234, n_tokens + 8, threads)
    prompt = np.random.default_rng(4).integers(0, cfg["n_vocab"], n_tokens).astype(np.int32)
    t0 = time.perf_counter()
    m.forward(prompt, 0)
    dt = time.perf_counter() - t0
    m.close()
    return {"value": n_tokens / dt, "unit": "tok/s", "cores": threads, "kind": "port", "cpu": host_cpu(),
            "sample": f"one {n_tokens}-token prompt prefilled from an empty cache (oracle/oracle.c, {threads} threads; "
                      f"its mat-muls run row by row, as the reference's gemv path)"}


# DRAM bytes (read + write) per mat-vec launch of the decode step, mean over the
# step's 145 launches: each launch's ncu figure (profiles/k_mv_qwen3_4b_decode.md,
# a 4-layer model of the same shapes; every layer reads the same bytes)
DECODE_MV_TRAFFIC = 15.67e6
DECODE_MV_TRAFFIC_SRC = ("ncu dram__bytes_read.sum + dram__bytes_write.sum per k_mv launch (4-layer case), "
                         "mean over the 145 launches of the 36-layer step")


def profile_cfg(cfg, args):
    """The workload's model, or (--n-layer) the same shapes with fewer layers:
    the same kernels on a few hundred MB, for ncu captures."""
    return dict(cfg, n_layer=args.n_layer) if args.n_layer > 0 else cfg


def profile_tag(args):
    return f"_profile_case_{args.n_layer}_layers" if args.n_layer > 0 else ""


def run_decode(args, rank, world):
    import torch
    import arclight_b200 as A
    from arclight_b200 import bench_util as BU
    from arclight_b200.configs import QWEN3_4B
    from arclight_b200.engine import Engine, nccl_unique_id

    cfg = profile_cfg(QWEN3_4B, args)
    L = A.lib()
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    A.check(L.alb_device_check(local), "device check")
    nid = None
    if world > 1:
        import torch.distributed as dist
        obj = [nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        nid = obj[0]
    n_prompt, n_gen = DECODE_PROMPT, args.steps
    max_ctx = n_prompt + max(n_gen, args.warmup) + 16
    e = Engine(cfg, 1234, max_ctx, 256, rank, world, nid, local)
    prompt = np.random.default_rng(1234).integers(0, cfg["n_vocab"], n_prompt).astype(np.int32)
    tok0 = e.prefill(prompt, 0)
    st = torch.cuda.ExternalStream(e.stream())
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        # warm-up: W greedy steps from the prompt end (re-run below from the same position)
        e.decode_loop(tok0, n_prompt, max(args.warmup, 3), want_tokens=False, sync=True)
        BU.barrier(world)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("timed")   # lets ncu --nvtx-include timed/ list exactly these launches
        e0.record(st)
        e.decode_loop(tok0, n_prompt, n_gen, want_tokens=False, sync=False)
        e1.record(st)
        torch.cuda.nvtx.range_pop()
        e1.synchronize()
    ms = BU.max_over_ranks(e0.elapsed_time(e1) / n_gen, world)
    tok_s = 1000.0 / ms
    info = e.info()   # launches per decode step (the captured graph)

    # e2e through the public C ABI with host buffers: token and position in
    # (8 B H2D), next token out (4 B D2H), one call per step
    BU.barrier(world)
    tok = tok0
    t_e2e = time.perf_counter()
    for i in range(n_gen):
        tok = e.decode(tok, n_prompt + i)
    e2e_ms = BU.max_over_ranks((time.perf_counter() - t_e2e) * 1000.0 / n_gen, world)

    # dominant kernel (the Q4_0 mat-vec family) timed live: the step's mat-vec
    # launches replayed from a CUDA graph on the same weights
    gemv = BU.time_decode_gemvs(e, cfg, world, rank, reps=3)

    peaks = load_peaks()
    pos_mean = n_prompt + (n_gen - 1) / 2.0
    bpt = decode_bytes_per_token(cfg, pos_mean)
    step_gbs = bpt * tok_s / 1e9
    # dominant kernel: the Q4_0 mat-vec (k_mv), every launch of the step (QKV,
    # O, gate/up, down of each layer, lm head) with the step's input modes
    roofline = {"bound": "hbm", "achieved": gemv["gbs"], "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": gemv["gbs"] / peaks["hbm_gbs"], "traffic": DECODE_MV_TRAFFIC,
                "traffic_src": DECODE_MV_TRAFFIC_SRC, "peak_src": peaks["src"],
                "kernel": "k_mv: q4_0 x q8_0 mat-vec (all decode-step launches, replayed from a CUDA graph)",
                "algorithmic_bytes_per_launch": gemv["bytes_per_launch"], "avg_launch_us": gemv["us_per_launch"]}
    out = {
        "metric": "Qwen3-4B Q4_0 decode tok/s bs=1",
        "value": tok_s, "unit": "tok/s", "n_gpus": world, "steps": n_gen, "warmup": max(args.warmup, 3),
        "ms_per_step": ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": DTYPE_DECODE,
        "data": "synthetic: seeded random-init Qwen3-4B-shaped weights (device-generated), uniform random prompt",
        "config": {"workload": "config3_decode_qwen3_4b" + profile_tag(args), "prompt": n_prompt, "decode_steps": n_gen,
                   "parallelism": f"tp{world}", "global_batch": 1,
                   "l2": "inputs larger than L2 (2.26 GB of weights per token)",
                   "launches_per_token": info["launches_per_step"], "attn_splits": info["attn_splits"]},
        "roofline": roofline,
        "gemv_family": {"kernel": "q4_0 x q8_0 mat-vec launches of the multi-kernel step, replayed from a CUDA graph",
                        "achieved_gbs": gemv["gbs"], "frac": gemv["gbs"] / peaks["hbm_gbs"],
                        "bytes_per_launch": gemv["bytes_per_launch"], "avg_launch_us": gemv["us_per_launch"]},
        "step_roofline": {"bytes_per_token": bpt, "achieved_gbs": step_gbs, "peak_gbs": peaks["hbm_gbs"] * world,
                          "frac": step_gbs / (peaks["hbm_gbs"] * world),
                          "roofline_tok_s": peaks["hbm_gbs"] * world * 1e9 / bpt},
        "e2e": {"value": 1000.0 / e2e_ms, "unit": "tok/s", "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 4},
        "gpu_launches": info["launches_per_step"] * n_gen,
        "clocks": clk.summary(),
    }
    e.close()
    if world == 1:
        out["config1_gemv"] = gemv_config1_record()
    return out


# ----------------------------------------------------------------- long context (config 5)
LONG_CTX = 32768


# ----------------------------------------------------------------- attention alone (config 5 shape)
ATT_HQ, ATT_HKV, ATT_CELLS, ATT_COPIES = 32, 8, 32768, 4
ATT_BYTES = 2 * ATT_CELLS * ATT_HKV * 128 * 2 + 2 * ATT_HQ * 128 * 4   # K + V + q + out per call
# DRAM bytes (read + write) per call: ncu figures of its two kernels
# (profiles/k_att_split_config5_attention.md: scores 67.95 MB, P.V 72.40 MB)
ATT_TRAFFIC = 140.35e6


def cpu_attn_baseline(seconds: float = 10.0):
    """The oracle's attention (mode 0, one thread) at the same shape, bounded sample."""
    from oracle import lib as O
    rng = np.random.default_rng(2)
    k = rng.standard_normal((ATT_CELLS, ATT_HKV, 128)).astype(np.float16).view(np.uint16)
    v = rng.standard_normal((ATT_CELLS, ATT_HKV, 128)).astype(np.float16).view(np.uint16)
    q = rng.standard_normal((1, ATT_HQ, 128)).astype(np.float32)
    kv_len = np.array([ATT_CELLS], np.int32)
    n, t0 = 0, time.perf_counter()
    while n == 0 or time.perf_counter() - t0 < seconds:
        O.flash_attn(q, k, v, kv_len, 1.0 / np.sqrt(128.0), 0)
        n += 1
    dt = (time.perf_counter() - t0) / n
    return {"value": ATT_BYTES / dt / 1e9, "unit": "GB/s", "cores": 1, "kind": "port", "cpu": host_cpu(),
            "sample": f"{n} attention calls ({ATT_HQ}/{ATT_HKV} heads over {ATT_CELLS} cells) in {seconds:.0f} s"}


def run_attn(args, rank, world):
    """Config 5's attention alone: split-K flash decode of one token over a
    32768-cell fp16 KV cache (Qwen3-8B heads: 32 query / 8 KV), one call per
    step through the C ABI, rotating over 4 cache copies (512 MB > L2)."""
    import torch
    import arclight_b200 as A
    from arclight_b200 import bench_util as BU

    L = A.lib()
    local = int(os.environ.get("LOCAL_RANK", 0))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    A.check(L.alb_device_check(local), "device check")
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    S = (4 * sms + ATT_HKV - 1) // ATT_HKV          # the engine's decode split count
    gen = torch.Generator(device=dev).manual_seed(7)
    kc = torch.randn((ATT_COPIES, ATT_CELLS, ATT_HKV, 128), generator=gen, device=dev).half()
    vc = torch.randn((ATT_COPIES, ATT_CELLS, ATT_HKV, 128), generator=gen, device=dev).half()
    q = torch.randn((1, ATT_HQ, 128), generator=gen, device=dev)
    out = torch.empty_like(q)
    ws = torch.zeros(L.alb_flash_attn_workspace_bytes(ATT_HQ, ATT_HKV, 1, S, ATT_CELLS), dtype=torch.uint8,
                     device=dev)
    scale = 1.0 / float(np.sqrt(128.0))
    s = torch.cuda.Stream()

    def call(i, qp=None, op=None):
        qp = q if qp is None else qp
        op = out if op is None else op
        A.check(L.alb_flash_attn(qp.data_ptr(), kc[i % ATT_COPIES].data_ptr(), vc[i % ATT_COPIES].data_ptr(),
                                 1, ATT_HQ, ATT_HKV, ATT_CELLS - 1, scale, S, ws.data_ptr(), op.data_ptr(),
                                 s.cuda_stream), "alb_flash_attn")

    with torch.cuda.stream(s):
        for i in range(ATT_COPIES):
            call(i)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for i in range(ATT_COPIES):
                call(i)
    reps = max(1, args.steps // ATT_COPIES)
    steps = reps * ATT_COPIES
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk, torch.cuda.stream(s):   # replays and events on the same stream
        for _ in range(max(args.warmup, 3)):
            g.replay()
        torch.cuda.synchronize()
        BU.barrier(world)
        torch.cuda.nvtx.range_push("timed")
        e0.record(s)
        for _ in range(reps):
            g.replay()
        e1.record(s)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
    ms = BU.max_over_ranks(e0.elapsed_time(e1) / steps, world)

    # e2e through the C ABI with host buffers: H2D q, attention, D2H out
    qh = torch.randn((1, ATT_HQ, 128)).pin_memory()
    oh = torch.empty((1, ATT_HQ, 128)).pin_memory()
    qd, od = torch.empty_like(q), torch.empty_like(q)
    with torch.cuda.stream(s):
        for i in range(3):
            qd.copy_(qh, non_blocking=True)
            call(i, qd, od)
            oh.copy_(od, non_blocking=True)
        torch.cuda.synchronize()
        e0.record(s)
        for i in range(steps):
            qd.copy_(qh, non_blocking=True)
            call(i, qd, od)
            oh.copy_(od, non_blocking=True)
        e1.record(s)
        torch.cuda.synchronize()
    e2e_ms = BU.max_over_ranks(e0.elapsed_time(e1) / steps, world)
    peaks = load_peaks()
    achieved = ATT_BYTES / (ms * 1e-3) / 1e9
    return {
        "metric": "split-K flash decode GB/s (config 5 attention: 32/8 heads, 32768 fp16 cells)",
        "value": achieved * world, "unit": "GB/s", "n_gpus": world, "steps": steps, "warmup": max(args.warmup, 3),
        "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "fp16 KV, fp32 scores (sequential fma), fp32 softmax sums within 128-cell chunks, fp64 across chunks",
        "data": "synthetic: N(0,1) q/K/V",
        "config": {"workload": "config5_attention", "n_head": ATT_HQ, "n_head_kv": ATT_HKV, "cells": ATT_CELLS,
                   "splits": S, "kv_copies": ATT_COPIES, "l2": "inputs larger than L2: 4 rotating caches (512 MB)"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / peaks["hbm_gbs"], "traffic": ATT_TRAFFIC, "peak_src": peaks["src"],
                     "traffic_src": "ncu dram__bytes_read.sum + dram__bytes_write.sum of the two kernels of one call",
                     "kernel": "k_att_scores + k_att_pv (one call)",
                     "algorithmic_bytes_per_launch": ATT_BYTES},
        "e2e": {"value": ATT_BYTES / (e2e_ms * 1e-3) / 1e9 * world, "unit": "GB/s",
                "h2d_bytes_per_step": ATT_HQ * 128 * 4, "d2h_bytes_per_step": ATT_HQ * 128 * 4},
        "gpu_launches": 2 * steps,
        "clocks": clk.summary(),
    }


def run_long(args, rank, world):
    """Config 5: Qwen3-8B shape, KV cache pre-filled to 32768 positions with
    N(0,1) fp16, then greedy batch-1 decode (split-K attention over the cache)."""
    import torch
    import arclight_b200 as A
    from arclight_b200 import bench_util as BU
    from arclight_b200.configs import QWEN3_8B
    from arclight_b200.engine import Engine, nccl_unique_id

    cfg = QWEN3_8B
    L = A.lib()
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    A.check(L.alb_device_check(local), "device check")
    nid = None
    if world > 1:
        import torch.distributed as dist
        obj = [nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        nid = obj[0]
    n_gen = args.steps
    max_ctx = LONG_CTX + max(n_gen, args.warmup) + 16
    e = Engine(cfg, 1234, max_ctx, 16, rank, world, nid, local)
    e.fill_kv(LONG_CTX, 99)
    tok0 = 1
    st = torch.cuda.ExternalStream(e.stream())
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e.decode_loop(tok0, LONG_CTX, max(args.warmup, 3), want_tokens=False, sync=True)
        BU.barrier(world)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("timed")
        e0.record(st)
        e.decode_loop(tok0, LONG_CTX, n_gen, want_tokens=False, sync=False)
        e1.record(st)
        torch.cuda.nvtx.range_pop()
        e1.synchronize()
    ms = BU.max_over_ranks(e0.elapsed_time(e1) / n_gen, world)
    info = e.info()
    BU.barrier(world)
    tok = tok0
    t_e2e = time.perf_counter()
    for i in range(min(n_gen, 32)):
        tok = e.decode(tok, LONG_CTX + i)
    e2e_ms = BU.max_over_ranks((time.perf_counter() - t_e2e) * 1000.0 / min(n_gen, 32), world)
    peaks = load_peaks()
    E, F, Lr, V = cfg["n_embd"], cfg["n_ff"], cfg["n_layer"], cfg["n_vocab"]
    Dq, Dkv = cfg["n_head"] * 128, cfg["n_head_kv"] * 128
    weights = (Lr * (E * (Dq + 2 * Dkv) + Dq * E + 3 * E * F) + V * E) * 18 // 32
    kv = Lr * 2 * Dkv * 2 * (LONG_CTX + (n_gen - 1) / 2.0 + 1)
    bpt = weights + kv + (Lr * (2 * E + 256) + E) * 4
    gbs_total = bpt * 1000.0 / ms / 1e9
    gbs_gpu = gbs_total / world
    out = {
        "metric": "Qwen3-8B Q4_0 decode tok/s bs=1 at 32768-token context",
        "value": 1000.0 / ms, "unit": "tok/s", "n_gpus": world, "steps": n_gen, "warmup": max(args.warmup, 3),
        "ms_per_step": ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": DTYPE_DECODE,
        "data": "synthetic: seeded random-init Qwen3-8B-shaped weights; KV cache filled with seeded N(0,1) fp16",
        "config": {"workload": "config5_long_qwen3_8b", "context": LONG_CTX, "decode_steps": n_gen,
                   "parallelism": f"tp{world}", "global_batch": 1,
                   "l2": "inputs larger than L2 (4.26 GB of weights + 4.83 GB of KV per token)",
                   "launches_per_token": info["launches_per_step"], "attn_splits": info["attn_splits"]},
        "roofline": {"bound": "hbm", "achieved": gbs_gpu, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": gbs_gpu / peaks["hbm_gbs"], "traffic": None, "peak_src": peaks["src"],
                     "kernel": "decode step (multi-kernel CUDA graph: mat-vecs + split-K flash decode), per GPU",
                     "algorithmic_bytes_per_launch": bpt / world, "avg_launch_us": ms * 1000.0},
        "gbs_per_gpu": gbs_gpu,
        "e2e": {"value": 1000.0 / e2e_ms, "unit": "tok/s", "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 4},
        "gpu_launches": info["launches_per_step"] * n_gen,
        "clocks": clk.summary(),
    }
    e.close()
    return out


# ----------------------------------------------------------------- prefill (config 4)
PREFILL_T = 2048
INT8_PEAK_TOPS = 4500.0   # nominal dense int8 (no measured int8 peak in MEASURED_PEAKS.json)


def run_prefill(args, rank, world):
    import torch
    import arclight_b200 as A
    from arclight_b200 import bench_util as BU
    from arclight_b200.configs import QWEN3_4B
    from arclight_b200.engine import Engine, nccl_unique_id
    import ctypes as C

    cfg = profile_cfg(QWEN3_4B, args)
    L = A.lib()
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    A.check(L.alb_device_check(local), "device check")
    nid = None
    if world > 1:
        import torch.distributed as dist
        obj = [nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        nid = obj[0]
    T = PREFILL_T
    e = Engine(cfg, 1234, T + 16, T, rank, world, nid, local)
    prompt = np.random.default_rng(4).integers(0, cfg["n_vocab"], T).astype(np.int32)
    st = torch.cuda.ExternalStream(e.stream())
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    with ClockSampler(local) as clk:
        for _ in range(args.warmup):
            A.check(L.alb_engine_reset(e.h))
            e.prefill(prompt, 0)
        info = e.info()                      # launches of one prefill ubatch
        BU.barrier(world)
        torch.cuda.synchronize()
        walls = []
        torch.cuda.nvtx.range_push("timed")
        for k in range(args.steps):
            A.check(L.alb_engine_reset(e.h))  # empty cache before every prompt (not timed)
            t0 = time.perf_counter()
            ev[k][0].record(st)
            e.prefill(prompt, 0)                # host tokens in, greedy next token out
            ev[k][1].record(st)
            walls.append(time.perf_counter() - t0)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
    ms = BU.max_over_ranks(sum(a.elapsed_time(b) for a, b in ev) / args.steps, world)
    wall_ms = BU.max_over_ranks(1000.0 * sum(walls) / len(walls), world)
    us = C.c_float()
    ops = C.c_double()
    A.check(L.alb_engine_time_prefill_gemm(e.h, 3, C.byref(us), C.byref(ops)), "time_prefill_gemm")
    tops = ops.value / (us.value * 1e-6) / 1e12
    total_ops = 2.0 * T * (cfg["n_layer"] * ((cfg["n_head"] + 2 * cfg["n_head_kv"]) * 128 * cfg["n_embd"]
                                             + cfg["n_head"] * 128 * cfg["n_embd"] + 3 * cfg["n_embd"] * cfg["n_ff"]))
    out = {
        "metric": "Qwen3-4B Q4_0 prefill tok/s (2048-token prompt, 1/TTFT)",
        "value": T * 1000.0 / ms, "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "ttft_ms": ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "q4_0 x q8_0 int8 tensor cores (tcgen05 kind::i8), the reference's fp32 block chain, fp16 KV",
        "data": "synthetic: seeded random-init Qwen3-4B-shaped weights, uniform random prompt",
        "config": {"workload": "config4_prefill_qwen3_4b" + profile_tag(args), "prompt": T, "parallelism": f"tp{world}",
                   "global_batch": 1, "l2": "inputs larger than L2 (2.26 GB of weights per prefill)",
                   "launches_per_prefill": info["launches_per_step"]},
        "roofline": {"bound": "tensor", "achieved": tops, "peak": INT8_PEAK_TOPS, "unit": "TOP/s",
                     "frac": tops / INT8_PEAK_TOPS, "traffic": None, "peak_src": "nominal dense int8 (B200)",
                     "kernel": "k_prefill_gemm (tcgen05 kind::i8, TMEM accumulators; + its activation quantizer)",
                     "algorithmic_ops_per_launch": ops.value, "avg_launch_us": us.value},
        "prefill_int8_ops": total_ops,
        "e2e": {"value": T * 1000.0 / wall_ms, "unit": "tok/s", "h2d_bytes_per_step": 4 * T, "d2h_bytes_per_step": 4},
        "gpu_launches": info["launches_per_step"] * args.steps,
        "clocks": clk.summary(),
    }
    e.close()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="decode", choices=["decode", "gemv", "prefill", "long", "attn"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--n-layer", type=int, default=0,
                    help="decode/prefill with this many layers: a small case for ncu captures, not a bench value")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.steps is None:
        args.steps = {"decode": 256, "gemv": 2400, "prefill": 5, "long": 128, "attn": 400}[args.workload]
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    if world > 1:
        import torch.distributed as dist
        import datetime
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))

    if args.impl == "reference":
        if rank == 0:
            if args.workload == "decode":
                from arclight_b200.configs import QWEN3_4B
                cb = cpu_decode_baseline(QWEN3_4B, seconds=min(60.0, 5.0 + 0.2 * args.steps))
                metric, unit, cfgname = "Qwen3-4B Q4_0 decode tok/s bs=1", "tok/s", "config3_decode_qwen3_4b"
            elif args.workload == "prefill":
                from arclight_b200.configs import QWEN3_4B
                cb = cpu_prefill_baseline(QWEN3_4B)
                metric, unit = "Qwen3-4B Q4_0 prefill tok/s (2048-token prompt, 1/TTFT)", "tok/s"
                cfgname = "config4_prefill_qwen3_4b"
            elif args.workload == "long":
                from arclight_b200.configs import QWEN3_8B
                cb = cpu_long_baseline(QWEN3_8B, LONG_CTX, seconds=min(60.0, 5.0 + 0.2 * args.steps))
                metric, unit = "Qwen3-8B Q4_0 decode tok/s bs=1 at 32768-token context", "tok/s"
                cfgname = "config5_long_qwen3_8b"
            elif args.workload == "attn":
                cb = cpu_attn_baseline(seconds=10.0)
                metric, unit = "split-K flash decode GB/s (config 5 attention: 32/8 heads, 32768 fp16 cells)", "GB/s"
                cfgname = "config5_attention"
            else:
                cb = cpu_gemv_baseline(seconds=min(20.0, 2.0 + 0.005 * args.steps))
                metric, unit, cfgname = "Q4_0xQ8_0 GEMV HBM GB/s (config 1, W 9728x2560)", "GB/s", "config1_gemv"
            line = {"impl": "reference", "metric": metric, "value": cb["value"], "unit": unit, "n_gpus": world,
                    "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
                    "scaling": "weak" if args.workload in ("gemv", "attn") else "strong", "vs_baseline": None,
                    "dtype": "q4_0 x q8_0", "data": "synthetic", "config": {"workload": cfgname},
                    "cpu_baseline": cb,
                    "e2e": {"value": cb["value"], "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
            print(json.dumps(line), flush=True)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return

    if args.workload == "decode":
        out = run_decode(args, rank, world)
    elif args.workload == "prefill":
        out = run_prefill(args, rank, world)
    elif args.workload == "long":
        out = run_long(args, rank, world)
    elif args.workload == "attn":
        out = run_attn(args, rank, world)
    else:
        out = run_gemv(args, rank, world)
    if rank == 0:
        if not args.no_cpu_baseline:
            if args.workload == "decode":
                from arclight_b200.configs import QWEN3_4B
                out["cpu_baseline"] = cpu_decode_baseline(QWEN3_4B, seconds=20.0)
            elif args.workload == "prefill":
                from arclight_b200.configs import QWEN3_4B
                out["cpu_baseline"] = cpu_prefill_baseline(QWEN3_4B)
            elif args.workload == "long":
                from arclight_b200.configs import QWEN3_8B
                out["cpu_baseline"] = cpu_long_baseline(QWEN3_8B, LONG_CTX, seconds=20.0)
            elif args.workload == "attn":
                out["cpu_baseline"] = cpu_attn_baseline(seconds=10.0)
            else:
                out["cpu_baseline"] = cpu_gemv_baseline(seconds=10.0)
        print(json.dumps(out), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
