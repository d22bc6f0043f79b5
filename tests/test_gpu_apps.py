"""The host C++ on top of the C ABI, on a B200.

* al_bench (the al-gen flow over the engine): its greedy tokens after a seeded
  prompt equal the oracle model's, through the per-token calls and through the
  device-resident loop;
* the nnml operator shim (libalb_nnml_ops.so): each operator, called the way
  nnml calls it (tensor views, a compute state whose thread 0 launches), gives
  the same bits as the direct C ABI call it wraps (and thus as the oracle).
"""
import ctypes as C
import math
import os
import subprocess

import numpy as np
import pytest

import arclight_b200 as A
from arclight_b200 import build as B
from arclight_b200.configs import TINY, TINY_GQA
from oracle import lib as O
from tests.test_apps import State, Tensor, shim

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

L = None


def lib():
    global L
    if L is None:
        L = A.lib()
    return L


def stream():
    return torch.cuda.current_stream().cuda_stream


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.uint8).reshape(-1).copy()).cuda()


def run_bench(args):
    r = subprocess.run([B.AL_BENCH, *args], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    lines = {l.split(":", 1)[0]: l.split(":", 1)[1] for l in r.stdout.splitlines() if ":" in l}
    prompt = [int(t) for t in lines["prompt"].split()]
    tokens = [int(t) for t in lines["tokens"].split()]
    assert "prefill time" in lines and "decode time" in lines
    return prompt, tokens


@pytest.mark.parametrize("name,cfg", [("tiny", TINY), ("tiny_gqa", TINY_GQA)])
def test_al_bench_matches_oracle(name, cfg):
    n_prompt, n_gen, seed = 40, 8, 5
    prompt, toks = run_bench(["--model", name, "--prompt", str(n_prompt), "--max_gen", str(n_gen), "--seed", str(seed),
                              "--ubatch", "16", "--print_tokens"])
    assert len(prompt) == n_prompt and len(toks) == n_gen
    m = O.Model(cfg, seed, n_prompt + n_gen + 8, max(1, min(16, os.cpu_count() or 8)))
    try:
        lg, _ = m.forward(np.array(prompt, np.int32), 0, 0)
        ref = [O.argmax(lg)]
        for i in range(n_gen - 1):
            lg, _ = m.forward([ref[-1]], n_prompt + i, 0)
            ref.append(O.argmax(lg))
    finally:
        m.close()
    assert toks == ref
    _, toks_loop = run_bench(["--model", name, "--prompt", str(n_prompt), "--max_gen", str(n_gen), "--seed", str(seed),
                              "--ubatch", "16", "--print_tokens", "--loop"])
    assert toks_loop == toks


def test_al_bench_loads_gguf(tmp_path):
    # a GGUF file of the engine's seeded tiny_gqa weights: al_bench --gguf
    # generates the same greedy tokens as al_bench on the generated weights
    from arclight_b200 import gguf as G
    from arclight_b200.engine import Engine
    seed = 11
    e = Engine(TINY_GQA, seed, 64, 16)
    path = str(tmp_path / "tiny_gqa.gguf")
    G.engine_to_gguf(e, path)
    e.close()
    args = ["--prompt", "24", "--max_gen", "6", "--seed", str(seed), "--ubatch", "16", "--print_tokens"]
    p_gen, t_gen = run_bench(["--model", "tiny_gqa", *args])
    p_file, t_file = run_bench(["--gguf", path, *args])
    assert p_file == p_gen and t_file == t_gen


def view(t, shape, esize):
    v = Tensor()
    for i in range(4):
        v.ne[i] = shape[i] if i < len(shape) else 1
    v.nb[0] = esize
    for i in range(1, 4):
        v.nb[i] = v.nb[i - 1] * v.ne[i - 1]
    v.data = t.data_ptr()
    return v


def call(op, dst, srcs, params=()):
    S = shim()
    for i, s in enumerate(srcs):
        dst.src[i] = C.pointer(s)
    for i, p in enumerate(params):
        dst.op_params[i] = p
    f = getattr(S, op)
    f.restype = C.c_int
    f.argtypes = [C.c_void_p, C.c_void_p]
    xq = torch.zeros(64 * 1024, dtype=torch.uint8, device="cuda")
    ws = torch.zeros(8 << 20, dtype=torch.uint8, device="cuda")
    st = State(ith=0, nth=4, stream=stream(), xq=xq.data_ptr(), xq_bytes=xq.numel(), attn_ws=ws.data_ptr(),
               attn_ws_bytes=ws.numel())
    rc = f(C.byref(st), C.byref(dst))
    torch.cuda.synchronize()
    return rc


def f32bits(x):
    return int(np.array([x], np.float32).view(np.int32)[0])


@pytest.mark.parametrize("repacked", [1, 0])
def test_shim_mul_mat(repacked):
    N, K = 1000, 2560
    rng = np.random.default_rng(3)
    wq = O.quantize_q4_0((rng.standard_normal((N, K)) * 0.02).astype(np.float32))
    src = dev(wq)
    W = torch.empty(lib().alb_q4_0_gpu_bytes(N, K), dtype=torch.uint8, device="cuda")
    A.check(lib().alb_repack_q4_0(W.data_ptr(), src.data_ptr(), N, K, stream()))
    x = torch.from_numpy(rng.standard_normal(K).astype(np.float32)).cuda()
    y = torch.empty(N, device="cuda")
    w_v = view(W, [K, N], 1)
    assert call("nnml_gpu_forward_mul_mat", view(y, [N], 4), [w_v, view(x, [K, 1], 4)], [repacked]) == 0
    xq = torch.empty((K // 32) * 34, dtype=torch.uint8, device="cuda")
    ref = torch.empty(N, device="cuda")
    A.check(lib().alb_quantize_q8_0(x.data_ptr(), xq.data_ptr(), K, 1, stream()))
    if repacked:
        A.check(lib().alb_gemv_q4_0_q8_0(W.data_ptr(), xq.data_ptr(), ref.data_ptr(), N, K, None, stream()))
    else:
        A.check(lib().alb_mul_mat_q4_0_q8_0(W.data_ptr(), xq.data_ptr(), ref.data_ptr(), N, K, stream()))
    torch.cuda.synchronize()
    assert torch.equal(y, ref)
    # and the reference's own chains
    q8 = O.quantize_q8_0(x.cpu().numpy())
    want = O.gemv(wq, q8, 8)[0] if repacked else O.mul_mat_generic(wq, q8, 8)
    np.testing.assert_array_equal(y.cpu().numpy(), want)


def test_shim_elementwise_and_sampling():
    rng = np.random.default_rng(4)
    rows, n = 3, 2560
    x = torch.from_numpy((rng.standard_normal((rows, n)) * 5).astype(np.float32)).cuda()
    w = torch.from_numpy((1 + 0.01 * rng.standard_normal(n)).astype(np.float32)).cuda()
    y, ref = torch.empty_like(x), torch.empty_like(x)
    assert call("nnml_gpu_forward_rms_norm_mul", view(y, [n, rows], 4), [view(x, [n, rows], 4), view(w, [n], 4)],
                [f32bits(1e-6)]) == 0
    A.check(lib().alb_rms_norm(x.data_ptr(), w.data_ptr(), ref.data_ptr(), rows, n, C.c_float(1e-6), stream()))
    torch.cuda.synchronize()
    assert torch.equal(y, ref)
    g = torch.from_numpy(rng.standard_normal(9728).astype(np.float32)).cuda()
    u = torch.from_numpy(rng.standard_normal(9728).astype(np.float32)).cuda()
    h, href = torch.empty_like(g), torch.empty_like(g)
    assert call("nnml_gpu_forward_swiglu", view(h, [9728], 4), [view(g, [9728], 4), view(u, [9728], 4)]) == 0
    A.check(lib().alb_swiglu(g.data_ptr(), u.data_ptr(), href.data_ptr(), 9728, stream()))
    torch.cuda.synchronize()
    assert torch.equal(h, href)
    np.testing.assert_array_equal(h.cpu().numpy(), O.swiglu(g.cpu().numpy(), u.cpu().numpy()))
    logits = torch.from_numpy(rng.standard_normal(151936).astype(np.float32)).cuda()
    tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert call("nnml_gpu_sample_greedy", view(tok, [1], 4), [view(logits, [151936], 4)]) == 0
    assert int(tok.item()) == O.argmax(logits.cpu().numpy())


def test_shim_get_rows():
    V, E = 4096, 512
    rng = np.random.default_rng(6)
    wq = O.quantize_q4_0((rng.standard_normal((V, E)) * 0.02).astype(np.float32))
    src = dev(wq)
    W = torch.empty(lib().alb_q4_0_gpu_bytes(V, E), dtype=torch.uint8, device="cuda")
    A.check(lib().alb_repack_q4_0(W.data_ptr(), src.data_ptr(), V, E, stream()))
    ids = torch.tensor([5, 0, 4095, 17], dtype=torch.int32, device="cuda")
    out, ref = torch.empty((4, E), device="cuda"), torch.empty((4, E), device="cuda")
    assert call("nnml_gpu_forward_get_rows", view(out, [E, 4], 4), [view(W, [E, V], 1), view(ids, [4], 4)]) == 0
    A.check(lib().alb_get_rows_q4_0(W.data_ptr(), V, E, ids.data_ptr(), 4, ref.data_ptr(), stream()))
    torch.cuda.synchronize()
    assert torch.equal(out, ref)


def test_shim_set_rows():
    rng = np.random.default_rng(8)
    rows = torch.from_numpy(rng.standard_normal((5, 1024)).astype(np.float32)).cuda()
    idx = torch.tensor([9, 0, 3, 63, 7], dtype=torch.int64, device="cuda")
    cache = torch.zeros((64, 1024), dtype=torch.int16, device="cuda")
    assert call("nnml_gpu_forward_set_rows", view(cache, [1024, 64], 2), [view(rows, [1024, 5], 4), view(idx, [5], 8)]) == 0
    torch.cuda.synchronize()
    want = np.zeros((64, 1024), np.uint16)
    want[idx.cpu().numpy()] = O.fp32_to_fp16(rows.cpu().numpy())
    np.testing.assert_array_equal(cache.cpu().numpy().view(np.uint16), want)


@pytest.mark.parametrize("T,pos0,splits", [(1, 700, 74), (24, 0, 1)])
def test_shim_flash_attn(T, pos0, splits):
    Hq, Hkv = 32, 8
    rng = np.random.default_rng(T + pos0)
    cells = pos0 + T
    k = O.fp32_to_fp16(rng.standard_normal((cells, Hkv, 128)).astype(np.float32))
    v = O.fp32_to_fp16(rng.standard_normal((cells, Hkv, 128)).astype(np.float32))
    q = (rng.standard_normal((T, Hq, 128)) * 0.5).astype(np.float32)
    Kd, Vd = dev(k.view(np.int16)), dev(v.view(np.int16))
    Qd = torch.from_numpy(q).cuda()
    out = torch.empty((T, Hq, 128), device="cuda")
    scale = 1.0 / math.sqrt(128.0)
    assert call("nnml_gpu_forward_flash_attn_ext", view(out, [128, Hq, T], 4),
                [view(Qd, [128, Hq, T], 4), view(Kd, [128, Hkv, cells], 2), view(Vd, [128, Hkv, cells], 2)],
                [pos0, f32bits(scale), splits]) == 0
    ref = O.flash_attn(q, k, v, (pos0 + np.arange(T) + 1).astype(np.int32), scale, 0)
    np.testing.assert_array_equal(out.cpu().numpy(), ref)
