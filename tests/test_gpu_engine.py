"""End-to-end parity of the GPU Qwen3 engine against the oracle model.

north_star bar: last-layer logits within 2e-2 max-abs, identical greedy tokens
for the first 32 decode steps, on the seeded random-init weights.

Two comparisons:

* against the oracle with the reference's own mat-vec arithmetic (the NEON fp32
  chains of gemm.cpp:127-190 and vec_dot_q4_0_q8_0, arm.cpp:633-692) and the
  fp32 attention of oracle mode 0: the GPU must be bit-identical -- every
  logit of every step, every greedy token -- at the config-2, config-3 and
  config-5 shapes (config 5 with the KV cache pre-filled to 32768 cells);
* against the reference's complete semantics, including its fp16-accumulating
  attention (oracle mode 1), teacher-forced on the reference's greedy tokens.
  Random-init Qwen3 logits amplify any rounding difference before a Q8_0
  re-quantization: an fp64 attention (oracle mode 2) is itself 4e-2..6e-2
  max-abs away from the reference and picks different greedy tokens.  The bar
  is therefore that the GPU is no farther from the reference than the fp64
  computation is (within 25 %), with the measured numbers printed.

The synthetic weights themselves must be bit-identical to the oracle's.
"""
import numpy as np
import pytest

from arclight_b200.configs import QWEN3_0_6B, QWEN3_4B, QWEN3_8B, TINY, TINY_GQA
from oracle import lib as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

LOGIT_ATOL = 2e-2   # north_star: logits within 2e-2 max-abs


def engine(cfg, seed, max_ctx, max_ub=64):
    from arclight_b200.engine import Engine
    return Engine(cfg, seed, max_ctx, max_ub)


def oracle_threads():
    import os
    return max(1, min(32, os.cpu_count() or 8))


@pytest.mark.parametrize("cfg", [TINY, TINY_GQA], ids=["tiny", "tiny_gqa"])
def test_generated_weights_match_oracle(cfg):
    e = engine(cfg, seed=11, max_ctx=64)
    m = O.Model(cfg, 11, 64)
    try:
        for layer in (0, cfg["n_layer"] - 1):
            for kind in (O.T_WQ, O.T_WK, O.T_WV, O.T_WO, O.T_GATE, O.T_UP, O.T_DOWN):
                np.testing.assert_array_equal(e.weight_blocks(layer, kind).view(np.uint8),
                                              m.q4_tensor(layer, kind).view(np.uint8), err_msg=f"{layer}/{kind}")
            for kind, n in ((O.T_ATTN_NORM, cfg["n_embd"]), (O.T_FFN_NORM, cfg["n_embd"]), (O.T_Q_NORM, 128),
                            (O.T_K_NORM, 128)):
                np.testing.assert_array_equal(e.norm_weights(layer, kind, n), m.f32_tensor(layer, kind))
        np.testing.assert_array_equal(e.weight_blocks(-1, O.T_TOK_EMBD).view(np.uint8),
                                      m.q4_tensor(-1, O.T_TOK_EMBD).view(np.uint8))
    finally:
        e.close()
        m.close()


def run_parity(cfg, seed, n_prompt, n_gen, max_ub, n_fill=0, loop=True):
    """GPU vs the oracle (reference mat-vec chains, attention mode 0): every
    logit of every step bit-identical, identical greedy tokens.  n_fill > 0:
    no prompt; the KV cache holds n_fill seeded N(0,1) positions and decoding
    starts at position n_fill with token 1 (the long-context workload)."""
    rng = np.random.default_rng(seed)
    prompt = rng.integers(0, cfg["n_vocab"], n_prompt).astype(np.int32)
    max_ctx = n_fill + n_prompt + n_gen + 8
    e = engine(cfg, seed, max_ctx, max_ub)
    m = O.Model(cfg, seed, max_ctx, oracle_threads())
    try:
        if n_fill:
            e.fill_kv(n_fill, 99)
            m.fill_kv(n_fill, 99)
            tok, pos0 = 1, n_fill
            gpu_toks, ref_toks = [tok], [tok]
            steps = n_gen
        else:
            tok = e.prefill(prompt, 0)
            lg_ref, _ = m.forward(prompt, 0, 0)
            np.testing.assert_array_equal(e.logits(), lg_ref, err_msg="prefill logits")
            assert tok == O.argmax(lg_ref)
            gpu_toks, ref_toks = [tok], [tok]
            pos0, steps = n_prompt, n_gen - 1
        for i in range(steps):
            nxt = e.decode(gpu_toks[-1], pos0 + i)
            lg_ref, _ = m.forward([ref_toks[-1]], pos0 + i, 0)
            np.testing.assert_array_equal(e.logits(), lg_ref, err_msg=f"decode step {i} logits")
            gpu_toks.append(nxt)
            ref_toks.append(O.argmax(lg_ref))
        assert gpu_toks == ref_toks, f"greedy tokens diverge: {gpu_toks} vs {ref_toks}"
        if loop:
            # the device-resident loop (graph replays, no host round trip) gives the same tokens
            out = e.decode_loop(gpu_toks[0], pos0, len(gpu_toks) - 1)
            assert list(out) == gpu_toks[1:]
        return gpu_toks
    finally:
        e.close()
        m.close()


@pytest.mark.parametrize("cfg,ub", [(TINY, 64), (TINY, 5), (TINY_GQA, 16)], ids=["tiny", "tiny_ub5", "tiny_gqa"])
def test_engine_tiny_greedy_32(cfg, ub):
    run_parity(cfg, seed=5, n_prompt=40, n_gen=32, max_ub=ub)


def test_engine_qwen3_0_6b_config2_greedy_32():
    """Config 2 shape (Qwen3-0.6B, random init): 128-token prompt, 32 greedy steps."""
    run_parity(QWEN3_0_6B, seed=1234, n_prompt=128, n_gen=32, max_ub=128)


def test_engine_qwen3_4b_config3_greedy_32():
    """Config 3 shape (Qwen3-4B): 128-token prompt, 32 greedy steps, one GPU."""
    run_parity(QWEN3_4B, seed=4321, n_prompt=128, n_gen=32, max_ub=128, loop=False)


def test_engine_qwen3_8b_config5_prefilled_32768():
    """Config 5 shape (Qwen3-8B, untied lm head): KV cache pre-filled to 32768
    cells, then 2 greedy decode steps at positions 32768 and 32769."""
    run_parity(QWEN3_8B, seed=77, n_prompt=0, n_gen=2, max_ub=16, n_fill=32768, loop=False)


def test_prefilled_kv_long_context_decode():
    """Config-5 path at a small shape: 1000 pre-filled positions, 8 steps."""
    run_parity(TINY_GQA, seed=21, n_prompt=0, n_gen=8, max_ub=16, n_fill=1000)


def teacher_forced_vs_reference(cfg, seed, n_prompt, n_steps, max_ub):
    """Feeds the reference's greedy tokens (oracle, attention mode 1) to the GPU
    and to the fp64-attention oracle (mode 2); returns the per-step logit
    max-abs of each against the reference and the argmax agreement counts."""
    rng = np.random.default_rng(seed)
    prompt = rng.integers(0, cfg["n_vocab"], n_prompt).astype(np.int32)
    max_ctx = n_prompt + n_steps + 8
    e = engine(cfg, seed, max_ctx, max_ub)
    ref = O.Model(cfg, seed, max_ctx, oracle_threads())
    f64 = O.Model(cfg, seed, max_ctx, oracle_threads())
    d_gpu, d_64, agree_gpu, agree_64 = [], [], 0, 0
    try:
        e.prefill(prompt, 0)
        lr, _ = ref.forward(prompt, 0, 1)
        l64, _ = f64.forward(prompt, 0, 2)
        toks = [O.argmax(lr)]
        for i in range(n_steps + 1):
            lg = e.logits()
            d_gpu.append(float(np.max(np.abs(lg.astype(np.float64) - lr))))
            d_64.append(float(np.max(np.abs(l64.astype(np.float64) - lr))))
            agree_gpu += int(O.argmax(lg) == O.argmax(lr))
            agree_64 += int(O.argmax(l64) == O.argmax(lr))
            if i == n_steps:
                break
            e.decode(toks[-1], n_prompt + i)
            lr, _ = ref.forward([toks[-1]], n_prompt + i, 1)
            l64, _ = f64.forward([toks[-1]], n_prompt + i, 2)
            toks.append(O.argmax(lr))
    finally:
        e.close()
        ref.close()
        f64.close()
    return d_gpu, d_64, agree_gpu, agree_64


@pytest.mark.parametrize("cfg,n_prompt,n_steps", [(TINY_GQA, 40, 16), (QWEN3_0_6B, 128, 16)], ids=["tiny_gqa", "0.6b"])
def test_engine_vs_reference_attention_semantics(cfg, n_prompt, n_steps):
    d_gpu, d_64, a_gpu, a_64 = teacher_forced_vs_reference(cfg, 5, n_prompt, n_steps, 128)
    print(f"vs reference (fp16 attention): GPU max-abs {max(d_gpu):.3e} (argmax agree {a_gpu}/{len(d_gpu)}), "
          f"fp64-attention oracle max-abs {max(d_64):.3e} (agree {a_64}/{len(d_64)})")
    assert max(d_gpu) <= 1.25 * max(d_64) + 1e-3, (d_gpu, d_64)


def test_fresh_engines_are_deterministic():
    """Engines created one after another (device memory recycled from the
    previous engine, different cache sizes) give bit-identical residual streams
    after a 128-token prefill and identical logits over 3 decode steps.  Guards
    the prefill mat-mul's activation-scale ring against cross-warp reuse."""
    cfg = dict(QWEN3_4B, n_layer=12)
    prompt = np.random.default_rng(4321).integers(0, cfg["n_vocab"], 128).astype(np.int32)
    runs = []
    for ctx in (137, 168, 200, 137):
        e = engine(cfg, 4321, ctx, 128)
        try:
            tok = e.prefill(prompt, 0)
            hid = e.hidden(128)
            lg = []
            for i in range(3):
                tok = e.decode(tok, 128 + i)
                lg.append(e.logits())
            runs.append((hid, np.stack(lg)))
        finally:
            e.close()
    for i, (hid, lg) in enumerate(runs[1:], 1):
        np.testing.assert_array_equal(hid, runs[0][0], err_msg=f"prefill residual stream, engine {i}")
        np.testing.assert_array_equal(lg, runs[0][1], err_msg=f"decode logits, engine {i}")
