"""GPU parity of the Q4_0 x Q8_0 mat-vec path against the oracle, through the C ABI.

Bar (north_star): int32 block dots bit-exact; y within 1e-3 relative
(tests/util.py) of the reference's NEON fp32 chain; Q8_0 quantization and the
GPU repack bit-exact.  The kernel runs the reference's own fp32 fma chain over
the blocks in order (gemm.cpp:179-181), so y is asserted bit-identical to the
oracle's restatement of that chain, and the lm-head path (generic mul_mat,
vec_dot_q4_0_q8_0 lanes, arm.cpp:633-692) bit-identical to its restatement.
"""
import numpy as np
import pytest

import arclight_b200 as A
from oracle import lib as O
from tests.util import assert_rel

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def stream():
    return torch.cuda.current_stream().cuda_stream


def dev(a: np.ndarray):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.uint8).reshape(-1).copy()).cuda()


def make_case(N, K, seed):
    """Config-1 recipe: W ~ N(0, 0.02) -> Q4_0 (types.cpp:352-378); x ~ N(0,1) -> Q8_0 (RNE)."""
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    x = rng.standard_normal(K).astype(np.float32)
    return O.quantize_q4_0(w), x


def upload_weight(wq: np.ndarray):
    N, nb = wq.shape
    K = nb * 32
    src = dev(wq)
    W = torch.empty(A.lib().alb_q4_0_gpu_bytes(N, K), dtype=torch.uint8, device="cuda")
    A.check(A.lib().alb_repack_q4_0(W.data_ptr(), src.data_ptr(), N, K, stream()), "repack")
    return W


SHAPES = [
    (9728, 2560),    # config 1 (ffn gate/up of Qwen3-4B)
    (6144, 2560),    # fused QKV 4B
    (2560, 4096),    # o_proj 4B
    (2560, 9728),    # down_proj 4B
    (1024, 3072),    # down 0.6B
    (4096, 12288),   # down 8B (K at the maximum the kernel supports)
    (1216, 2560),    # TP=8 gate shard
    (2560, 1216),    # TP=8 down shard
    (33, 96),        # ragged: odd rows, 3 blocks
    (1, 32),         # minimal
]


@pytest.mark.parametrize("N,K", SHAPES)
def test_gemv_block_dots_bit_exact_and_y_within_tol(N, K):
    wq, x = make_case(N, K, seed=N * 131 + K)
    xq = O.quantize_q8_0(x)
    y_ref, dots_ref = O.gemv(wq, xq)

    W = upload_weight(wq)
    Xq = dev(xq)
    y = torch.empty(N, dtype=torch.float32, device="cuda")
    I = torch.empty((N, K // 32), dtype=torch.int32, device="cuda")
    A.check(A.lib().alb_gemv_q4_0_q8_0(W.data_ptr(), Xq.data_ptr(), y.data_ptr(), N, K, None, stream()), "gemv")
    A.check(A.lib().alb_gemv_q4_0_q8_0_block_dots(W.data_ptr(), Xq.data_ptr(), I.data_ptr(), N, K, stream()), "dots")
    torch.cuda.synchronize()
    np.testing.assert_array_equal(I.cpu().numpy(), dots_ref)
    assert_rel(y.cpu().numpy(), y_ref, what=f"gemv {N}x{K}")
    np.testing.assert_array_equal(y.cpu().numpy(), y_ref)   # the NEON chain, bit for bit


@pytest.mark.parametrize("N,K", [(151936 // 8, 2560), (4096, 1024), (2048, 4096), (37, 96), (5, 32), (300, 2592)])
def test_mul_mat_vec_dot_chain_bit_exact(N, K):
    """The lm head's generic mul_mat (vec_dot lanes, pair chains, fixed add tree;
    odd block counts take the scalar tail) against its restatement."""
    wq, x = make_case(N, K, seed=N + 3 * K)
    xq = O.quantize_q8_0(x)
    W = upload_weight(wq)
    Xq = dev(xq)
    y = torch.full((N,), float("nan"), dtype=torch.float32, device="cuda")
    for _ in range(2):
        A.check(A.lib().alb_mul_mat_q4_0_q8_0(W.data_ptr(), Xq.data_ptr(), y.data_ptr(), N, K, stream()), "mul_mat")
        torch.cuda.synchronize()
        ref = O.mul_mat_generic(wq, xq)
        assert_rel(y.cpu().numpy(), O.gemv(wq, xq)[0], rtol=1e-3, what=f"mul_mat {N}x{K} vs gemv chain")
        np.testing.assert_array_equal(y.cpu().numpy(), ref)


def test_gemv_residual_add():
    N, K = 2560, 4096
    wq, x = make_case(N, K, seed=7)
    xq = O.quantize_q8_0(x)
    y_ref, _ = O.gemv(wq, xq)
    res = np.random.default_rng(8).standard_normal(N).astype(np.float32)
    W = upload_weight(wq)
    Xq = dev(xq)
    r = torch.from_numpy(res).cuda()
    y = r.clone()  # in place, as the residual stream x = o + x
    A.check(A.lib().alb_gemv_q4_0_q8_0(W.data_ptr(), Xq.data_ptr(), y.data_ptr(), N, K, y.data_ptr(), stream()))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(y.cpu().numpy(), (y_ref + res).astype(np.float32))


@pytest.mark.parametrize("rows,K", [(1, 2560), (7, 4096), (3, 9728), (2048, 2560)])
def test_quantize_q8_0_bit_exact(rows, K):
    rng = np.random.default_rng(rows + K)
    x = (rng.standard_normal((rows, K)) * np.exp2(rng.integers(-8, 8, (rows, 1)))).astype(np.float32)
    x[0, :32] = 0.0                       # zero block
    x[-1, 32:64] = np.arange(32) - 15.5   # exact .5 ties after scaling
    ref = O.quantize_q8_0(x)
    X = torch.from_numpy(x).cuda()
    Y = torch.empty(rows * (K // 32) * 34, dtype=torch.uint8, device="cuda")
    A.check(A.lib().alb_quantize_q8_0(X.data_ptr(), Y.data_ptr(), K, rows, stream()))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(Y.cpu().numpy(), ref.reshape(-1).view(np.uint8))


def test_repack_round_trip():
    wq, _ = make_case(64, 4096, seed=3)
    W = upload_weight(wq)
    back = torch.empty(wq.size * 18, dtype=torch.uint8, device="cuda")
    A.check(A.lib().alb_unpack_q4_0(back.data_ptr(), W.data_ptr(), 64, 4096, stream()))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(back.cpu().numpy(), wq.reshape(-1).view(np.uint8))


def test_gemv_zero_activation_and_zero_weight():
    N, K = 64, 256
    wq = O.quantize_q4_0(np.zeros((N, K), np.float32))
    xq = O.quantize_q8_0(np.zeros(K, np.float32))
    W = upload_weight(wq)
    Xq = dev(xq)
    y = torch.full((N,), 7.0, dtype=torch.float32, device="cuda")
    A.check(A.lib().alb_gemv_q4_0_q8_0(W.data_ptr(), Xq.data_ptr(), y.data_ptr(), N, K, None, stream()))
    torch.cuda.synchronize()
    assert not y.cpu().numpy().any()
