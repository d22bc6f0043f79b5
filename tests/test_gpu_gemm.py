"""GPU parity of the prefill Q4_0 x Q8_0 mat-mul (tcgen05 kind::i8 block dots,
fp32 chains in the epilogue) against the oracle, row by row.

Bar (north_star): per-op fp32 outputs within 1e-3 relative of the reference's
NEON chain.  The reference's gemm (gemm.cpp:495-974) accumulates each output
with the same fp32 fma chain over the blocks as its gemv, so every GPU output
row is asserted bit-identical to the oracle's NEON-chain mat-vec of that row,
including the config-4 prefill shapes (M = 2048 tokens, N = 6144 / 19456,
K = 2560; rows sampled across every M tile).
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


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.uint8).reshape(-1).copy()).cuda()


def upload_weight(wq):
    N, nb = wq.shape
    K = nb * 32
    src = dev(wq)
    W = torch.empty(A.lib().alb_q4_0_gpu_bytes(N, K), dtype=torch.uint8, device="cuda")
    A.check(A.lib().alb_repack_q4_0(W.data_ptr(), src.data_ptr(), N, K, stream()), "repack")
    return W


@pytest.mark.parametrize("M,N,K", [
    (256, 512, 2560),    # 4B hidden, two M tiles
    (100, 200, 4096),    # ragged M and N (o_proj K)
    (1, 64, 32),         # minimal
    (300, 64, 9728),     # down_proj K
    (128, 1216, 2560),   # TP=8 gate/up shard width
    (2048, 6144, 2560),  # config 4: fused QKV of the 4B over a 2048-token prompt
    (2048, 19456, 2560), # config 4: gate/up
    (2048, 2560, 9728),  # config 4: down
])
def test_gemm_rows_match_chain_gemv(M, N, K):
    rng = np.random.default_rng(M * 7 + N + K)
    wq = O.quantize_q4_0((rng.standard_normal((N, K)) * 0.02).astype(np.float32))
    x = rng.standard_normal((M, K)).astype(np.float32)
    x[0, :32] = 0.0                                   # an all-zero activation block
    xq = O.quantize_q8_0(x)                           # [M][K/32] block_q8_0
    W = upload_weight(wq)
    Xq = dev(xq)
    ws = torch.empty(A.lib().alb_gemm_workspace_bytes(M, K), dtype=torch.uint8, device="cuda")
    y = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
    A.check(A.lib().alb_gemm_q4_0_q8_0(W.data_ptr(), Xq.data_ptr(), y.data_ptr(), M, N, K, None, ws.data_ptr(),
                                       stream()), "gemm")
    torch.cuda.synchronize()
    assert A.lib().alb_device_error(0) == 0
    got = y.cpu().numpy()
    assert np.all(np.isfinite(got)), "unwritten outputs"
    rows = range(M) if M <= 300 else sorted(set(list(range(0, M, 61)) + [1, 127, 128, 1023, M - 1]))
    for m in rows:
        ref, _ = O.gemv(wq, xq[m])
        np.testing.assert_array_equal(got[m], ref, err_msg=f"row {m}")
    ref_neon, _ = O.gemv(wq, xq[M - 1])
    assert_rel(got[M - 1], ref_neon, what=f"gemm {M}x{N}x{K} vs NEON chain")


def test_gemm_residual():
    M, N, K = 130, 128, 2560
    rng = np.random.default_rng(5)
    wq = O.quantize_q4_0((rng.standard_normal((N, K)) * 0.02).astype(np.float32))
    xq = O.quantize_q8_0(rng.standard_normal((M, K)).astype(np.float32))
    res = rng.standard_normal((M, N)).astype(np.float32)
    W, Xq = upload_weight(wq), dev(xq)
    ws = torch.empty(A.lib().alb_gemm_workspace_bytes(M, K), dtype=torch.uint8, device="cuda")
    r = torch.from_numpy(res).cuda()
    y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    A.check(A.lib().alb_gemm_q4_0_q8_0(W.data_ptr(), Xq.data_ptr(), y.data_ptr(), M, N, K, r.data_ptr(),
                                       ws.data_ptr(), stream()))
    torch.cuda.synchronize()
    got = y.cpu().numpy()
    for m in (0, 64, M - 1):
        exp = (O.gemv(wq, xq[m])[0] + res[m]).astype(np.float32)
        np.testing.assert_array_equal(got[m], exp)
