"""alb_flash_attn_static (fixed device workspace, no allocation) against
alb_flash_attn on the same inputs, two calls in a row each.

Collected last (file name) so that it also runs after every other test has
used the device; it passes alone as well.
"""
import math

import numpy as np
import pytest

import arclight_b200 as A

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _fp16(rng, shape):
    return torch.from_numpy(rng.standard_normal(shape).astype(np.float16)).cuda()


@pytest.mark.parametrize("Hq,Hkv,T,pos0,S", [
    (32, 8, 1, 639, 18),     # 4B decode, split over 18 CTAs per kv head
    (32, 8, 1, 0, 74),       # first token: most splits empty
    (16, 8, 1, 200, 16),     # GQA 2:1
    (32, 8, 4, 300, 4),      # a few tokens, split
    (32, 8, 7, 100, 1),      # small ubatch, one split
    (32, 8, 512, 0, 1),      # prefill ubatch: the tiled kernel needs no workspace, so no size limit applies
])
def test_static_workspace_matches_caller_workspace(Hq, Hkv, T, pos0, S):
    L = A.lib()
    stream = torch.cuda.current_stream().cuda_stream
    rng = np.random.default_rng(7 * Hq + T + pos0)
    cells = pos0 + T
    k, v = _fp16(rng, (cells, Hkv, 128)), _fp16(rng, (cells, Hkv, 128))
    q = torch.from_numpy((rng.standard_normal((T, Hq, 128)) * 0.5).astype(np.float32)).cuda()
    scale = 1.0 / math.sqrt(128.0)
    need = L.alb_flash_attn_workspace_bytes(Hq, Hkv, T, S, cells)
    if not (T > 1 and S == 1):
        assert need <= A.ALB_FLASH_ATTN_STATIC_BYTES
    ws = torch.zeros(max(1, min(need, A.ALB_FLASH_ATTN_STATIC_BYTES)), dtype=torch.uint8, device="cuda")
    ref = torch.empty((T, Hq, 128), dtype=torch.float32, device="cuda")
    out = torch.empty_like(ref)
    for rep in range(2):
        A.check(L.alb_flash_attn(q.data_ptr(), k.data_ptr(), v.data_ptr(), T, Hq, Hkv, pos0, scale, S,
                                 ws.data_ptr(), ref.data_ptr(), stream), "alb_flash_attn")
        out.fill_(float("nan"))
        A.check(L.alb_flash_attn_static(q.data_ptr(), k.data_ptr(), v.data_ptr(), T, Hq, Hkv, pos0, scale, S,
                                        out.data_ptr(), stream), "alb_flash_attn_static")
        torch.cuda.synchronize()
        assert A.lib().alb_device_error(0) == 0
        np.testing.assert_array_equal(out.cpu().numpy(), ref.cpu().numpy(), err_msg=f"call {rep}")


def test_static_workspace_rejects_oversized_calls():
    L = A.lib()
    stream = torch.cuda.current_stream().cuda_stream
    # 32 q heads over 100 000 cells in 18 splits: the score rows alone exceed 4 MiB
    assert L.alb_flash_attn_workspace_bytes(32, 8, 1, 18, 100000) > A.ALB_FLASH_ATTN_STATIC_BYTES
    dummy = torch.zeros(16, dtype=torch.float32, device="cuda")
    rc = L.alb_flash_attn_static(dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(), 1, 32, 8, 99999,
                                 1.0, 18, dummy.data_ptr(), stream)
    assert rc == A.ALB_ERR_INVALID
    assert b"ALB_FLASH_ATTN_STATIC_BYTES" in L.alb_last_error()
