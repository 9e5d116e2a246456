"""The failure path of the kernels' bounded waits (failure detection), on the GPU, without a fault.

Every device-side wait polls a bounded number of times (``wt_set_wait_limit``) and then records an error code in
the call's device error word and gives up, so that the kernel returns and the context stays usable. Here the wait
is made to run out on purpose: the test hook ``wt_set_test_withhold_stage`` makes the fused cross-attention issue
no copy for the first ring stage of its first streaming warp (a barrier nothing completes), with a short limit of
2^10 polls. The call must return (the synchronisation below ends), the error word must be set, and the next call
-- the hook off, the workspace re-zeroed -- must match the oracle within the attention tolerance (2e-3).
"""

import numpy as np
import pytest
import torch

from oracle import attn as oracle
from whisper_trt_b200 import _lib

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]


def _call(lib, q, k, v, ws):
    w, s, _ = q.shape
    h, t = k.shape[1], k.shape[2]
    y = torch.full_like(q, float("nan"))
    st = lib.wt_cross_attn(_lib.WT_F16, q.data_ptr(), k.data_ptr(), v.data_ptr(), y.data_ptr(), w, s, h, t, 64,
                           ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream)
    assert st == _lib.WT_OK, lib.wt_last_error()
    return y


@pytest.mark.parametrize("windows,S", [(2, 5), (32, 5), (4, 16)])  # (window kernel; 16 queries: stream-K kernel)
def test_cross_attn_wait_runs_out_then_recovers(windows, S):
    lib = _lib.load()
    g = torch.Generator().manual_seed(windows)
    H, T = 20, 1500
    q = torch.randn(windows, S, H * 64, generator=g).half().cuda()
    k = torch.randn(windows, H, T, 64, generator=g).half().cuda()
    v = torch.randn(windows, H, T, 64, generator=g).half().cuda()
    nbytes = lib.wt_cross_attn_workspace(windows, S, H, T, 64)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    prev_limit = lib.wt_set_wait_limit(1 << 10)
    prev_hook = lib.wt_set_test_withhold_stage(1)
    try:
        _call(lib, q, k, v, ws)
        torch.cuda.synchronize()  # (returns: the wait ran out instead of hanging)
    finally:
        lib.wt_set_test_withhold_stage(prev_hook)
        lib.wt_set_wait_limit(prev_limit)
    assert int(ws[:4].view(torch.int32).item()) != 0  # the timeout was recorded
    ws.zero_()
    y = _call(lib, q, k, v, ws)
    torch.cuda.synchronize()
    assert int(ws[:4].view(torch.int32).item()) == 0
    want = oracle.cross_attn(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy())
    err = float(np.abs(y.float().cpu().numpy() - want).max())
    assert err <= 2e-3, err


def test_wait_limit_setting_round_trips():
    lib = _lib.load()
    prev = lib.wt_set_wait_limit(12345)
    try:
        assert lib.wt_set_wait_limit(0) == 12345  # (0 restores the default)
        assert lib.wt_set_wait_limit(prev) == 1 << 22
    finally:
        lib.wt_set_wait_limit(prev)
