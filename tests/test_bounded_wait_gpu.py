"""The failure path of the kernels' bounded waits (failure detection), on the GPU, without a fault.

Every device-side wait polls a bounded number of times (``wt_set_wait_limit``) and then records an error code in
the call's device error word and gives up, so that the kernel returns and the context stays usable. Here the wait
is made to run out on purpose: the test hook ``wt_set_test_withhold_stage`` makes the fused cross-attention issue
no copy for the first ring stage of its first streaming warp, and logits32 / the decoder GEMMs leave out the row
block of their first CTA's first stage (a barrier nothing completes), with a short limit of 2^10 polls. The call
must return (the synchronisation below ends), the error word must be set, and the next call -- the hook off, the
workspace re-zeroed -- must match the oracle within the tolerance of the kernel's own parity tests.
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


@pytest.mark.parametrize("windows,S", [(2, 5), (32, 5), (24, 5), (4, 16)])  # (window kernel, its 3 shapes; stream-K)
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


def test_logits_wait_runs_out_then_recovers():
    """logits32's producer leaves out the row block of CTA 0's first stage: the MMA issuer's wait on it runs out and
    raises the CTA's stop flag, the other roles stop, the copies that were issued are waited for and the tensor
    memory is freed. The call returns with its error word set; the next call matches an fp64 product."""
    lib = _lib.load()
    g = torch.Generator(device="cuda").manual_seed(5)
    rows, vocab, d = 160, 4096, 1280
    x = torch.randn(rows, d, generator=g, device="cuda").half()
    w = (torch.randn(vocab, d, generator=g, device="cuda") * 0.02).half()
    err = torch.zeros(64, dtype=torch.int32, device="cuda")
    y = torch.full((rows, vocab), float("nan"), device="cuda")

    def call():
        st = lib.wt_logits32(_lib.WT_F16, x.data_ptr(), w.data_ptr(), y.data_ptr(), rows, vocab, d, err.data_ptr(),
                             torch.cuda.current_stream().cuda_stream)
        assert st == _lib.WT_OK, lib.wt_last_error()

    prev_limit = lib.wt_set_wait_limit(1 << 10)
    prev_hook = lib.wt_set_test_withhold_stage(1)
    try:
        call()
        torch.cuda.synchronize()
    finally:
        lib.wt_set_test_withhold_stage(prev_hook)
        lib.wt_set_wait_limit(prev_limit)
    assert int(err[0].item()) != 0
    err.zero_()
    call()
    torch.cuda.synchronize()
    assert int(err[0].item()) == 0
    ref = (x.double() @ w.double().t()).float()
    assert ((y - ref).abs() <= 1e-4 * (1 + ref.abs())).all()


@pytest.mark.parametrize("rows,out,inp", [(160, 1280, 1280), (160, 1280, 5120), (40, 3840, 1280)])
def test_dec_linear_wait_runs_out_then_recovers(rows, out, inp):
    """The decoder GEMM (k splits over a cluster where the shape takes them): CTA 0's producer leaves out its first
    stage's row block; its MMA issuer's wait runs out, the CTA stops issuing, still meets its cluster's barriers,
    waits for its copies and frees its tensor memory. The call returns with the error word set; the next call on a
    re-zeroed workspace matches the oracle (one unit in the last place of fp16)."""
    import cases
    from oracle import decoder as od

    lib = _lib.load()
    t = {k_: v_.half().cuda() for k_, v_ in cases.linear_case(m=rows, n=out, k=inp, seed=rows + out).items()}
    nbytes = lib.wt_dec_linear_workspace(rows, out, inp, 0)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    y = torch.full((rows, out), float("nan"), device="cuda").half()

    def call():
        st = lib.wt_linear_residual(_lib.WT_F16, t["x"].data_ptr(), t["w"].data_ptr(), t["b"].data_ptr(),
                                    t["res"].data_ptr(), y.data_ptr(), rows, out, inp, ws.data_ptr(), ws.numel(),
                                    torch.cuda.current_stream().cuda_stream)
        assert st == _lib.WT_OK, lib.wt_last_error()

    prev_limit = lib.wt_set_wait_limit(1 << 10)
    prev_hook = lib.wt_set_test_withhold_stage(1)
    try:
        call()
        torch.cuda.synchronize()
    finally:
        lib.wt_set_test_withhold_stage(prev_hook)
        lib.wt_set_wait_limit(prev_limit)
    assert int(ws[:4].view(torch.int32).item()) != 0
    ws.zero_()
    call()
    torch.cuda.synchronize()
    assert int(ws[:4].view(torch.int32).item()) == 0
    f = lambda a: a.float().cpu().numpy()  # noqa: E731
    want = od.linear_residual(f(t["x"]), f(t["w"]), f(t["b"]), f(t["res"]))
    np.testing.assert_allclose(f(y), want, rtol=2e-3, atol=2e-3)
