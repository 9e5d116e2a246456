"""GPU parity: the decode-step self-attention with a group's shared slot-table prefix attended once
(``wt_self_attn_step_prefix``, ``self_attn_step_triton(shared_prefix_group=...)``) against the oracle.

The same tolerance as the step kernel (max-abs 2e-3 for fp16 in / fp32 accumulate, bf16 adds its rounding); the cache
append bit-exact. Cases: a prompt every row of a window reads from the window's first row (sampled windows, the
best-of-5 shape), rows that share more, less or nothing, offsets that differ inside a group, a last group that is
short, bf16, graph capture."""

import numpy as np
import pytest
import torch

from oracle import attn as oa
from whisper_trt_b200 import _lib
from whisper_trt_b200 import attn_plugin as ap

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]
ATOL = 2e-3


def assert_close(out: torch.Tensor, ref: np.ndarray, dtype=torch.float16):
    o = out.float().cpu().numpy()
    bound = ATOL + (2.0**-8 * np.abs(ref) if dtype == torch.bfloat16 else 0.0)
    assert np.isfinite(o).all()
    err = np.abs(o - ref)
    assert (err <= bound).all(), f"max err {err.max():.3e}"


def run_oracle(qkv, kc, vc, off, src):
    return oa.self_attn_step(qkv.float().cpu().numpy(), kc.float().cpu().numpy(), vc.float().cpu().numpy(),
                             off.cpu().numpy(), src.cpu().numpy())


def prompt_case(windows, k, c, prefix, lo, hi, dtype=torch.float16, seed=0, h=20):
    """Rows in windows of k: slots [0, prefix) read from the window's first row (a shared prompt), the rest from the
    row itself; offsets per window U[lo, hi]."""
    g = torch.Generator().manual_seed(seed)
    n = windows * k
    qkv = torch.randn(n, 1, 3 * h * 64, generator=g).to(dtype)
    kc = torch.randn(n, h, c, 64, generator=g).to(dtype)
    vc = torch.randn(n, h, c, 64, generator=g).to(dtype)
    rows = torch.arange(n)
    src = rows[:, None].repeat(1, c).clone()
    first = (rows // k * k)[:, None]
    src[:, :prefix] = first
    off = torch.randint(lo, hi + 1, (windows,), generator=g).repeat_interleave(k)
    return [t.cuda() for t in (qkv, kc, vc, off.long(), src.to(torch.int32))]


@pytest.mark.parametrize("windows,k,c,prefix,lo,hi", [(16, 5, 448, 224, 224, 447), (4, 5, 448, 224, 224, 230),
                                                     (3, 4, 96, 40, 40, 96), (2, 8, 228, 100, 50, 228),
                                                     (6, 5, 228, 3, 4, 228)])
def test_shared_prompt(windows, k, c, prefix, lo, hi):
    qkv, kc, vc, off, src = prompt_case(windows, k, c, prefix, lo, hi, seed=windows + c)
    ref = run_oracle(qkv, kc, vc, off, src)
    y = ap.self_attn_step_triton(qkv, kc, vc, off, src, shared_prefix_group=k)
    assert_close(y, ref)
    y2 = ap.self_attn_step_triton(qkv, kc, vc, off, src, shared_prefix_group=k, min_shared=1)
    assert_close(y2, ref)
    assert ap.workspace_errors() == 0


def test_append_is_bit_exact():
    qkv, kc, vc, off, src = prompt_case(4, 5, 448, 224, 224, 447, seed=7)
    k1, v1 = kc.clone(), vc.clone()
    ap.self_attn_step_triton(qkv, k1, v1, off, src, write_cache=True)
    k2, v2 = kc.clone(), vc.clone()
    ap.self_attn_step_triton(qkv, k2, v2, off, src, write_cache=True, shared_prefix_group=5)
    assert torch.equal(k1, k2) and torch.equal(v1, v2)


def test_partial_and_no_sharing():
    """Rows of a group diverge from the first row at different positions (some below min_shared, one at once), and
    a beam-like random slot table where little is shared: every row still gets its own attention."""
    qkv, kc, vc, off, src = prompt_case(6, 5, 228, 0, 100, 228, seed=3)
    src = src.cpu()
    for w in range(6):
        a = 5 * w
        for n, p in zip(range(5), (228, 150, 31, 0, 64)):
            src[a + n, :p] = a if n else src[a + n, :p]
    src = src.cuda()
    ref = run_oracle(qkv, kc, vc, off, src)
    for ms in (1, 32, 200):
        assert_close(ap.self_attn_step_triton(qkv, kc, vc, off, src, shared_prefix_group=5, min_shared=ms), ref)
    g = torch.Generator().manual_seed(11)
    n, c = 30, 228
    rnd = ((torch.arange(n) // 5 * 5)[:, None] + torch.randint(0, 5, (n, c), generator=g)).to(torch.int32).cuda()
    ref = run_oracle(qkv, kc, vc, off, rnd)
    assert_close(ap.self_attn_step_triton(qkv, kc, vc, off, rnd, shared_prefix_group=5, min_shared=1), ref)


def test_offsets_differ_inside_a_group_and_short_last_group():
    qkv, kc, vc, off, src = prompt_case(3, 5, 228, 120, 60, 228, seed=5)
    # 13 rows in groups of 5: the last group is 3 rows; offsets differ row by row (some below the prompt's end)
    n = 13
    qkv, kc, vc, src = qkv[:n].contiguous(), kc[:n].contiguous(), vc[:n].contiguous(), src[:n].contiguous()
    off = torch.tensor([228, 100, 150, 60, 121, 7, 119, 200, 228, 30, 180, 120, 90], device="cuda")
    ref = run_oracle(qkv, kc, vc, off, src)
    assert_close(ap.self_attn_step_triton(qkv, kc, vc, off, src, shared_prefix_group=5, min_shared=8), ref)


def test_bf16():
    qkv, kc, vc, off, src = prompt_case(5, 5, 448, 224, 224, 447, dtype=torch.bfloat16, seed=9)
    ref = run_oracle(qkv, kc, vc, off, src)
    assert_close(ap.self_attn_step_triton(qkv, kc, vc, off, src, shared_prefix_group=5), ref, torch.bfloat16)


def test_graph_capture_and_errors():
    qkv, kc, vc, off, src = prompt_case(8, 5, 448, 224, 224, 447, seed=13)
    ref = run_oracle(qkv, kc, vc, off, src)
    out = torch.empty(40, 1, 20 * 64, device="cuda", dtype=torch.float16)
    ap.self_attn_step_triton(qkv, kc, vc, off, src, shared_prefix_group=5, out=out)  # (warm-up: the workspace)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        ap.self_attn_step_triton(qkv, kc, vc, off, src, shared_prefix_group=5, out=out)
    out.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert_close(out, ref)
    with pytest.raises(ValueError):
        ap.self_attn_step_triton(qkv, kc, vc, off, src, shared_prefix_group=5, kv_splits=2)
    with pytest.raises(ValueError):
        ap.self_attn_step_triton(qkv, kc, vc, off, src, shared_prefix_group=9)
    lib = _lib.load()
    assert lib.wt_self_attn_step_prefix_workspace(40, 20, 64) == 40 * 20 * 66 * 4
