"""GPU parity: the decode-step self-attention kernel (C ABI ``wt_self_attn_step``) against the oracle.

Tolerance: max-abs 2e-3 for fp16 in / fp32 accumulate (the reference's own bar for this kernel,
test_attn_plugin.py:57); bf16 outputs add their rounding: 2e-3 + 2^-8 * |ref|. The cache append is bit-exact, and
writing it leaves the attention output bit-identical (test_attn_plugin.py:58-70)."""

import numpy as np
import pytest
import torch

import cases
from oracle import attn as oa
from whisper_trt_b200 import attn_plugin as ap

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]
ATOL = 2e-3


def tol(dtype, ref):
    return ATOL + (2.0**-8 * np.abs(ref) if dtype == torch.bfloat16 else 0.0)


def assert_close(out: torch.Tensor, ref: np.ndarray, dtype=torch.float16):
    o = out.float().cpu().numpy()
    err = np.abs(o - ref)
    bound = tol(dtype, ref)
    assert np.isfinite(o).all()
    assert (err <= bound).all(), f"max err {err.max():.3e} (bound {np.max(bound):.3e})"


def run_oracle(qkv, kc, vc, off, src):
    return oa.self_attn_step(qkv.float().cpu().numpy(), kc.float().cpu().numpy(), vc.float().cpu().numpy(),
                             off.cpu().numpy(), src.cpu().numpy())


def test_golden_step_case(attn_golden):
    """The reference's own step case (test_attn_plugin.py:50-57) against the stored reference output."""
    inp = cases.make_attn_inputs(*cases.ATTN_CASES["self_step_f16"])
    d = {k: v.cuda() for k, v in inp.items()}
    for splits in (1, 2, 5):
        y = ap.self_attn_step_triton(d["qkv"], d["kc"], d["vc"], d["offset"], d["src"], kv_splits=splits)
        assert_close(y, attn_golden["self_step_f16/self"])
    off40 = torch.full_like(d["offset"], 40)
    y = ap.self_attn_step_triton(d["qkv"], d["kc"], d["vc"], off40, d["src"])
    assert_close(y, attn_golden["self_step_f16/self_off40"])


def test_write_cache_is_bit_exact_and_does_not_change_the_output():
    qkv, kc, vc, offset, src = (t.cuda() for t in cases.plugin_case(b=10, s=1, h=20, c=96, dtype=torch.float16))
    offset.fill_(40)  # a window's rows share their offset: no row reads the slot being written
    out = ap.self_attn_step_triton(qkv, kc, vc, offset, src)
    k2, v2 = kc.clone(), vc.clone()
    again = ap.self_attn_step_triton(qkv, k2, v2, offset, src, write_cache=True)
    assert torch.equal(again, out)
    new = qkv.view(10, 3, 20, 64)
    k_exp, v_exp = kc.clone(), vc.clone()
    k_exp[:, :, 40], v_exp[:, :, 40] = new[:, 1], new[:, 2]
    assert torch.equal(k2, k_exp) and torch.equal(v2, v_exp)


def test_config1(attn_golden):
    """Benchmark config 1 (2 windows x beam 5, 24 cached + the new token), fp16 inputs; append into slot 24."""
    c1 = cases.config1_case(dtype=torch.float16)
    d = {k: v.cuda() for k, v in c1.items()}
    ref = run_oracle(d["qkv"], d["kc"], d["vc"], d["offset"], d["src"])
    k2, v2 = d["kc"].clone(), d["vc"].clone()
    y = ap.self_attn_step_triton(d["qkv"], k2, v2, d["offset"], d["src"], write_cache=True)
    assert_close(y, ref)
    assert np.abs(ref - attn_golden["config1_f32/self"]).max() < 5e-3  # (fp16-rounded inputs vs the fp32 case)
    assert torch.equal(k2[:, :, 24], d["qkv"].view(10, 3, 20, 64)[:, 1])


def rand_case(n, h, c, d, dtype, seed, offsets=None, src_lo=None, src_hi=None):
    g = torch.Generator().manual_seed(seed)
    qkv = torch.randn(n, 1, 3 * h * d, generator=g).to(dtype)
    kc = torch.randn(n, h, c, d, generator=g).to(dtype)
    vc = torch.randn(n, h, c, d, generator=g).to(dtype)
    off = torch.randint(0, c + 1, (n,), generator=g) if offsets is None else torch.as_tensor(offsets)
    src = torch.randint(0 if src_lo is None else src_lo, n if src_hi is None else src_hi, (n, c), generator=g)
    return [t.cuda() for t in (qkv, kc, vc, off.long(), src.to(torch.int32))]


@pytest.mark.parametrize("c", [1, 15, 16, 17, 63, 96, 228, 448])
@pytest.mark.parametrize("splits", [None, 1, 3])
def test_ragged_offsets_and_capacities(c, splits):
    qkv, kc, vc, off, src = rand_case(12, 5, c, 64, torch.float16, seed=c)
    off[0], off[1] = 0, c  # only the new token; a full cache (no write there: slot C does not exist)
    ref = run_oracle(qkv, kc, vc, off, src)
    y = ap.self_attn_step_triton(qkv, kc, vc, off, src, kv_splits=splits)
    assert_close(y, ref)
    # the append alone (rows with different offsets may read each other's written slot: the output is checked
    # above without writing, as in the reference's contract)
    k2, v2 = kc.clone(), vc.clone()
    ap.self_attn_step_triton(qkv, k2, v2, off, src, write_cache=True, kv_splits=splits)
    ke, ve = kc.cpu().numpy().copy(), vc.cpu().numpy().copy()
    oa.cache_append(ke, ve, qkv.cpu().numpy(), off.clamp(0, c).cpu().numpy())
    assert np.array_equal(k2.cpu().numpy().view(np.int16), ke.view(np.int16))
    assert np.array_equal(v2.cpu().numpy().view(np.int16), ve.view(np.int16))
    assert torch.equal(k2[1], kc[1])  # offset == C: nothing written


@pytest.mark.parametrize("d", [16, 32, 64, 128])
def test_head_dims(d):
    qkv, kc, vc, off, src = rand_case(6, 3, 40, d, torch.float16, seed=d)
    assert_close(ap.self_attn_step_triton(qkv, kc, vc, off, src), run_oracle(qkv, kc, vc, off, src))
    assert_close(ap.self_attn_step_triton(qkv, kc, vc, off, src, kv_splits=4), run_oracle(qkv, kc, vc, off, src))


@pytest.mark.parametrize("splits", [1, 2, 6])
def test_bf16(splits):
    qkv, kc, vc, off, src = rand_case(10, 20, 96, 64, torch.bfloat16, seed=7)
    y = ap.self_attn_step_triton(qkv, kc, vc, off, src, kv_splits=splits)
    assert_close(y, run_oracle(qkv, kc, vc, off, src), torch.bfloat16)


def test_out_of_range_offsets_and_rows_are_clamped():
    """offset clamped to [0, C], src to [0, N-1] (attn_plugin.py:321, :338-339): no fault, the oracle's result."""
    qkv, kc, vc, off, src = rand_case(8, 4, 32, 64, torch.float16, seed=3, src_lo=-5, src_hi=20)
    off[:4] = torch.tensor([-7, 0, 33, 1000])
    y = ap.self_attn_step_triton(qkv, kc, vc, off, src)
    assert_close(y, run_oracle(qkv, kc, vc, off, src))


def test_split_workspace_is_left_zeroed_and_reusable():
    qkv, kc, vc, off, src = rand_case(4, 2, 200, 64, torch.float16, seed=11)
    ref = run_oracle(qkv, kc, vc, off, src)
    for _ in range(3):  # the last CTA resets its counter: repeated launches stay correct
        assert_close(ap.self_attn_step_triton(qkv, kc, vc, off, src, kv_splits=8), ref)
    ws = ap._workspaces[(torch.cuda.current_device(), "self", (4, 2, 64, 8))]
    assert int(ws[: 4 * 2 * 4].view(torch.int32).abs().sum()) == 0


def test_large_rows_heads_config2_shape():
    """Config 2's per-layer shape (40 rows x 20 heads, 80 cached, C = 228), a random parent permutation per window."""
    g = torch.Generator().manual_seed(5)
    n, h, c, d = 40, 20, 228, 64
    qkv = torch.randn(n, 1, 3 * h * d, generator=g).half().cuda()
    kc = torch.randn(n, h, c, d, generator=g).half().cuda()
    vc = torch.randn(n, h, c, d, generator=g).half().cuda()
    off = torch.full((n,), 80, dtype=torch.long, device="cuda")
    src = torch.stack([torch.randperm(5, generator=g) for _ in range(8 * c)]).view(8, c, 5).permute(0, 2, 1)
    src = (src + (torch.arange(8) * 5)[:, None, None]).reshape(n, c).to(torch.int32).cuda()
    y = ap.self_attn_step_triton(qkv, kc, vc, off, src, write_cache=True)
    assert_close(y, run_oracle(qkv, kc, vc, off, src))


def test_graph_capture_replays_the_same():
    qkv, kc, vc, off, src = rand_case(10, 20, 96, 64, torch.float16, seed=21)
    y = ap.self_attn_step_triton(qkv, kc, vc, off, src)  # warm-up outside capture
    out = torch.empty_like(y)
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        ap.self_attn_step_triton(qkv, kc, vc, off, src, out=out)
    gr.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, y)
