"""GPU parity: split / combined / fused cross-attention kernels (C ABI) against the oracle.

Tolerance: max-abs 2e-3 on the attention output (fp16 in, fp32 accumulate; bf16 adds its output rounding,
2^-8 * |ref|). The split partials are compared after normalisation: per slice the maximum m (log2 units) within
2e-3 * max(1, |m|) and acc / l within the output tolerance, l relative 1e-3 (exp2 of fp16-rounded scores)."""

import numpy as np
import pytest
import torch

import cases
from oracle import attn as oa
from whisper_trt_b200 import attn_plugin as ap

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]
ATOL = 2e-3


def assert_close(out, ref, dtype=torch.float16):
    o = out.float().cpu().numpy()
    bound = ATOL + (2.0**-8 * np.abs(ref) if dtype == torch.bfloat16 else 0.0)
    err = np.abs(o - ref)
    assert np.isfinite(o).all()
    assert (err <= bound).all(), f"max err {err.max():.3e}"


def oracle_inputs(q, k, v):
    return q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy()


def assert_parts_close(part, ref_part, dtype=torch.float16):
    p = part.cpu().numpy()
    d = p.shape[-1] - 2
    m, rm = p[..., d], ref_part[..., d]
    empty = np.isneginf(rm)
    assert np.array_equal(np.isneginf(m), empty)
    assert (np.abs(m[~empty] - rm[~empty]) <= 2e-3 * np.maximum(1, np.abs(rm[~empty]))).all()
    l, rl = p[..., d + 1], ref_part[..., d + 1]
    assert (np.abs(l[~empty] - rl[~empty]) <= 1e-3 * np.abs(rl[~empty]) + 1e-4).all()
    o = p[..., :d][~empty] / l[~empty][:, None]
    ro = ref_part[..., :d][~empty] / rl[~empty][:, None]
    bound = ATOL + (2.0**-8 * np.abs(ro) if dtype == torch.bfloat16 else 0.0)
    assert (np.abs(o - ro) <= bound).all(), np.abs(o - ro).max()


@pytest.mark.parametrize("name", ["cross_s1_f16", "cross_s5_f16", "cross_s20_f16"])
def test_golden_cross_cases(name, attn_golden):
    """The reference's cross cases (test_attn_plugin.py:73-107) against the stored reference outputs."""
    inp = {k: v.cuda() for k, v in cases.make_attn_inputs(*cases.ATTN_CASES[name]).items()}
    q, k, v = inp["q"], inp["xk"], inp["xv"]
    ref = attn_golden[f"{name}/cross"]
    assert_close(ap.cross_attn_triton(q, k, v), ref)
    part = ap.cross_attn_split_triton(q, k, v)
    assert_close(ap.cross_attn_combine_triton(part, q), ref)


def test_config1_split_partials(attn_golden):
    """Config 1's cross-attention (2 windows x 5 beams over 1500 frames): partials per slice and the output."""
    c1 = cases.config1_case(dtype=torch.float16)
    q, k, v = (c1[n].cuda() for n in ("q", "xk", "xv"))
    qn, kn, vn = oracle_inputs(q, k, v)
    ref_part = oa.cross_attn_split(qn, kn, vn)
    part = ap.cross_attn_split_triton(q, k, v)
    assert part.shape == (2, 20, 8, 5, 66)
    assert_parts_close(part, ref_part)
    ref = oa.cross_attn(qn, kn, vn)
    assert_close(ap.cross_attn_combine_triton(part, q), ref)
    assert_close(ap.cross_attn_triton(q, k, v), ref)
    assert np.abs(ref - attn_golden["config1_f32/cross"]).max() < 5e-3


def rand_cross(w, s, h, t, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(w, s, h * 64, generator=g).to(dtype).cuda()
    k = torch.randn(w, h, t, 64, generator=g).to(dtype).cuda()
    v = torch.randn(w, h, t, 64, generator=g).to(dtype).cuda()
    return q, k, v


@pytest.mark.parametrize("t", [1, 7, 15, 16, 17, 100, 188, 189, 1500])
@pytest.mark.parametrize("s", [1, 5, 8, 9])
def test_ragged_frames_and_query_counts(t, s):
    q, k, v = rand_cross(2, s, 3, t, torch.float16, seed=t * 31 + s)
    qn, kn, vn = oracle_inputs(q, k, v)
    ref = oa.cross_attn(qn, kn, vn)
    assert_close(ap.cross_attn_triton(q, k, v), ref)
    part = ap.cross_attn_split_triton(q, k, v)
    assert_parts_close(part, oa.cross_attn_split(qn, kn, vn))  # includes empty slices when t < 8
    assert_close(ap.cross_attn_combine_triton(part, q), ref)


@pytest.mark.parametrize("s", [16, 20, 32, 33, 40])
def test_many_queries(s):
    q, k, v = rand_cross(2, s, 2, 300, torch.float16, seed=s)
    ref = oa.cross_attn(*oracle_inputs(q, k, v))
    assert_close(ap.cross_attn_triton(q, k, v), ref)
    assert_close(ap.cross_attn_combine_triton(ap.cross_attn_split_triton(q, k, v), q), ref)


@pytest.mark.parametrize("w,s", [(4, 16), (4, 15), (8, 12), (32, 16), (4, 24), (4, 40)])
def test_stream_kernel_repeated_launches(w, s):
    """More than 8 queries per window take the persistent stream-K kernel, whose warps stream many blocks each at
    whisper's 20 heads x 1500 frames. Every one of 20 launches must match the oracle: a ring stage refilled by its
    copy before the warp's fragment loads of it are done corrupts one (window, head) at random, which a single launch
    can miss."""
    q, k, v = rand_cross(w, s, 20, 1500, torch.float16, seed=100 * w + s)
    ref = torch.from_numpy(oa.cross_attn(*oracle_inputs(q, k, v))).cuda()
    outs = [ap.cross_attn_triton(q, k, v) for _ in range(20)]
    errs = [float((y.float() - ref).abs().max()) for y in outs]
    assert max(errs) <= ATOL, errs
    assert all(torch.equal(y, outs[0]) for y in outs)  # (and every launch gives the same bits)


@pytest.mark.parametrize("w,s", [(8, 5), (32, 5), (16, 8), (3, 1), (24, 5)])
def test_window_kernel_repeated_launches(w, s):
    """At most 8 queries per window take the one-CTA-per-(window, head) kernel; 20 launches each match the oracle
    and give the same bits (its TMA rings are refilled while the warps still compute, as the stream-K kernel's).
    The launch picks its shape by the window count: 8 warps x 3 stages at 3 and 8 windows, 4 x 4 at 16 and 32,
    4 x 3 (4 CTAs per SM) at 24."""
    q, k, v = rand_cross(w, s, 20, 1500, torch.float16, seed=200 * w + s)
    ref = torch.from_numpy(oa.cross_attn(*oracle_inputs(q, k, v))).cuda()
    outs = [ap.cross_attn_triton(q, k, v) for _ in range(20)]
    assert max(float((y.float() - ref).abs().max()) for y in outs) <= ATOL
    assert all(torch.equal(y, outs[0]) for y in outs)


@pytest.mark.parametrize("w,s", [(32, 5), (8, 5), (4, 16)])
def test_split_repeated_launches(w, s):
    """The reference-shaped split (8 key slices per (window, head), on the stream-K kernel in slice mode): 20
    launches give the same partials, and their combine matches the oracle."""
    q, k, v = rand_cross(w, s, 20, 1500, torch.float16, seed=300 * w + s)
    parts = [ap.cross_attn_split_triton(q, k, v) for _ in range(20)]
    assert all(torch.equal(p, parts[0]) for p in parts)
    assert_close(ap.cross_attn_combine_triton(parts[0], q), oa.cross_attn(*oracle_inputs(q, k, v)))


@pytest.mark.parametrize("w", [1, 8, 32])
def test_whisper_shapes(w):
    """20 heads x 64 over 1500 frames, beam 5 (configs 2 / 3 per layer) -- fused and split paths."""
    q, k, v = rand_cross(w, 5, 20, 1500, torch.float16, seed=w)
    ref = oa.cross_attn(*oracle_inputs(q, k, v))
    assert_close(ap.cross_attn_triton(q, k, v), ref)
    assert_close(ap.cross_attn_combine_triton(ap.cross_attn_split_triton(q, k, v), q), ref)


def test_bf16():
    q, k, v = rand_cross(3, 5, 20, 1500, torch.bfloat16, seed=9)
    qn, kn, vn = oracle_inputs(q, k, v)
    ref = oa.cross_attn(qn, kn, vn)
    assert_close(ap.cross_attn_triton(q, k, v), ref, torch.bfloat16)
    part = ap.cross_attn_split_triton(q, k, v)
    assert_parts_close(part, oa.cross_attn_split(qn, kn, vn), torch.bfloat16)
    assert_close(ap.cross_attn_combine_triton(part, q), ref, torch.bfloat16)


def test_peaked_softmax_precision():
    """Large scores (one key dominating) stress the fp16 rounding of P before the P.V product."""
    q, k, v = rand_cross(2, 5, 4, 1500, torch.float16, seed=13)
    q = (q.float() * 6).half()
    ref = oa.cross_attn(*oracle_inputs(q, k, v))
    assert_close(ap.cross_attn_triton(q, k, v), ref)


def test_fused_workspace_reuse_and_graph_capture():
    q, k, v = rand_cross(4, 5, 20, 1500, torch.float16, seed=17)
    ref = oa.cross_attn(*oracle_inputs(q, k, v))
    y = ap.cross_attn_triton(q, k, v)
    assert_close(y, ref)
    out = torch.empty_like(y)
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        ap.cross_attn_triton(q, k, v, out=out)
    for _ in range(3):
        gr.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, y)


def test_split_matches_reference_slice_boundaries():
    """Slice i covers [i*188, min((i+1)*188, 1500)) as the reference's chunk = ceil(T / SPLITS)."""
    q, k, v = rand_cross(1, 5, 2, 1500, torch.float16, seed=3)
    v2 = v.clone()
    v2[:, :, 188:] = 0  # only slice 0 sees nonzero values
    part = ap.cross_attn_split_triton(q, k, v2)
    assert part[:, :, 0, :, :64].abs().sum() > 0
    assert part[:, :, 1:, :, :64].abs().sum() == 0


def test_fused_alternating_shapes():
    """Shapes with different in-kernel split counts one after another (each shape keeps its own workspace)."""
    cases_ = [rand_cross(w, 5, 20, 1500, torch.float16, seed=40 + w) for w in (1, 8, 2, 8, 1)]
    refs = [oa.cross_attn(*oracle_inputs(*c)) for c in cases_]
    for _ in range(2):
        for c, ref in zip(cases_, refs):
            assert_close(ap.cross_attn_triton(*c), ref)


def test_no_device_errors_recorded():
    """No kernel of the tests above gave up a bounded wait (the workspaces' device error words are zero)."""
    q, k, v = rand_cross(2, 5, 20, 1500, torch.float16, seed=77)
    ap.cross_attn_triton(q, k, v)
    assert ap.workspace_errors() == 0
