"""GPU parity against the reference's own Triton kernels (its ``attn_plugin`` and ``beam_kernels`` launchers, run
unmodified as black boxes) on the same inputs: a second anchor beside the CPU oracle.

Needs the reference package staged at ``baseline/_ref/whisper_trt`` (git-ignored; see the design notes) and Triton;
skipped otherwise. Tolerances: attention outputs within max-abs 2e-3 (the path's fp16 bar), logits32 within 1e-4
relative, beam scoring the same best 2K candidates with scores within 1e-5.
"""

import sys
from pathlib import Path
from types import SimpleNamespace

import pytest
import torch

pytestmark = pytest.mark.gpu

REF = Path(__file__).resolve().parent.parent / "baseline" / "_ref"


@pytest.fixture(scope="module")
def ref():
    if not (REF / "whisper_trt" / "attn_plugin.py").is_file():
        pytest.skip("the reference package is not staged under baseline/_ref")
    pytest.importorskip("triton")
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    from whisper_trt import attn_plugin, beam_kernels

    return SimpleNamespace(ap=attn_plugin, bk=beam_kernels)


def _g(seed):
    return torch.Generator(device="cuda").manual_seed(seed)


@pytest.mark.parametrize("n,c,lo,hi", [(10, 64, 0, 63), (40, 228, 80, 80), (160, 228, 4, 224)])
def test_self_step_matches_reference(ref, n, c, lo, hi):
    from whisper_trt_b200 import attn_plugin as ap

    g = _g(n)
    H, D, K = 20, 64, 5
    kc = torch.randn(n, H, c, D, generator=g, device="cuda").half()
    vc = torch.randn(n, H, c, D, generator=g, device="cuda").half()
    qkv = torch.randn(n, 1, 3 * H * D, generator=g, device="cuda").half()
    off = torch.randint(lo, hi + 1, (n // K,), generator=g, device="cuda").repeat_interleave(K)
    src = ((torch.arange(n, device="cuda") // K * K)[:, None]
           + torch.randint(0, K, (n, c), generator=g, device="cuda")).to(torch.int32)
    kc2, vc2 = kc.clone(), vc.clone()
    want = ref.ap.self_attn_step_triton(qkv, kc, vc, off, src, write_cache=True)
    got = ap.self_attn_step_triton(qkv, kc2, vc2, off, src, write_cache=True)
    torch.cuda.synchronize()
    assert (got.float() - want.float()).abs().max().item() <= 2e-3
    assert torch.equal(kc2, kc) and torch.equal(vc2, vc)  # the same appended keys / values, bit for bit


@pytest.mark.parametrize("w,s", [(2, 5), (8, 5), (3, 17)])
def test_cross_matches_reference(ref, w, s):
    from whisper_trt_b200 import attn_plugin as ap

    g = _g(w * 100 + s)
    H, T, D = 20, 1500, 64
    q = torch.randn(w, s, H * D, generator=g, device="cuda").half()
    k = torch.randn(w, H, T, D, generator=g, device="cuda").half()
    v = torch.randn(w, H, T, D, generator=g, device="cuda").half()
    want = ref.ap.cross_attn_combine_triton(ref.ap.cross_attn_split_triton(q, k, v), q)
    want_unsplit = ref.ap.cross_attn_triton(q, k, v)
    got = ap.cross_attn_triton(q, k, v)
    part = ap.cross_attn_split_triton(q, k, v)
    got_split = ap.cross_attn_combine_triton(part, q)
    torch.cuda.synchronize()
    for y in (got, got_split):
        assert (y.float() - want.float()).abs().max().item() <= 2e-3
        assert (y.float() - want_unsplit.float()).abs().max().item() <= 2e-3


def test_prompt_matches_reference(ref):
    from whisper_trt_b200 import attn_plugin as ap

    g = _g(7)
    n, S, C, H, D = 10, 17, 64, 20, 64
    qkv = torch.randn(n, S, 3 * H * D, generator=g, device="cuda").half()
    kc = torch.randn(n, H, C, D, generator=g, device="cuda").half()
    vc = torch.randn(n, H, C, D, generator=g, device="cuda").half()
    off = torch.tensor([0, 3, 16, 17, 40, 0, 5, 33, 47, 2], device="cuda")
    src = ((torch.arange(n, device="cuda") // 5 * 5)[:, None]
           + torch.randint(0, 5, (n, C), generator=g, device="cuda")).to(torch.int32)
    want = ref.ap.self_attn_triton(qkv, kc, vc, off, src)
    got = ap.self_attn_triton(qkv, kc, vc, off, src)
    torch.cuda.synchronize()
    assert (got.float() - want.float()).abs().max().item() <= 2e-3


@pytest.mark.parametrize("rows,vocab", [(5, 1024), (160, 51866)])
def test_logits32_matches_reference(ref, rows, vocab):
    from whisper_trt_b200 import attn_plugin as ap

    g = _g(rows)
    x = torch.randn(rows, 1, 1280, generator=g, device="cuda").half()
    w = (torch.randn(vocab, 1280, generator=g, device="cuda") * 0.02).half()
    want = ref.ap.logits32_triton(x, w)
    got = ap.logits32_triton(x, w)
    torch.cuda.synchronize()
    assert (got - want).abs().max().item() <= 1e-4 * max(1.0, want.abs().max().item())


@pytest.mark.parametrize("windows", [1, 32])
def test_beam_scores_match_reference(ref, windows):
    from whisper_trt_b200 import slots

    g = _g(windows)
    K, V = 5, 51866
    cfg = SimpleNamespace(no_speech=50362, no_timestamps=50363, timestamp_begin=50365, eot=50257, vocab_size=V)
    s = SimpleNamespace(K=K, B=windows, cfg=cfg, timestamps=False, mixed=False,
                        suppress=torch.zeros(V, dtype=torch.bool, device="cuda"),
                        begin=torch.zeros(V, dtype=torch.bool, device="cuda"),
                        t=torch.full((windows,), 5, dtype=torch.int64, device="cuda"),
                        cum=torch.randn(windows * K, generator=g, device="cuda"),
                        hist=torch.zeros(windows * K, 224, dtype=torch.int64, device="cuda"),
                        max_initial=torch.tensor([50], device="cuda"),
                        sampling=torch.zeros(windows, dtype=torch.bool, device="cuda"))
    s.suppress[torch.randint(0, V, (300,), generator=g, device="cuda")] = True
    logits = torch.randn(windows * K, V, generator=g, device="cuda") * 3
    scores = torch.empty(windows * K, V, device="cuda")
    ns_r = torch.empty(windows, device="cuda")
    ns_o = torch.empty(windows, device="cuda")
    ref.bk.scores(s, logits, scores, ns_r)
    want_s, want_i = scores.view(windows, -1).topk(2 * K, dim=1)
    got_s, got_i = slots.best(s, logits, ns_o)
    torch.cuda.synchronize()
    assert torch.equal(got_i, want_i)
    assert (got_s - want_s).abs().max().item() <= 1e-5
    assert (ns_o - ns_r).abs().max().item() <= 1e-6
