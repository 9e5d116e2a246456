"""GPU parity: the vocabulary projection on the tcgen05 tensor cores (C ABI ``wt_logits32``) against an fp32
reference of the reference op's body (attn_plugin.py:202-212: ``x.float() @ w.float().t()``).

Tolerance: the products of fp16 / bf16 inputs are exact in fp32, so the kernel and the reference differ only in the
order of the fp32 sums: |err| <= 1e-4 * (1 + |y|) at d 1280 with whisper-like magnitudes."""

import pytest
import torch

from whisper_trt_b200 import attn_plugin as ap

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]


def _case(rows, vocab, d, dtype=torch.float16, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(rows, 1, d, generator=g, device="cuda").to(dtype)
    w = (torch.randn(vocab, d, generator=g, device="cuda") * 0.02).to(dtype)
    return x, w


def _check(x, w, y):
    ref = (x.double() @ w.double().t()).float()
    err = (y - ref).abs()
    bound = 1e-4 * (1 + ref.abs())
    assert torch.isfinite(y).all()
    assert (err <= bound).all(), f"max err {err.max().item():.3e}"


@pytest.mark.parametrize("rows,vocab,d", [(160, 51866, 1280), (40, 51866, 1280), (1, 1000, 1280), (5, 129, 1280),
                                          (16, 128, 64), (17, 300, 384), (300, 2000, 512), (256, 640, 1280),
                                          (320, 51866, 1280), (600, 2000, 256), (160, 51865, 1280),
                                          (7, 301, 256)])
def test_shapes(rows, vocab, d):
    x, w = _case(rows, vocab, d)
    y = ap.logits32_triton(x, w)
    assert y.shape == (rows, 1, vocab) and y.dtype == torch.float32
    _check(x, w, y)
    assert ap.workspace_errors() == 0


def test_bf16_and_prompt_shape():
    x, w = _case(24, 5000, 1280, torch.bfloat16, seed=3)
    _check(x, w, ap.logits32_triton(x.view(4, 6, 1280), w).view(24, 1, 5000))


def test_custom_op_graph_and_out():
    x, w = _case(40, 4096, 1280, seed=5)
    out = torch.empty(40, 1, 4096, device="cuda")
    ap.logits32_triton(x, w, out=out)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        ap.logits32_triton(x, w, out=out)
    out.zero_()
    g.replay()
    torch.cuda.synchronize()
    _check(x, w, out)
    _check(x, w, torch.ops.whisper_trt_b200.logits32(x, w))


def test_repeated_launches_identical():
    """20 launches at the config-3 shape give the same bits and stay within the tolerance: the TMA ring and the
    tensor-memory accumulators are reused across items and launches, so a stage refilled or an accumulator drained
    early would show up as a launch that differs."""
    x, w = _case(160, 51866, 1280, seed=11)
    outs = [ap.logits32_triton(x, w) for _ in range(20)]
    _check(x, w, outs[0])
    assert all(torch.equal(o, outs[0]) for o in outs)
