"""The torch custom ops' fake kernels (what tracing and graph capture see without running a kernel), checked on meta
tensors without a GPU: the same output shapes and dtypes as the reference's ops' fake kernels
(attn_plugin.py:124-126 self_attn, :139-141 cross_attn, :177-179 cross_attn_split, :197-199 cross_attn_combine,
:210-212 logits32)."""

import pytest
import torch

from whisper_trt_b200 import attn_plugin  # noqa: F401  (registers the ops)

OPS = torch.ops.whisper_trt_b200
M = {"device": "meta"}


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("s", [1, 17])
def test_self_attn_fake(dtype, s):
    n, h, c, d = 10, 20, 64, 64
    qkv = torch.empty(n, s, 3 * h * d, dtype=dtype, **M)
    kc = torch.empty(n, h, c, d, dtype=dtype, **M)
    off = torch.empty(n, dtype=torch.long, **M)
    src = torch.empty(n, c, dtype=torch.int32, **M)
    y = OPS.self_attn(qkv, kc, kc, off, src)
    assert y.shape == (n, s, h * d) and y.dtype == dtype
    if s == 1:
        for op in (OPS.self_attn_step, OPS.self_attn_step_append):
            y = op(qkv, kc, kc, off, src)
            assert y.shape == (n, 1, h * d) and y.dtype == dtype


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_cross_attn_fakes(dtype):
    w, s, h, t, d = 3, 5, 20, 1500, 64
    q = torch.empty(w, s, h * d, dtype=dtype, **M)
    k = torch.empty(w, h, t, d, dtype=dtype, **M)
    y = OPS.cross_attn(q, k, k)
    assert y.shape == q.shape and y.dtype == dtype
    part = OPS.cross_attn_split(q, k, k)
    assert part.shape == (w, h, attn_plugin.SPLITS, s, d + 2) and part.dtype == torch.float32
    y = OPS.cross_attn_combine(part, q)
    assert y.shape == q.shape and y.dtype == dtype


def test_logits32_fake():
    x = torch.empty(4, 1, 1280, dtype=torch.float16, **M)
    w = torch.empty(51866, 1280, dtype=torch.float16, **M)
    y = OPS.logits32(x, w)
    assert y.shape == (4, 1, 51866) and y.dtype == torch.float32
