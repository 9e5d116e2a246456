"""Seeded input generators for the parity cases (CPU, ``torch.Generator``), shared by ``make_golden.py`` (which
runs the reference on them) and the tests (which regenerate the same inputs and check their digest first).

Shapes and distributions follow the reference's own tests (``tests/test_attn_plugin.py:10-17`` ``_case``,
``:73-107``) and the benchmark configurations (config 1: 2 windows x beam 5, 20 heads x 64, 24 cached positions,
q/k/v ~ N(0,1)*0.125 from seed 0, parents uniform in [0, 5) per row, cross K/V ~ N(0,1) over 1500 frames).
"""

from __future__ import annotations

import hashlib

import numpy as np
import torch


def digest(*arrays) -> str:
    """sha256 over the raw bytes of the arrays (numpy or CPU torch), in order."""
    h = hashlib.sha256()
    for a in arrays:
        if isinstance(a, torch.Tensor):
            a = a.detach().cpu()
            a = a.view(torch.int16) if a.dtype in (torch.float16, torch.bfloat16) else a
            a = a.numpy()
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def plugin_case(b=6, s=1, h=4, c=32, d=64, dtype=torch.float32, seed=0):
    """The reference's ``_case`` (test_attn_plugin.py:10-17): qkv/kc/vc ~ N(0,1), offset in [1, c-s),
    src uniform over all rows."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    qkv = torch.randn(b, s, 3 * h * d, generator=g).to(dtype)
    kc = torch.randn(b, h, c, d, generator=g).to(dtype)
    vc = torch.randn(b, h, c, d, generator=g).to(dtype)
    offset = torch.randint(1, c - s, (b,), generator=g)
    src = torch.randint(0, b, (b, c), generator=g).to(torch.int32)
    return qkv, kc, vc, offset, src


def cross_case(w=3, s=5, h=20, t=1500, d=64, dtype=torch.float16, seed=1):
    """test_attn_plugin.py:76-79 / :98-101: q [W, S, H*D], k/v [W, H, T, D] ~ N(0,1)."""
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(w, s, h * d, generator=g).to(dtype)
    k = torch.randn(w, h, t, d, generator=g).to(dtype)
    v = torch.randn(w, h, t, d, generator=g).to(dtype)
    return q, k, v


def config1_case(dtype=torch.float32, windows=2, beams=5, heads=20, head_dim=64, cached=24, capacity=25,
                 frames=1500, seed=0):
    """Benchmark config 1 (one decoder layer): N = windows*beams rows, ``cached`` positions in every row's cache
    (offset), capacity ``capacity`` (the new token's slot = cached), q/k/v ~ N(0,1)*0.125, src[r, j] =
    (r // beams)*beams + uniform[0, beams) (duplicates allowed: each slot from a random beam of the row's window),
    cross queries ~ N(0,1)*0.125 and cross K/V ~ N(0,1) [windows, heads, frames, head_dim]."""
    g = torch.Generator().manual_seed(seed)
    n, hd = windows * beams, heads * head_dim
    qkv = (torch.randn(n, 1, 3 * hd, generator=g) * 0.125).to(dtype)
    kc = (torch.randn(n, heads, capacity, head_dim, generator=g) * 0.125).to(dtype)
    vc = (torch.randn(n, heads, capacity, head_dim, generator=g) * 0.125).to(dtype)
    offset = torch.full((n,), cached, dtype=torch.long)
    base = (torch.arange(n) // beams * beams)[:, None]
    src = (base + torch.randint(0, beams, (n, capacity), generator=g)).to(torch.int32)
    q = (torch.randn(windows, beams, hd, generator=g) * 0.125).to(dtype)
    xk = torch.randn(windows, heads, frames, head_dim, generator=g).to(dtype)
    xv = torch.randn(windows, heads, frames, head_dim, generator=g).to(dtype)
    return dict(qkv=qkv, kc=kc, vc=vc, offset=offset, src=src, q=q, xk=xk, xv=xv)


# --- the list of stored attention cases: name -> (generator, kwargs) ---------------------------------------
ATTN_CASES = {
    # test_attn_plugin.py:20-34 (reference op through the slot table, S=3, fp32)
    "self_s3_f32": ("plugin", dict(b=6, s=3, h=4, c=32, d=64, dtype=torch.float32, seed=0)),
    # test_attn_plugin.py:50-57 (step: one token, fp16 inputs, offset[0] = 0)
    "self_step_f16": ("plugin_step", dict(b=10, s=1, h=20, c=96, dtype=torch.float16, seed=0)),
    # test_attn_plugin.py:40-47 (multi-token prefill shapes, fp16 inputs)
    "self_s4_f16": ("plugin", dict(b=10, s=4, h=20, c=96, dtype=torch.float16, seed=0)),
    "self_s17_f16": ("plugin", dict(b=10, s=17, h=20, c=96, dtype=torch.float16, seed=0)),
    # test_attn_plugin.py:73-83 (cross-attention, fp16 inputs)
    "cross_s1_f16": ("cross", dict(w=3, s=1, seed=1)),
    "cross_s5_f16": ("cross", dict(w=3, s=5, seed=1)),
    "cross_s20_f16": ("cross", dict(w=3, s=20, seed=1)),
    # test_attn_plugin.py:86-92 (split + combine == full, fp32, 4 heads)
    "split_s5_f32": ("cross", dict(w=2, s=5, h=4, dtype=torch.float32, seed=2)),
    # benchmark config 1 (fp32, one layer)
    "config1_f32": ("config1", dict(dtype=torch.float32, seed=0)),
}


def make_attn_inputs(kind: str, kw: dict) -> dict:
    if kind == "plugin":
        qkv, kc, vc, offset, src = plugin_case(**kw)
        return dict(qkv=qkv, kc=kc, vc=vc, offset=offset, src=src)
    if kind == "plugin_step":
        qkv, kc, vc, offset, src = plugin_case(**kw)
        offset[0] = 0  # (only the new token), test_attn_plugin.py:54
        return dict(qkv=qkv, kc=kc, vc=vc, offset=offset, src=src)
    if kind == "cross":
        q, k, v = cross_case(**kw)
        return dict(q=q, xk=k, xv=v)
    if kind == "config1":
        return config1_case(**kw)
    raise KeyError(kind)


def inputs_digest(inp: dict) -> str:
    return digest(*[inp[k] for k in sorted(inp)])


# --- the decoder step's fused linear layers (decoder_kernels.py) -------------------------------------------------
def linear_case(m=5, n=128, k=64, seed=3):
    """Inputs of one fused linear layer: x ~ N(0,1) [m, k], LN gamma ~ 1 + N(0,1)*0.1, beta ~ N(0,1)*0.1 [k],
    w ~ N(0,1)*0.02 [n, k] (nn.Linear layout), b ~ N(0,1)*0.02 [n], residual ~ N(0,1) [m, n], a bias for
    layer_norm_bias ~ N(0,1)*0.02 [k]; all fp16."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(m, k, generator=g).half()
    gamma = (1 + 0.1 * torch.randn(k, generator=g)).half()
    beta = (0.1 * torch.randn(k, generator=g)).half()
    w = (0.02 * torch.randn(n, k, generator=g)).half()
    b = (0.02 * torch.randn(n, generator=g)).half()
    res = torch.randn(m, n, generator=g).half()
    bias = (0.02 * torch.randn(k, generator=g)).half()
    return {"x": x, "gamma": gamma, "beta": beta, "w": w, "b": b, "res": res, "bias": bias}


# name -> linear_case kwargs: rows 1 / 5 / 40 (a token, a window of beam 5, config 2's 40 rows), a multi-tile
# feature count, ragged k blocks (k = 200: 64-element blocks with a partial last one) and whisper's d = 1280
DEC_CASES = {
    "row1": dict(m=1, n=128, k=64, seed=3),
    "beam5": dict(m=5, n=384, k=200, seed=4),
    "rows40": dict(m=40, n=256, k=1280, seed=5),
    "rows17_wide": dict(m=17, n=1280, k=256, seed=6),
}
