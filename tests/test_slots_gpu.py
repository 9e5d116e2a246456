"""GPU parity, bit-exact: slot-table bookkeeping, cache append and gather kernels against the oracle."""

import types

import numpy as np
import pytest
import torch

import cases
from oracle import attn as oa
from oracle import slots as osl
from whisper_trt_b200 import attn_plugin as ap
from whisper_trt_b200 import slots

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]

FIELDS = ("t", "pos", "sot_pos", "no_speech", "done", "hist", "cum", "src", "tokens", "forced", "h_count", "h_score",
          "h_len", "h_tokens", "last_t")


def _steps(golden):
    return sorted({k.split("/")[0] for k in golden.files})


def test_beam_update_matches_oracle_on_reference_steps(slots_golden):
    """Every recorded step of three reference decodes (beam 3 and 5, refills, prefilled prompts): the kernel's
    state after the step equals the oracle's, field by field, bit for bit (done windows included)."""
    for key in _steps(slots_golden):
        K, P, V, EOT, _ = slots_golden[f"{key}/meta"].tolist()
        before = {f: slots_golden[f"{key}/before/{f}"] for f in FIELDS}
        st = {f: before[f].copy() for f in FIELDS}
        st["tokens"] = st["tokens"][:, 0].copy()
        st.update(K=K, P=P)
        top_s, top_i, ns = (slots_golden[f"{key}/{n}"] for n in ("top_s", "top_i", "ns"))
        osl.beam_update(st, top_s, top_i, ns, V, EOT)
        s = types.SimpleNamespace(K=K, P=P, cfg=types.SimpleNamespace(vocab_size=V, eot=EOT))
        for f in FIELDS:
            setattr(s, f, torch.from_numpy(np.ascontiguousarray(before[f])).cuda())
        s.tokens = s.tokens[:, 0].contiguous()
        slots.update(s, torch.from_numpy(top_s).cuda(), torch.from_numpy(top_i).cuda(), torch.from_numpy(ns).cuda())
        for f in FIELDS:
            got = getattr(s, f).cpu().numpy()
            assert np.array_equal(got, st[f]), (key, f)


@pytest.mark.parametrize("K,C,T", [(5, 228, 224), (3, 40, 20), (1, 17, 9), (32, 64, 16)])
def test_beam_reorder_matches_oracle(K, C, T):
    rng = np.random.default_rng(K * 1000 + C)
    B = 7
    n = B * K
    src = rng.integers(0, n, (n, C)).astype(np.int32)
    hist = rng.integers(0, 50000, (n, T)).astype(np.int64)
    parent = np.stack([rng.permutation(K) if b % 2 else rng.integers(0, K, K) for b in range(B)]).astype(np.int64)
    pos = rng.integers(0, C + 2, B).astype(np.int64)  # C and C+1: no mark (out of the table)
    t = rng.integers(-1, T, B).astype(np.int64)
    token = rng.integers(0, 50000, n).astype(np.int64)
    live = rng.random(B) < 0.7
    exp = [a.copy() for a in (src, hist, pos)]
    osl.beam_reorder(exp[0], parent, exp[2], hist=exp[1], token=token, t=t, live=live)
    g = [torch.from_numpy(a.copy()).cuda() for a in (src, hist, pos)]
    offset = torch.zeros(n, dtype=torch.long, device="cuda")
    slots.beam_reorder(g[0], torch.from_numpy(parent).cuda(), g[2], hist=g[1], token=torch.from_numpy(token).cuda(),
                       t=torch.from_numpy(t).cuda(), live=torch.from_numpy(live).cuda(), offset=offset)
    for a, b in zip(g, exp):
        assert np.array_equal(a.cpu().numpy(), b)
    assert np.array_equal(offset.cpu().numpy(), np.repeat(exp[2], K))


def test_slot_reset():
    src = torch.full((12, 10), 7, dtype=torch.int32, device="cuda")
    slots.slot_reset(src, torch.tensor([0, 3], device="cuda"), 3, prefilled=False)
    slots.slot_reset(src, torch.tensor([2], device="cuda"), 3, prefilled=True)
    exp = np.full((12, 10), 7, dtype=np.int32)
    osl.slot_reset(exp, np.array([0, 3]), 3, prefilled=False)
    osl.slot_reset(exp, np.array([2]), 3, prefilled=True)
    assert np.array_equal(src.cpu().numpy(), exp)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_gather_cache_bit_exact(dtype):
    qkv, kc, vc, off, src = cases.plugin_case(b=10, s=1, h=20, c=96, dtype=dtype)
    src[0, :5] = torch.tensor([-3, 10, 11, 99, 9], dtype=torch.int32)  # clamped to [0, N-1]
    out = ap.gather_cache(kc.cuda(), src.cuda()).cpu()
    exp = oa.gather_cache(kc.view(torch.int16).numpy(), np.clip(src.numpy(), 0, 9))
    assert np.array_equal(out.view(torch.int16).numpy(), exp)


def test_cache_append_bit_exact():
    qkv, kc, vc, off, src = cases.plugin_case(b=10, s=1, h=20, c=96, dtype=torch.float16)
    off[:3] = torch.tensor([-1, 96, 95])
    k2, v2 = kc.cuda(), vc.cuda()
    ap.cache_append(qkv.cuda(), k2, v2, off.cuda())
    ke, ve = kc.numpy().copy(), vc.numpy().copy()
    oa.cache_append(ke, ve, qkv.numpy(), off.numpy())
    assert np.array_equal(k2.cpu().numpy().view(np.int16), ke.view(np.int16))
    assert np.array_equal(v2.cpu().numpy().view(np.int16), ve.view(np.int16))
