"""The oracle pinned against the reference's own outputs (tests/golden, made by make_golden.py from the reference
source). CPU only: these decide whether the oracle may be trusted as the checker of the CUDA kernels."""

import numpy as np
import pytest

import cases
from oracle import attn as oa
from oracle import slots as osl

ATOL = 1e-5  # the reference's own CPU tolerance (test_attn_plugin.py:34, :92)


def _np(t):
    return t.float().numpy() if t.is_floating_point() else t.numpy()


@pytest.mark.parametrize("name", list(cases.ATTN_CASES))
def test_inputs_regenerate(name, attn_golden):
    kind, kw = cases.ATTN_CASES[name]
    inp = cases.make_attn_inputs(kind, kw)
    assert cases.inputs_digest(inp) == str(attn_golden[f"{name}/digest"]), "seeded inputs drifted"


@pytest.mark.parametrize("name", list(cases.ATTN_CASES))
def test_oracle_matches_reference(name, attn_golden):
    kind, kw = cases.ATTN_CASES[name]
    inp = cases.make_attn_inputs(kind, kw)
    checked = 0
    if "qkv" in inp:
        qkv, kc, vc = (_np(inp[k]) for k in ("qkv", "kc", "vc"))
        off, src = inp["offset"].numpy(), inp["src"].numpy()
        y = oa.self_attn(qkv, kc, vc, off, src)
        np.testing.assert_allclose(y, attn_golden[f"{name}/self"], atol=ATOL, rtol=0)
        checked += 1
        if f"{name}/self_off40" in attn_golden:
            y = oa.self_attn(qkv, kc, vc, np.full_like(off, 40), src)
            np.testing.assert_allclose(y, attn_golden[f"{name}/self_off40"], atol=ATOL, rtol=0)
        if qkv.shape[1] == 1:  # the step semantics (clamps, no write) equal the op on in-range inputs
            y = oa.self_attn_step(qkv, kc.copy(), vc.copy(), off, src)
            np.testing.assert_allclose(y, attn_golden[f"{name}/self"], atol=ATOL, rtol=0)
    if "q" in inp:
        q, k, v = _np(inp["q"]), _np(inp["xk"]), _np(inp["xv"])
        np.testing.assert_allclose(oa.cross_attn(q, k, v), attn_golden[f"{name}/cross"], atol=ATOL, rtol=0)
        checked += 1
        if f"{name}/part" in attn_golden:
            part = oa.cross_attn_split(q, k, v)
            ref = attn_golden[f"{name}/part"]
            np.testing.assert_allclose(part[..., -2], ref[..., -2], atol=ATOL, rtol=0)  # slice maxima
            np.testing.assert_allclose(part, ref, atol=1e-4, rtol=1e-5)  # sums of up to 188 terms
            np.testing.assert_allclose(oa.cross_attn_combine(ref), attn_golden[f"{name}/combined"], atol=ATOL,
                                       rtol=0)
            np.testing.assert_allclose(oa.cross_attn_combine(part), attn_golden[f"{name}/cross"], atol=ATOL,
                                       rtol=0)
    assert checked


def test_gather_cache_matches_explicit_rows():
    """attn_plugin.py:92-99 against a per-slot loop (test_attn_plugin.py:26-29)."""
    qkv, kc, vc, offset, src = cases.plugin_case(b=6, s=1, h=4, c=32)
    kc, src = kc.numpy(), src.numpy()
    g = oa.gather_cache(kc, src)
    for r in range(6):
        for j in range(32):
            assert np.array_equal(g[r, :, j], kc[src[r, j], :, j])


def test_cache_append_only_touches_own_slot():
    qkv, kc, vc, offset, src = cases.plugin_case(b=6, s=1, h=4, c=32, dtype=__import__("torch").float16)
    qkv, kc, vc = qkv.numpy(), kc.numpy(), vc.numpy()
    k2, v2 = kc.copy(), vc.copy()
    off = np.array([0, 5, 31, 32, 40, -3])  # 32 and 40 are >= C: no write (the kernel's ``off < C`` mask)
    oa.cache_append(k2, v2, qkv, np.clip(off, 0, 32))
    hd = 4 * 64
    for r in range(6):
        o = int(np.clip(off[r], 0, 32))
        ke, ve = kc[r].copy(), vc[r].copy()
        if o < 32:
            ke[:, o] = qkv[r, 0, hd:2 * hd].reshape(4, 64)
            ve[:, o] = qkv[r, 0, 2 * hd:].reshape(4, 64)
        assert np.array_equal(k2[r].view(np.int16), ke.view(np.int16))
        assert np.array_equal(v2[r].view(np.int16), ve.view(np.int16))


# --- bookkeeping ---------------------------------------------------------------------------------------------
def _steps(golden):
    return sorted({k.split("/")[0] for k in golden.files})


def _state(golden, key, which):
    return {f: golden[f"{key}/{which}/{f}"].copy() for f in
            ("t", "pos", "sot_pos", "no_speech", "done", "hist", "cum", "src", "tokens", "forced", "h_count",
             "h_score", "h_len", "h_tokens", "last_t")}


def test_beam_update_matches_reference_bookkeeping(slots_golden):
    """beam_kernels._update_kernel's restatement against the reference's PyTorch bookkeeping (search.py:242-265,
    :283-313, :367-409), step by step over three streamed decodes with refills. The two reference paths differ
    only on windows already done (PyTorch reorders them anyway; the fused kernel leaves them) and on the unused
    hypothesis slot 2K, which are excluded; done windows must come out untouched."""
    n_live = 0
    for key in _steps(slots_golden):
        K, P, V, EOT, _ = slots_golden[f"{key}/meta"].tolist()
        st = _state(slots_golden, key, "before")
        before = _state(slots_golden, key, "before")
        ref = _state(slots_golden, key, "after")
        st.update(K=K, P=P)
        st["tokens"] = st["tokens"][:, 0].copy()
        osl.beam_update(st, slots_golden[f"{key}/top_s"], slots_golden[f"{key}/top_i"], slots_golden[f"{key}/ns"],
                        V, EOT)
        live = ~before["done"]
        rows = np.repeat(live, K)
        n_live += int(live.sum())
        for f in ("t", "pos", "done", "h_count"):
            assert np.array_equal(st[f][live], ref[f][live]), (key, f)
            assert np.array_equal(st[f][~live], before[f][~live]), (key, f)
        assert np.array_equal(st["no_speech"], ref["no_speech"]), key
        for f in ("hist", "src"):
            assert np.array_equal(st[f][rows], ref[f][rows]), (key, f)
            assert np.array_equal(st[f][~rows], before[f][~rows]), (key, f)
        assert np.array_equal(st["cum"][rows], ref["cum"][rows]), key
        assert np.array_equal(st["tokens"][rows], ref["tokens"][rows, 0]), key
        S = st["h_score"].shape[1]
        keep = np.arange(S) < 2 * K  # slot 2K: where the PyTorch path parks unregistered candidates
        for f in ("h_score", "h_len", "h_tokens"):
            assert np.array_equal(st[f][live][:, keep], ref[f][live][:, keep]), (key, f)
    assert n_live > 100


def test_beam_reorder_is_the_update_given_parents(slots_golden):
    """The parents-given reorder (the slot-table part alone) reproduces the reference's src/hist on every step
    where no candidate ended (then the new beams' parents are just top_i[:, :K] // V)."""
    checked = 0
    for key in _steps(slots_golden):
        K, P, V, EOT, _ = slots_golden[f"{key}/meta"].tolist()
        before = _state(slots_golden, key, "before")
        ref = _state(slots_golden, key, "after")
        top_i = slots_golden[f"{key}/top_i"]
        tok = top_i[:, :K] % V
        live = ~before["done"] & (before["t"] >= 0) & ~(tok == EOT).any(1) & (before["t"] != before["last_t"])
        if not live.any():
            continue
        src, hist, pos = before["src"].copy(), before["hist"].copy(), before["pos"].copy()
        osl.beam_reorder(src, top_i[:, :K] // V, pos, hist=hist, token=tok.reshape(-1), t=before["t"], live=live)
        rows = np.repeat(live, K)
        assert np.array_equal(src[rows], ref["src"][rows]), key
        assert np.array_equal(hist[rows], ref["hist"][rows]), key
        assert np.array_equal(pos[live], ref["pos"][live]), key
        checked += 1
    assert checked > 20


def test_slot_reset():
    src = np.full((9, 6), 7, dtype=np.int32)
    osl.slot_reset(src, np.array([0, 2]), 3, prefilled=False)
    assert (src[0:3] == np.arange(3)[:, None]).all() and (src[6:9] == np.arange(6, 9)[:, None]).all()
    assert (src[3:6] == 7).all()
    osl.slot_reset(src, np.array([1]), 3, prefilled=True)
    assert (src[3:6] == 3).all()


def _score_steps(z):
    return sorted({k.split("/")[0] for k in z.files})


def score_inputs(z, key):
    K, V, ts, mi, ns_id, nots, tsb, eot, _ = z[f"{key}/meta"].tolist()
    return dict(logits=z[f"{key}/logits"], suppress=z[f"{key}/suppress"], begin=z[f"{key}/begin"], t=z[f"{key}/t"],
                cum=z[f"{key}/cum"], hist=z[f"{key}/hist"], max_initial=mi, K=K, timestamps=bool(ts),
                no_speech=ns_id, no_timestamps=nots, ts_begin=tsb, eot=eot)


def test_beam_scores_match_reference(scores_golden):
    """The candidate scores (masks, timestamp rules, log-softmax + cum) and no-speech probabilities of 191 beam
    steps of the reference Search (with and without timestamps) from the oracle restatement: finite scores within
    1e-5, the same masked entries, the same best 2K (none of them tied: the fixture's decodes keep 2K allowed
    tokens at every step)."""
    text_masked = 0
    for key in _score_steps(scores_golden):
        inp = score_inputs(scores_golden, key)
        sc, ns = osl.beam_scores(**inp)
        ref = scores_golden[f"{key}/scores"]
        fin = ref > -1e30
        assert np.array_equal(sc > -1e30, fin), key
        assert np.abs(sc[fin] - ref[fin]).max() < 1e-5, key
        assert np.abs(ns - scores_golden[f"{key}/ns"]).max() < 1e-6, key
        top_s, top_i = osl.beam_topk(sc, inp["K"])
        assert np.array_equal(top_i, scores_golden[f"{key}/top_i"]), key
        assert np.allclose(top_s, scores_golden[f"{key}/top_s"], atol=1e-5, rtol=0), key
        if inp["timestamps"]:
            tsb = inp["ts_begin"]
            text_masked += int(((ref[:, :tsb] < -1e30).all(1) & fin[:, tsb:].any(1)).sum())
    assert text_masked > 50  # the timestamp probability check fired (text masked in favour of timestamps)
