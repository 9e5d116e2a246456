"""GPU parity: the scoring half of a beam step (C ABI ``wt_beam_scores``) against the reference.

* the 191 recorded beam steps of the reference Search (tests/golden/scores_golden.npz: two decodes without and two
  with CTranslate2's timestamp rules): the candidate scores within 1e-5 of the reference's (the same masked
  entries), the no-speech probabilities within 1e-6, the best 2K identical;
* whisper-large-v3-sized rows (V 51866, 32 windows x beam 5) against the oracle restatement, with and without
  timestamps; equal scores come out in index order.
"""

from types import SimpleNamespace

import numpy as np
import pytest
import torch

from oracle import slots as osl
from whisper_trt_b200 import slots

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]


def _state(K, suppress, begin, t, cum, hist, max_initial, no_speech, nots, tsb, eot, vocab, timestamps):
    dev = "cuda"
    cfg = SimpleNamespace(no_speech=no_speech, no_timestamps=nots, timestamp_begin=tsb, eot=eot, vocab_size=vocab)
    return SimpleNamespace(K=K, cfg=cfg, timestamps=timestamps,
                           suppress=torch.as_tensor(suppress, dtype=torch.bool, device=dev),
                           begin=torch.as_tensor(begin, dtype=torch.bool, device=dev),
                           t=torch.as_tensor(t, dtype=torch.int64, device=dev),
                           cum=torch.as_tensor(cum, dtype=torch.float32, device=dev),
                           hist=torch.as_tensor(hist, dtype=torch.int64, device=dev).contiguous(),
                           max_initial=torch.tensor([max_initial], dtype=torch.int64, device=dev))


def test_reference_steps(scores_golden):
    z = scores_golden
    steps = sorted({k.split("/")[0] for k in z.files})
    worst = 0.0
    for key in steps:
        K, V, ts, mi, ns_id, nots, tsb, eot, _ = z[f"{key}/meta"].tolist()
        s = _state(K, z[f"{key}/suppress"], z[f"{key}/begin"], z[f"{key}/t"], z[f"{key}/cum"], z[f"{key}/hist"], mi,
                   ns_id, nots, tsb, eot, V, bool(ts))
        logits = torch.as_tensor(z[f"{key}/logits"], device="cuda").contiguous()
        B = s.t.shape[0]
        out = torch.empty_like(logits)
        ns = torch.empty(B, dtype=torch.float32, device="cuda")
        top_s, top_i = slots.best(s, logits, ns, out=out)
        ref = z[f"{key}/scores"]
        got = out.cpu().numpy()
        fin = ref > -1e30
        assert np.array_equal(got > -1e30, fin), key
        d = float(np.abs(got[fin] - ref[fin]).max())
        worst = max(worst, d)
        assert d < 1e-5, (key, d)
        assert np.abs(ns.cpu().numpy() - z[f"{key}/ns"]).max() < 1e-6, key
        assert np.array_equal(top_i.cpu().numpy(), z[f"{key}/top_i"]), key
        assert np.allclose(top_s.cpu().numpy(), z[f"{key}/top_s"], atol=1e-5, rtol=0), key
    print(f"{len(steps)} reference steps; max |score diff| {worst:.2e}")


def _whisper_case(seed, timestamps, W=32, K=5, V=51866, T=224):
    rng = np.random.default_rng(seed)
    logits = (rng.standard_normal((W * K, V)) * 3.0).astype(np.float32)
    suppress = np.zeros(V, bool)
    suppress[rng.choice(V, 90, replace=False)] = True
    begin = np.zeros(V, bool)
    begin[[220 % V, 50257 % V]] = True
    t = rng.integers(0, 40, W)
    t[:3] = [0, -2, 1]
    cum = (-rng.random(W * K) * 20).astype(np.float32)
    tsb = 50365
    hist = rng.integers(0, tsb, (W * K, T))
    if timestamps:  # some rows end on timestamps, pairs of them, or have an earlier one
        for r in range(0, W * K, 3):
            g = int(max(t[r // K], 0))
            if g >= 1:
                hist[r, g - 1] = tsb + rng.integers(0, 100)
            if g >= 2 and r % 2 == 0:
                hist[r, g - 2] = tsb + rng.integers(0, 50)
        logits[:, tsb:] += 2.0
    return dict(logits=logits, suppress=suppress, begin=begin, t=t, cum=cum, hist=hist, max_initial=50,
                no_speech=50362, nots=50363, tsb=tsb, eot=50257, K=K, V=V)


@pytest.mark.parametrize("timestamps", [False, True])
def test_whisper_sized_rows(timestamps):
    c = _whisper_case(3 + int(timestamps), timestamps)
    K, V = c["K"], c["V"]
    s = _state(K, c["suppress"], c["begin"], c["t"], c["cum"], c["hist"], c["max_initial"], c["no_speech"],
               c["nots"], c["tsb"], c["eot"], V, timestamps)
    logits = torch.as_tensor(c["logits"], device="cuda")
    B = s.t.shape[0]
    out = torch.empty_like(logits)
    ns = torch.empty(B, dtype=torch.float32, device="cuda")
    top_s, top_i = slots.best(s, logits, ns, out=out)
    ref, ref_ns = osl.beam_scores(c["logits"], c["suppress"], c["begin"], c["t"], c["cum"], c["hist"],
                                  c["max_initial"], K, timestamps, c["no_speech"], c["nots"], c["tsb"], c["eot"])
    got = out.cpu().numpy()
    fin = ref > -1e30
    assert np.array_equal(got > -1e30, fin)
    assert np.abs(got[fin] - ref[fin]).max() < 2e-5
    assert np.abs(ns.cpu().numpy() - ref_ns).max() < 1e-6
    r_s, r_i = osl.beam_topk(ref, K)
    g_s, g_i = top_s.cpu().numpy(), top_i.cpu().numpy()
    assert np.allclose(g_s, r_s, atol=2e-5, rtol=0)
    # the same candidates, except where two of them are within the scores' rounding (none expected here)
    assert (g_i == r_i).mean() > 0.999, (g_i != r_i).sum()
    # without writing the scores: the same best 2K
    ns2 = torch.empty_like(ns)
    t2_s, t2_i = slots.best(s, logits, ns2)
    assert torch.equal(t2_i, top_i) and torch.equal(t2_s, top_s) and torch.equal(ns2, ns)


def test_equal_scores_come_out_in_index_order():
    K, V, W = 4, 1000, 3
    s = _state(K, np.zeros(V, bool), np.zeros(V, bool), [5, 5, 5], np.zeros(W * K), np.zeros((W * K, 8)), 50, 3, 0,
               0, 1, V, False)
    logits = torch.zeros(W * K, V, device="cuda")
    ns = torch.empty(W, device="cuda")
    top_s, top_i = slots.best(s, logits, ns)
    assert torch.equal(top_i.cpu(), torch.arange(2 * K).repeat(W, 1))
    assert torch.allclose(top_s, torch.full_like(top_s, -float(np.log(V))))


def test_best_in_a_graph():
    """The scoring kernel captured in a CUDA graph and replayed (its workspace made before the capture)."""
    c = _whisper_case(9, False, W=4, K=5, V=2000, T=16)
    K, V = c["K"], c["V"]
    s = _state(K, c["suppress"], c["begin"], np.full(4, 3), np.zeros(20), c["hist"] % V, 50, 3, 0, 0, 1, V, False)
    s.cfg.eot, s.cfg.no_speech = 1, 3
    logits = torch.as_tensor(c["logits"], device="cuda")
    ns = torch.empty(4, device="cuda")
    ref_s, ref_i = slots.best(s, logits, ns)
    g = torch.cuda.CUDAGraph()
    out_s = torch.empty_like(ref_s)
    out_i = torch.empty_like(ref_i)
    with torch.cuda.graph(g):
        slots.best(s, logits, ns, top=(out_s, out_i))
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out_s, ref_s) and torch.equal(out_i, ref_i)
