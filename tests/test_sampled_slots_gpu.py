"""Beam search with sampled slots (the reference's ``Search(sampling_slots=True)``) on this package's kernels.

Fixtures (``tests/golden/mixed_golden.npz``, written by ``make_golden.py --only mixed``) record 131 steps of the
reference's own Search decoding a stream of windows at temperatures 0 (beam search, beam 3 and 4), 0.5 and 1.0
(sampled, some windows on fewer rows than their slot), with its PyTorch bookkeeping on CPU (search.py:290-312
_choose, :342-354 _greedy, :367-409 _beam, :104-129 uniform). Each step's recorded state and logits go through the
fused step the reference's Search._body runs on the GPU (search.py:251-256): :func:`slots.scores` (the rows of
sampled windows without their cumulative score), the best 2K (torch.topk), :func:`slots.sample` (Gumbel-max with the
counter-based random numbers) and :func:`slots.update` (beam rules for beam windows, GreedySearch rules for sampled
ones). For every window still decoding, compared with the recorded state after the step: tokens of rows still
decoding, slot tables, histories, positions, steps, done flags, hypotheses (their first 2K slots; the PyTorch path
also writes a scratch slot 2K) and sampled rows' done flags and lengths bit for bit; cumulative scores, hypothesis
scores and no-speech probabilities within 1e-5 relative (log-softmax on the GPU against the CPU's). A window already
done is left exactly as it was, as the reference's fused bookkeeping leaves it (beam_kernels.py:15; its PyTorch path
goes on rewriting a done window's histories and tokens, which nothing reads before the slot is loaded again).
"""

from types import SimpleNamespace

import numpy as np
import pytest
import torch

from whisper_trt_b200 import slots

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]

FIELDS = ("t", "pos", "sot_pos", "no_speech", "done", "hist", "cum", "src", "tokens", "forced", "h_count",
          "h_score", "h_len", "h_tokens", "last_t", "row_done", "length", "sampling", "temperature", "seed",
          "suppress", "begin", "max_initial")


def _state(d, key):
    s = SimpleNamespace()
    for f in FIELDS:
        setattr(s, f, torch.from_numpy(d[f"{key}/before/{f}"].copy()).cuda())
    K, P, V, eot, no_speech, _ = (int(x) for x in d[f"{key}/meta"])
    B = s.pos.shape[0]
    s.K, s.P, s.B, s.mixed, s.timestamps = K, P, B, True, False
    s.cfg = SimpleNamespace(vocab_size=V, eot=eot, no_speech=no_speech, no_timestamps=None, timestamp_begin=None)
    s.scores = torch.empty(B * K, V, device="cuda")
    s.samp_tok = torch.zeros(B * K, dtype=torch.int64, device="cuda")
    s.samp_score = torch.zeros(B * K, device="cuda")
    s.ns = torch.empty(B, device="cuda")
    return s


def _close(a, b, rel=1e-5):
    fin = np.isfinite(b)
    return np.array_equal(fin, np.isfinite(a)) and bool(np.all(np.abs(a[fin] - b[fin]) <= rel * (1 + np.abs(b[fin]))))


def test_mixed_steps_match_reference(mixed_golden):
    d = mixed_golden
    steps = sorted({k.split("/")[0] for k in d.files})
    assert len(steps) >= 100
    sampled_steps = 0
    for key in steps:
        s = _state(d, key)
        B, K = s.B, s.K
        logits = torch.from_numpy(d[f"{key}/logits"]).cuda()
        slots.scores(s, logits, s.scores, s.ns)
        top_s, top_i = s.scores.view(B, -1).topk(2 * K, dim=1)
        slots.sample(s)
        slots.update(s, top_s.contiguous(), top_i.contiguous(), s.ns)
        torch.cuda.synchronize()
        got = {f: getattr(s, f).cpu().numpy() for f in FIELDS}
        want = {f: d[f"{key}/after/{f}"] for f in FIELDS}
        before = {f: d[f"{key}/before/{f}"] for f in FIELDS}
        samp, wdone = before["sampling"], before["done"]
        on = ~wdone  # windows still decoding
        rows_on = np.repeat(on, K)
        rows_samp = np.repeat(samp & on, K)
        live_before = rows_on & (~before["row_done"] | ~np.repeat(samp, K))  # (a done sampled row's token is unused)
        sampled_steps += int((samp & (before["t"] >= 0) & on).sum())
        for f in ("t", "pos", "done", "h_count"):
            assert np.array_equal(got[f][on], want[f][on]), (key, f)
        for f in ("hist", "src"):
            assert np.array_equal(got[f][rows_on], want[f][rows_on]), (key, f)
        assert np.array_equal(got["tokens"][live_before], want["tokens"][live_before]), key
        S2 = 2 * K
        for f in ("h_len", "h_tokens"):
            assert np.array_equal(got[f][on, :S2], want[f][on, :S2]), (key, f)
        for f in ("row_done", "length"):
            assert np.array_equal(got[f][rows_samp], want[f][rows_samp]), (key, f)
        assert _close(got["cum"][rows_on], want["cum"][rows_on]), key
        assert _close(got["h_score"][on, :S2], want["h_score"][on, :S2]), key
        assert _close(got["no_speech"], want["no_speech"]), key
        for f in FIELDS:  # a done window is left as it was
            if f in ("t", "pos", "done", "h_count", "h_score", "h_len", "h_tokens", "sot_pos", "forced", "last_t",
                     "sampling", "temperature", "seed"):
                idx = wdone
            elif f in ("suppress", "begin", "max_initial", "no_speech"):  # (no_speech: compared above, all windows)
                continue
            else:
                idx = np.repeat(wdone, K)
            assert np.array_equal(got[f][idx], before[f][idx]), (key, f, "done window changed")
    assert sampled_steps >= 100


def test_counter_uniform_matches_reference_hash():
    """The sampling kernel's random numbers are search.uniform's (search.py:104-129): a window whose scores are all
    equal takes the token with the largest uniform number -- checked against a numpy restatement of the hash."""
    V, K = 1000, 2
    seed, t = 12345, 7
    s = SimpleNamespace(K=K, B=1, pos=torch.zeros(1, dtype=torch.int64, device="cuda"))
    s.scores = torch.zeros(K, V, device="cuda")
    s.t = torch.tensor([t], device="cuda")
    s.done = torch.zeros(1, dtype=torch.bool, device="cuda")
    s.row_done = torch.zeros(K, dtype=torch.bool, device="cuda")
    s.sampling = torch.ones(1, dtype=torch.bool, device="cuda")
    s.temperature = torch.ones(1, device="cuda")
    s.seed = torch.tensor([seed], device="cuda")
    s.samp_tok = torch.zeros(K, dtype=torch.int64, device="cuda")
    s.samp_score = torch.zeros(K, device="cuda")
    slots.sample(s)
    m = 0xFFFFFFFF
    for r in range(K):
        x = (r * V + np.arange(V, dtype=np.int64) + (seed * 0x6C8E9CF5 + t * 0x85EBCA77)) & m
        for _ in range(2):
            x = (x * 747796405 + 2891336453) & m
            x = (((x >> ((x >> 28) + 4)) ^ x) * 277803737) & m
            x = ((x >> 22) ^ x) & m
        u = (x.astype(np.float32) + np.float32(0.5)) / np.float32(4294967296.0)
        # Gumbel-max of equal scores: the largest -log(-log u), i.e. the largest u (first on ties)
        assert int(s.samp_tok[r]) == int(np.argmax(u)), r
