"""Generate the golden fixtures by running the REFERENCE itself (its PyTorch op bodies and its PyTorch beam
bookkeeping, on CPU) on the seeded cases of ``cases.py``.

Run where the reference source tree is importable (it does not travel to the GPU box; the fixtures do):

    python tests/golden/make_golden.py --reference-src <path to the reference's src/ directory>

Writes ``attn_golden.npz`` (attention outputs + input digests), ``slots_golden.npz`` (per-step search states
before/after the reference's bookkeeping), ``scores_golden.npz`` (beam scoring), ``mixed_golden.npz`` (beam search
with sampled slots; ``--only mixed`` writes just this one) and ``decoder_golden.npz`` (the fused decoder linear
layers; ``--only decoder`` writes just this one) next to this script.
"""

from __future__ import annotations

import argparse
import sys
import zlib
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import cases  # noqa: E402

STATE_FIELDS = ("t", "pos", "sot_pos", "no_speech", "done", "hist", "cum", "src", "tokens", "forced", "h_count",
                "h_score", "h_len", "h_tokens", "last_t")


SPLIT_STORED = ("split_s5_f32", "config1_f32")


def attn_golden(ap) -> dict:
    out = {}
    for name, (kind, kw) in cases.ATTN_CASES.items():
        inp = cases.make_attn_inputs(kind, kw)
        out[f"{name}/digest"] = np.array(cases.inputs_digest(inp))
        if "qkv" in inp:
            f = {k: inp[k].float() for k in ("qkv", "kc", "vc")}
            y = ap.self_attn(f["qkv"], f["kc"], f["vc"], inp["offset"], inp["src"])
            out[f"{name}/self"] = y.numpy()
            if kind == "plugin_step":  # the write variant's offsets (test_attn_plugin.py:60)
                off40 = torch.full_like(inp["offset"], 40)
                out[f"{name}/self_off40"] = ap.self_attn(f["qkv"], f["kc"], f["vc"], off40, inp["src"]).numpy()
        if "q" in inp:
            q, k, v = inp["q"].float(), inp["xk"].float(), inp["xv"].float()
            out[f"{name}/cross"] = ap.cross_attn(q, k, v).numpy()
            if name in SPLIT_STORED:  # (the partials are large: stored for the small-head cases only)
                part = ap.cross_attn_split(q, k, v)
                out[f"{name}/part"] = part.numpy()
                out[f"{name}/combined"] = ap.cross_attn_combine(part, q).numpy()
    return out


# --- the beam bookkeeping: the reference Search (PyTorch bookkeeping, CPU) with a fake decoder ----------------
V, EOT, SOT, NOSPEECH = 40, 1, 2, 3


def _scores_of(history, seed):
    g = torch.Generator().manual_seed(zlib.crc32(repr((seed, history)).encode()))
    x = torch.randn(V, generator=g, dtype=torch.float64) * 2.5
    x[EOT] += 0.15 * len(history)
    return x


def _fake_step(seed):
    """test_search.py:34-48's fake decoder: cache values are token ids, read back through ``src``."""

    def step_fn(tokens, offset, cache, logits, new_kv, src):
        def run():
            for n in range(tokens.shape[0]):
                off = int(offset[n])
                hist = [int(round(float(cache[0, 0, int(src[n, j]), 0, j, 0]))) for j in range(off)]
                for s in range(tokens.shape[1]):
                    tok = int(tokens[n, s])
                    logits[n, s] = _scores_of(hist + [tok], seed).float()
                    new_kv[0, :, n, 0, s, :] = float(tok)
                    hist.append(tok)

        return run

    return step_fn


def slots_golden(ref_src: str) -> dict:
    from whisper_trt.config import WhisperConfig
    from whisper_trt.search import Search

    cfg = WhisperConfig(n_mels=4, d_model=4, enc_layers=1, enc_heads=1, enc_ffn=4, dec_layers=1, dec_heads=1,
                        dec_ffn=4, vocab_size=V, eot=EOT, sot=SOT, no_speech=NOSPEECH)
    out = {}
    step_no = 0
    for run, (K, seed, prefilled) in enumerate([(3, 0, False), (5, 1, False), (3, 2, True)]):
        W, M = 3, 7
        suppress, begin = [5, 6, 7], [8, EOT]
        if prefilled:
            prompts = [[4 + (w * 7 + j) % 30 for j in range(3 * w)] + [SOT, 10 + w, 20, 30] for w in range(M)]
            search = Search(cfg, _fake_step(seed), W, K, None, "beam", dtype=torch.float32, device="cpu",
                            max_length=40, graphs=False, fused=False)
        else:
            prompts = [[SOT, 10 + w, 20 + w % 3, 30] for w in range(M)]
            search = Search(cfg, _fake_step(seed), W, K, 4, "beam", dtype=torch.float32, device="cpu",
                            max_length=40, graphs=False, fused=False)
        rec = {}
        orig_beam, orig_body = search._beam, search._body

        def beam(logp, prompt, s=search, orig=orig_beam, rec=rec):
            scores = (logp + s.cum[:, None]).view(s.B, s.K * s.cfg.vocab_size)
            top_s, top_i = scores.topk(2 * s.K, dim=1)
            rec["top_s"], rec["top_i"] = top_s.clone(), top_i.clone()
            orig(logp, prompt)

        def body(s=search, orig=orig_body, rec=rec):
            nonlocal step_no
            before = {f: getattr(s, f).clone() for f in STATE_FIELDS}
            orig()
            after = {f: getattr(s, f).clone() for f in STATE_FIELDS}
            lg = s.logits[:: s.K, 0]
            ns = (lg[:, s.cfg.no_speech] - lg.logsumexp(-1)).exp()
            key = f"step{step_no:04d}"
            for f in STATE_FIELDS:
                out[f"{key}/before/{f}"] = before[f].numpy()
                out[f"{key}/after/{f}"] = after[f].numpy()
            out[f"{key}/top_s"] = rec["top_s"].numpy()
            out[f"{key}/top_i"] = rec["top_i"].numpy()
            out[f"{key}/ns"] = ns.numpy()
            out[f"{key}/meta"] = np.array([K, search.P, V, EOT, run], dtype=np.int64)
            step_no += 1

        search._beam = beam
        search._body = body
        if prefilled:
            def prefill(slots, ps, s=search):
                for sl, p in zip(slots, ps):
                    row = sl * s.K
                    for j, tok in enumerate(p[:-1]):
                        s.cache[0, :, row, 0, j, :] = float(tok)

            search.stream(prompts, lambda slots, windows: None, suppress, begin, check_every=1, ahead=1,
                          prefill=prefill)
        else:
            search.stream(prompts, lambda slots, windows: None, suppress, begin, check_every=1, ahead=1)
    return out


# --- beam search with sampled slots (Search(sampling_slots=True)): the reference Search, PyTorch path, CPU ---------
MIXED_V = 257  # (not a multiple of the sampling kernel's thread count)
MIXED_FIELDS = STATE_FIELDS + ("row_done", "length", "sampling", "temperature", "seed", "suppress", "begin",
                               "max_initial")


def _mixed_logits(history, seed):
    g = torch.Generator().manual_seed(zlib.crc32(repr(("mixed-golden", seed, history)).encode()))
    x = torch.randn(MIXED_V, generator=g, dtype=torch.float64) * 2.0
    x[EOT] += 0.12 * len(history)
    return x


def mixed_golden(ref_src: str) -> dict:
    """Per step of the reference's beam search with sampled slots (Search(sampling_slots=True), its PyTorch
    bookkeeping on CPU: search.py:290-312 _choose, :342-354 _greedy, :367-409 _beam, :104-129 uniform), decoding a
    stream of windows at temperatures 0 (beam), 0.5 and 1.0 (sampled, some on fewer rows than the slot has, as the
    reference's test_serve.py:62-72 makes them): the state before the step, the step's logits and the state after."""
    from whisper_trt.config import WhisperConfig
    from whisper_trt.search import Job, Search, mix_seed

    cfg = WhisperConfig(n_mels=4, d_model=4, enc_layers=1, enc_heads=1, enc_ffn=4, dec_layers=1, dec_heads=1,
                        dec_ffn=4, vocab_size=MIXED_V, eot=EOT, sot=SOT, no_speech=NOSPEECH)
    out = {}
    step_no = 0
    for run, (K, seed) in enumerate([(4, 20), (3, 21)]):
        W = 3
        jobs = []
        for w in range(7):
            temperature = (0.0, 0.5, 1.0)[w % 3]
            rows = (K if w % 2 else max(1, K - 1)) if temperature > 0 else None
            jobs.append(Job([SOT, 10 + w, 20 + w % 3, 30], temperature, mix_seed(7, w), rows, key=w))
        search = Search(cfg, _fake_step_with(_mixed_logits, seed), W, K, 4, "beam", dtype=torch.float32,
                        device="cpu", max_length=36, graphs=False, fused=False, sampling_slots=True)
        rec = {}
        orig_choose, orig_body = search._choose, search._body

        def choose(logits, s=search, orig=orig_choose, rec=rec):
            rec["logits"] = logits.clone()
            orig(logits)

        def body(s=search, orig=orig_body, rec=rec):
            nonlocal step_no
            before = {f: getattr(s, f).clone() for f in MIXED_FIELDS}
            orig()
            key = f"step{step_no:04d}"
            for f in MIXED_FIELDS:
                out[f"{key}/before/{f}"] = before[f].numpy()
                out[f"{key}/after/{f}"] = getattr(s, f).numpy().copy()
            out[f"{key}/logits"] = rec["logits"].numpy()
            out[f"{key}/meta"] = np.array([K, s.P, MIXED_V, EOT, NOSPEECH, run], dtype=np.int64)
            step_no += 1

        search._choose = choose
        search._body = body

        class Src:
            def __init__(self, jobs):
                self.ready = list(jobs)

            def take(self, n, block=False):
                got, self.ready = self.ready[:n], self.ready[n:]
                return got

            def load(self, slots, jobs):
                pass

            def result(self, job, result):
                pass

        search.serve(Src(jobs), [5, 6, 7], [8, EOT], check_every=1, ahead=1)
    return out


# --- the beam step's candidate scores: masks, timestamp rules, log-softmax + cum, top-2K (reference Search) ------
TS_V, TS_NOTS, TS_TSB = 120, 40, 41  # toy vocabulary with timestamps: text 4..39, <|notimestamps|> 40, 41.. times


def _ts_logits(history, seed):
    """Pseudo-random logits of a history that keep every timestamp rule busy: the timestamps just after the
    latest one are favoured, the rest disfavoured, and EOS grows likelier with length."""
    g = torch.Generator().manual_seed(zlib.crc32(repr(("ts-golden", seed, history)).encode()))
    x = torch.randn(TS_V, generator=g, dtype=torch.float64) * 2.5
    x[EOT] += 0.2 * len(history)
    latest = max([h - TS_TSB for h in history if h >= TS_TSB], default=-1)
    near = torch.arange(TS_V - TS_TSB)
    x[TS_TSB:] += torch.where((near > latest) & (near <= latest + 5), 2.0, -1.0).double()
    return x


def _fake_step_with(logits_of, seed):
    def step_fn(tokens, offset, cache, logits, new_kv, src):
        def run():
            for n in range(tokens.shape[0]):
                off = int(offset[n])
                hist = [int(round(float(cache[0, 0, int(src[n, j]), 0, j, 0]))) for j in range(off)]
                for s in range(tokens.shape[1]):
                    tok = int(tokens[n, s])
                    logits[n, s] = logits_of(hist + [tok], seed).float()
                    new_kv[0, :, n, 0, s, :] = float(tok)
                    hist.append(tok)

        return run

    return step_fn


def scores_golden(ref_src: str) -> dict:
    """Per beam step of the reference Search (PyTorch path, CPU): its inputs (logits, t, cum, hist) and its
    candidate scores (log-softmax of the masked logits + cum), best 2K and no-speech probabilities; two decodes
    without timestamps (V 40, beam 3 / 5) and two with CTranslate2's timestamp rules (V 120, beam 3 / 4)."""
    from whisper_trt.config import WhisperConfig
    from whisper_trt.search import Search

    out = {}
    step_no = 0
    runs = [(3, 10, False), (5, 11, False), (3, 12, True), (4, 13, True)]
    for run, (K, seed, ts) in enumerate(runs):
        if ts:
            cfg = WhisperConfig(n_mels=4, d_model=4, enc_layers=1, enc_heads=1, enc_ffn=4, dec_layers=1,
                                dec_heads=1, dec_ffn=4, vocab_size=TS_V, eot=EOT, sot=SOT, no_speech=NOSPEECH,
                                no_timestamps=TS_NOTS, timestamp_begin=TS_TSB)
            fake, vocab = _fake_step_with(_ts_logits, seed), TS_V
            prompts = [[SOT, 10 + w, 20 + w % 3] for w in range(5)]
        else:
            cfg = WhisperConfig(n_mels=4, d_model=4, enc_layers=1, enc_heads=1, enc_ffn=4, dec_layers=1,
                                dec_heads=1, dec_ffn=4, vocab_size=V, eot=EOT, sot=SOT, no_speech=NOSPEECH)
            fake, vocab = _fake_step_with(_scores_of, seed), V
            prompts = [[SOT, 10 + w, 20 + w % 3, 30] for w in range(5)]
        W = 2
        search = Search(cfg, fake, W, K, len(prompts[0]), "beam", dtype=torch.float32, device="cpu",
                        max_length=40 if not ts else 36, graphs=False, fused=False, timestamps=ts)
        rec = {}
        orig_choose, orig_beam = search._choose, search._beam

        def choose(logits, s=search, orig=orig_choose, rec=rec):
            rec.clear()
            rec["logits"] = logits.clone()
            rec["t"], rec["cum"], rec["hist"] = s.t.clone(), s.cum.clone(), s.hist.clone()
            orig(logits)

        def beam(logp, prompt, s=search, orig=orig_beam, rec=rec):
            nonlocal step_no
            sc = logp + s.cum[:, None]
            top_s, top_i = sc.view(s.B, -1).topk(2 * s.K, dim=1)
            lg = rec["logits"][:: s.K]
            ns = (lg[:, s.cfg.no_speech] - lg.logsumexp(-1)).exp()
            key = f"step{step_no:04d}"
            out[f"{key}/logits"] = rec["logits"].numpy()
            out[f"{key}/t"] = rec["t"].numpy()
            out[f"{key}/cum"] = rec["cum"].numpy()
            out[f"{key}/hist"] = rec["hist"].numpy()
            out[f"{key}/scores"] = sc.numpy()
            out[f"{key}/top_s"] = top_s.numpy()
            out[f"{key}/top_i"] = top_i.numpy()
            out[f"{key}/ns"] = ns.numpy()
            out[f"{key}/suppress"] = s.suppress.numpy()
            out[f"{key}/begin"] = s.begin.numpy()
            out[f"{key}/meta"] = np.array([K, vocab, int(ts), int(s.max_initial[0]), s.cfg.no_speech,
                                           s.cfg.no_timestamps or 0, s.cfg.timestamp_begin or 0, s.cfg.eot, run],
                                          dtype=np.int64)
            step_no += 1
            orig(logp, prompt)

        search._choose = choose
        search._beam = beam
        suppress, begin = [5, 6, 7], [8, EOT]
        search.stream(prompts, lambda slots, windows: None, suppress, begin, check_every=1, ahead=1,
                      **({"max_initial_timestamp_index": 10} if ts else {}))
    return out


def decoder_golden(ref_src: str) -> dict:
    """The fused linear layers of decoder_kernels.py as the reference's own modules compute them on CPU:
    ``modeling.LayerNorm`` (fp32 statistics with ``Precision.ln32``, rounded to fp16), ``modeling.gelu`` (fp32 with
    ``Precision.gelu32``), and the GEMM in fp32 rounded to fp16 before the GELU / residual (the rounding points the
    module's docstring states, decoder_kernels.py:1-15)."""
    from whisper_trt import modeling

    modeling.Precision.ln32 = True
    modeling.Precision.gelu32 = True
    out = {}
    for name, kw in cases.DEC_CASES.items():
        inp = cases.linear_case(**kw)
        out[f"{name}/digest"] = np.array(cases.digest(*[inp[k] for k in sorted(inp)]))
        k = inp["x"].shape[1]
        ln = modeling.LayerNorm(k).half()
        with torch.no_grad():
            ln.weight.copy_(inp["gamma"])
            ln.bias.copy_(inp["beta"])
            xn = ln(inp["x"])  # fp16
            h = (xn.float() @ inp["w"].float().t() + inp["b"].float()).half()
            out[f"{name}/ln_linear"] = h.numpy()
            out[f"{name}/ln_linear_gelu"] = modeling.gelu(h).numpy()
            g = (inp["x"].float() @ inp["w"].float().t() + inp["b"].float()).half()
            out[f"{name}/linear_residual"] = (g.float() + inp["res"].float()).half().numpy()
            out[f"{name}/layer_norm"] = xn.numpy()
            out[f"{name}/x_plus_bias"] = (inp["x"].float() + inp["bias"].float()).half().numpy()
    return out


def main() -> None:
    ap_ = argparse.ArgumentParser()
    ap_.add_argument("--reference-src", required=True)
    ap_.add_argument("--only", choices=["decoder", "mixed"], default=None, help="write only this fixture")
    args = ap_.parse_args()
    sys.path.insert(0, args.reference_src)
    if args.only == "mixed":
        m = mixed_golden(args.reference_src)
        np.savez_compressed(HERE / "mixed_golden.npz", **m)
        print(f"mixed-slot steps: {sum(k.endswith('/meta') for k in m)}")
        return
    if args.only == "decoder":
        d = decoder_golden(args.reference_src)
        np.savez_compressed(HERE / "decoder_golden.npz", **d)
        print(f"decoder cases: {len(cases.DEC_CASES)}")
        return
    from whisper_trt import attn_plugin

    attn_plugin.RUNTIME_TRITON = False
    torch.set_num_threads(max(1, torch.get_num_threads()))
    a = attn_golden(attn_plugin)
    np.savez_compressed(HERE / "attn_golden.npz", **a)
    s = slots_golden(args.reference_src)
    np.savez_compressed(HERE / "slots_golden.npz", **s)
    sc = scores_golden(args.reference_src)
    np.savez_compressed(HERE / "scores_golden.npz", **sc)
    np.savez_compressed(HERE / "decoder_golden.npz", **decoder_golden(args.reference_src))
    np.savez_compressed(HERE / "mixed_golden.npz", **mixed_golden(args.reference_src))
    print(f"attn cases: {len(cases.ATTN_CASES)}; bookkeeping steps: {sum(k.endswith('/meta') for k in s)}; "
          f"scoring steps: {sum(k.endswith('/meta') for k in sc)}")


if __name__ == "__main__":
    main()
