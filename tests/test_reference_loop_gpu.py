"""The drop-in through the reference's own decode loop.

The reference's ``Search`` (search.py:148-265: its step body, its PyTorch or fused bookkeeping, its CUDA-graph capture
:674-685) drives its ``TritonDecoderBackend`` (runtime.py:73-205) on a random-init whisper-large-v3-shaped
``WhisperModel(cfg)`` (modeling.py:283-288; the cross-attention keys/values from its own encoder on seeded features,
``TorchBackend.encode``, runtime.py:44-47). Nothing of the reference is modified: this package is installed into its
modules with ``install()`` (``attn_plugin`` always; ``decoder_kernels`` and ``beam_kernels`` in the variant that runs
the whole step here), and the same loop on the reference's own kernels -- the module unrouted, its Triton kernels --
is the reference.

* Teacher-forced: the two loops step in lockstep; after every step this package's loop is compared with the
  reference's (tokens, slot tables, histories, positions, done flags, hypotheses bit-exact; cumulative scores and
  no-speech probabilities within a tolerance) and then given the reference's state, so every step is compared on
  the same state. The bar is the north star's: identical at every step.
* Free-running: one beam decode through the reference's public ``Search.stream`` from start to end on each side;
  the windows' final hypotheses must be identical.

Needs the reference package staged at ``baseline/_ref/whisper_trt`` (git-ignored) and Triton; skipped otherwise.
"""

from __future__ import annotations

import contextlib
import functools
import sys
from pathlib import Path
from types import SimpleNamespace

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]

REF = Path(__file__).resolve().parent.parent / "baseline" / "_ref"
# whisper-large-v3 (its config.json): 128 mel bins, d 1280, 32 + 32 layers of 20 heads, MLP 5120, 51866 tokens
LARGE_V3 = dict(n_mels=128, d_model=1280, enc_layers=32, enc_heads=20, enc_ffn=5120, dec_layers=32, dec_heads=20,
                dec_ffn=5120, vocab_size=51866)
PROMPT = [50258, 50259, 50359, 50363]  # <|startoftranscript|> <|en|> <|transcribe|> <|notimestamps|>
WINDOWS = 4
INT_STATE = ("tokens", "pos", "t", "done", "row_done", "length", "hist", "src")
BEAM_STATE = ("h_count", "h_len", "h_tokens")
FLOAT_STATE = ("cum", "no_speech")


@pytest.fixture(scope="module")
def ref():
    if not (REF / "whisper_trt" / "runtime.py").is_file():
        pytest.skip("the reference package is not staged under baseline/_ref")
    pytest.importorskip("triton")
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    from whisper_trt import attn_plugin, beam_kernels, config, decoder_kernels, modeling, runtime, search

    return SimpleNamespace(attn_plugin=attn_plugin, beam_kernels=beam_kernels, config=config,
                           decoder_kernels=decoder_kernels, modeling=modeling, runtime=runtime, search=search)


@pytest.fixture(scope="module")
def model(ref):
    """The reference's WhisperModel at whisper-large-v3's shape on the GPU (fp16), and every layer's cross-attention
    keys/values of WINDOWS windows from its encoder on seeded features. The decoder's weights, biases and embeddings
    are re-drawn N(0, 0.02) (seed 0; LayerNorms as constructed), the weight scale the benchmark configs state: with
    the module's default initialisation the tied N(0, 1) token embedding dominates the residual stream and the
    decoder repeats its input token by a margin of ~300 logits, which no attention error could change."""
    cfg = ref.config.WhisperConfig(**LARGE_V3)
    torch.manual_seed(0)
    with torch.device("cuda"):
        m = ref.modeling.WhisperModel(cfg)
    g = torch.Generator(device="cuda").manual_seed(0)
    with torch.no_grad():
        for name, p in m.decoder.named_parameters():
            if "layer_norm" not in name:
                p.copy_(torch.randn(p.shape, generator=g, device="cuda") * 0.02)
    m = m.half().eval().requires_grad_(False)
    g = torch.Generator(device="cuda").manual_seed(1)
    feats = torch.randn(WINDOWS, cfg.n_mels, 3000, generator=g, device="cuda")
    L, H, D = cfg.dec_layers, cfg.dec_heads, cfg.head_dim
    cross = torch.empty(L, 2, WINDOWS, H, cfg.enc_frames, D, dtype=torch.float16, device="cuda")
    ref.runtime.TorchBackend(m).encode(feats, cross)
    assert bool(torch.isfinite(cross).all())
    return cfg, m, cross


@contextlib.contextmanager
def _installed(ref, whole_step: bool):
    """This package installed into the reference's modules for the duration, then the modules restored (graphs
    captured meanwhile keep the kernels they captured)."""
    from whisper_trt_b200 import attn_plugin, decoder_kernels, slots

    pairs = [(ref.attn_plugin, attn_plugin)]
    if whole_step:
        pairs += [(ref.decoder_kernels, decoder_kernels), (ref.beam_kernels, slots)]
    saved = [(mod, dict(vars(mod))) for mod, _ in pairs]
    for mod, ours in pairs:
        ours.install(mod)
    try:
        yield
    finally:
        for mod, names in saved:
            for name, value in names.items():
                setattr(mod, name, value)


def _search(ref, cfg, model, cross, mode, rows, gemm, fused):
    """The reference's Search over WINDOWS slots on its TritonDecoderBackend, graph captured, no window loaded."""
    backend = ref.runtime.TritonDecoderBackend(model, encoder=None, gemm=gemm)
    slots_cross = torch.zeros_like(cross)
    s = ref.search.Search(cfg, functools.partial(backend.step_fn, cross=slots_cross), WINDOWS, rows,
                          prompt_length=len(PROMPT), mode=mode, fused=fused, graphs=True)
    s.prepare()
    s.slots_cross = slots_cross
    return s


def _load(ref, s, cross, cfg):
    """WINDOWS windows into the slots, as Search.serve loads them (search.py:502-513): the windows' keys/values into
    the slots, the suppressed / begin-suppressed tokens, then Search._start."""
    s.slots_cross.copy_(cross)
    s.suppress.zero_()
    s.begin.zero_()
    s.begin[torch.tensor(list(cfg.begin_suppress_tokens), device="cuda")] = True
    s.done.fill_(True)
    s.row_done.fill_(True)
    s._start(list(range(WINDOWS)), [ref.search.Job(list(PROMPT)) for _ in range(WINDOWS)])


def _lockstep(ref, cfg, model, cross, mode, rows, gemm, fused, steps):
    """Both loops, teacher-forced; returns the report (and asserts identity at every step)."""
    theirs = _search(ref, cfg, model, cross, mode, rows, gemm, fused)
    with _installed(ref, whole_step=gemm == "triton"):
        ours = _search(ref, cfg, model, cross, mode, rows, gemm, fused)
    for s in (theirs, ours):
        _load(ref, s, cross, cfg)
    names = INT_STATE + (BEAM_STATE if mode == "beam" else ())
    floats = FLOAT_STATE + (("h_score",) if mode == "beam" else ())
    mismatches, worst_logit, worst_float, min_margin, chosen = [], 0.0, 0.0, float("inf"), []
    # (scores are sums of fp32 log-probabilities: compared relative to their size)
    for step in range(steps):
        theirs._run_step()
        ours._run_step()
        torch.cuda.synchronize()
        a, b = theirs.logits[:, 0], ours.logits[:, 0]
        worst_logit = max(worst_logit, float((a - b).abs().max()))
        top2 = a.topk(2, dim=-1).values
        min_margin = min(min_margin, float((top2[:, 0] - top2[:, 1]).min()))
        differ = [n for n in names if not torch.equal(getattr(theirs, n), getattr(ours, n))]
        for n in floats:
            x, y = getattr(theirs, n), getattr(ours, n)
            fin = torch.isfinite(x)
            if not torch.equal(fin, torch.isfinite(y)):
                differ.append(n)
            elif bool(fin.any()):
                worst_float = max(worst_float, float(((x[fin] - y[fin]).abs() / (1 + x[fin].abs())).max()))
        if differ:
            mismatches.append((step, differ))
        chosen.append(theirs.tokens[:, 0].clone())
        for n in names + floats:  # teacher forcing: the next step starts from the reference's state
            getattr(ours, n).copy_(getattr(theirs, n))
        if bool(theirs.done.all()):
            break
    distinct = len(set(torch.stack(chosen[len(PROMPT) - 1:]).flatten().tolist()))
    report = (f"{mode} x{rows}, gemm {gemm}, fused bookkeeping {fused}: {len(chosen)} steps, "
              f"{len(mismatches)} with a difference {mismatches[:5]}; max |logit diff| {worst_logit:.2e}, "
              f"max score / no-speech diff {worst_float:.2e} (relative to 1 + |score|), min top-1 margin "
              f"{min_margin:.3e}, "
              f"{distinct} distinct tokens chosen")
    print(report)
    assert not mismatches, report
    assert worst_float < 1e-2, report
    assert distinct > 1, report  # (the tokens depend on the windows: the attention is doing something)
    return report


def test_greedy_teacher_forced_identical(ref, model):
    cfg, m, cross = model
    _lockstep(ref, cfg, m, cross, "greedy", 1, "cublas", False, steps=64)


def test_beam_teacher_forced_identical(ref, model):
    cfg, m, cross = model
    _lockstep(ref, cfg, m, cross, "beam", 5, "cublas", False, steps=48)


def test_beam_whole_step_teacher_forced_identical(ref, model):
    """The whole step on this package: attention, the linear layers (the backend's ``gemm="triton"`` variant, routed
    to decoder_kernels), logits32 and the fused beam bookkeeping (beam_kernels routed to slots) -- against the
    reference's same configuration on its Triton kernels."""
    cfg, m, cross = model
    _lockstep(ref, cfg, m, cross, "beam", 5, "triton", True, steps=32)


def test_beam_stream_free_running_identical(ref, model):
    """One beam decode of the WINDOWS windows through the reference's public Search.stream, start to end, on each
    side: the same final hypotheses."""
    cfg, m, cross = model
    results = {}
    for side in ("theirs", "ours"):
        ctx = _installed(ref, whole_step=False) if side == "ours" else contextlib.nullcontext()
        with ctx:
            s = _search(ref, cfg, m, cross, "beam", 5, "cublas", False)

        def load(slots, windows, s=s):
            for slot, w in zip(slots, windows):
                s.slots_cross[:, :, slot].copy_(cross[:, :, w])

        out = s.stream([list(PROMPT)] * WINDOWS, load, suppress=[], begin_suppress=list(cfg.begin_suppress_tokens))
        results[side] = [(r.tokens, r.hypothesis.length, [h.tokens for h in r.hypotheses]) for r in out]
        scores = [r.hypothesis.score for r in out]
        results[side + "_scores"] = scores
    assert results["ours"] == results["theirs"]
    diff = max(abs(a - b) / (1 + abs(b)) for a, b in zip(results["ours_scores"], results["theirs_scores"]))
    assert diff < 1e-2, diff
    print(f"stream: {WINDOWS} windows, lengths {[r[1] for r in results['ours']]}, identical hypotheses; "
          f"max |score diff| {diff:.2e}")
