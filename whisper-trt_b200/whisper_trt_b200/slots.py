"""Slot-table bookkeeping of beam search on the GPU (the step part that feeds parent indices to the attention).

Beam search never moves the KV cache: row r (window r // K) reads each cache slot from the row ``src[r, slot]``
names. Per step a new beam takes its parent's table and marks the slot its parent just wrote. These wrap the C-ABI
kernels (``wt_beam_reorder``, ``wt_beam_update``, ``wt_slot_reset``); integer work, bit-exact with the reference:

* :func:`beam_reorder` -- the reorder with the parents given: search.py:258 + :401-409 + :263-264;
* :func:`update` -- a drop-in for the reference's ``beam_kernels.update(s, top_s, top_i, ns)``
  (beam_kernels.py:292-302, kernel :169-269) in beam mode: CTranslate2's candidate rules, hypotheses, the new
  beams' histories / tables / scores / tokens, prompt feeding, advancing;
* :func:`slot_reset` -- a window loaded into slots (search.py:440-446);
* :func:`scores` / :func:`best` -- the scoring half of the step: masked log-softmax + cumulative score (with
  CTranslate2's timestamp rules when ``s.timestamps``), no-speech probabilities and each window's best 2K
  candidates in one kernel (``wt_beam_scores``): the reference's beam_kernels.scores (beam_kernels.py:351-361,
  kernel :36-135) and the torch.topk after it (search.py:253);
* :func:`step_bookkeeping` -- scores, best 2K and update: the fused branch of the reference's Search._body
  (search.py:251-256) in two kernels;
* :func:`sample` -- sampled slots (Search(sampling_slots=True)): each sampled row's token by Gumbel-max with the
  reference's counter-based random numbers (beam_kernels.py:136-167, search.py:104-129), which :func:`update` then
  applies under CTranslate2's GreedySearch rules.
"""

from __future__ import annotations

import torch

from . import _lib


_workspaces: dict[tuple, torch.Tensor] = {}


def _workspace(dev: torch.device, key: tuple, nbytes: int) -> torch.Tensor:
    k = (dev.index if dev.index is not None else torch.cuda.current_device(),) + key
    ws = _workspaces.get(k)
    if ws is None or ws.numel() < nbytes:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError(f"beam_scores workspace of {nbytes} bytes needed during CUDA-graph capture: run the "
                               "call once before capturing")
        ws = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=dev)
        _workspaces[k] = ws
    return ws


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _need(what: str, t: torch.Tensor, dtype: torch.dtype, shape: tuple | None = None) -> None:
    if t.dtype != dtype:
        raise TypeError(f"{what}: expected {dtype}, got {t.dtype}")
    if not t.is_cuda or not t.is_contiguous():
        raise ValueError(f"{what}: contiguous CUDA tensors only")
    if shape is not None and tuple(t.shape) != tuple(shape):
        raise ValueError(f"{what}: expected shape {tuple(shape)}, got {tuple(t.shape)}")


def beam_reorder(src: torch.Tensor, parent: torch.Tensor, pos: torch.Tensor, hist: torch.Tensor | None = None,
                 token: torch.Tensor | None = None, t: torch.Tensor | None = None, live: torch.Tensor | None = None,
                 offset: torch.Tensor | None = None, advance: bool = True) -> None:
    """In place: for each live window b and new beam k with parent p = parent[b, k], ``src[b*K+k] = src[b*K+p]``
    with slot pos[b] marked as row b*K+p; ``hist`` likewise, with ``token`` written at t[b]; pos[b] += 1 when
    ``advance``; ``offset`` (if given) = the rows' new pos. src [N, C] int32, parent [B, K] int64, pos [B] int64,
    hist [N, T] int64, token [N] int64, t [B] int64, live [B] bool, offset [N] int64."""
    what = "beam_reorder"
    b, k = parent.shape
    n, c = src.shape
    if n != b * k:
        raise ValueError(f"{what}: src has {n} rows, parent {b} x {k}")
    _need(what, src, torch.int32)
    _need(what, parent, torch.int64)
    _need(what, pos, torch.int64, (b,))
    tl = 0
    if hist is not None:
        _need(what, hist, torch.int64)
        if hist.shape[0] != n:
            raise ValueError(f"{what}: hist must have N rows")
        tl = hist.shape[1]
    if token is not None:
        _need(what, token.view(-1), torch.int64, (n,))
        if hist is None or t is None:
            raise ValueError(f"{what}: token needs hist and t")
    if t is not None:
        _need(what, t, torch.int64, (b,))
    if live is not None:
        _need(what, live, torch.bool, (b,))
    if offset is not None:
        _need(what, offset, torch.int64, (n,))
    dev = src.device
    with torch.cuda.device(dev):
        st = _lib.load().wt_beam_reorder(src.data_ptr(), _ptr(hist), _ptr(token), _ptr(t), parent.data_ptr(),
                                         pos.data_ptr(), _ptr(live), _ptr(offset), b, k, c, tl, int(advance),
                                         torch.cuda.current_stream(dev).cuda_stream)
    _lib.check(st, what)


def update(s, top_s: torch.Tensor, top_i: torch.Tensor, ns: torch.Tensor) -> None:
    """The step's bookkeeping on ``s`` (a search state with the reference Search's buffers, beam mode) from the best
    2K candidates -- the reference's beam_kernels.update (beam_kernels.py:292-302). With sampled slots
    (``s.mixed``, Search(sampling_slots=True)) the sampled windows take their rows' tokens from :func:`sample`
    (``s.samp_tok``, ``s.samp_score``) under CTranslate2's GreedySearch rules."""
    what = "beam_update"
    mixed = bool(getattr(s, "mixed", False))
    B, K = s.pos.shape[0], s.K
    n, c = s.src.shape
    T = s.hist.shape[1]
    S = s.h_score.shape[1]
    _need(what, top_s, torch.float32, (B, 2 * K))
    _need(what, top_i, torch.int64, (B, 2 * K))
    _need(what, ns, torch.float32, (B,))
    for name, dt in (("t", torch.int64), ("pos", torch.int64), ("sot_pos", torch.int64), ("no_speech", torch.float32),
                     ("done", torch.bool), ("hist", torch.int64), ("cum", torch.float32), ("src", torch.int32),
                     ("tokens", torch.int64), ("forced", torch.int64), ("h_count", torch.int64),
                     ("h_score", torch.float32), ("h_len", torch.int64), ("h_tokens", torch.int64),
                     ("last_t", torch.int64)):
        _need(f"{what}.{name}", getattr(s, name), dt)
    mix = [None] * 5
    if mixed:
        for name, dt, shape in (("sampling", torch.bool, (B,)), ("samp_tok", torch.int64, (n,)),
                                ("samp_score", torch.float32, (n,)), ("row_done", torch.bool, (n,)),
                                ("length", torch.int64, (n,))):
            _need(f"{what}.{name}", getattr(s, name), dt, shape)
        mix = [s.sampling.data_ptr(), s.samp_tok.data_ptr(), s.samp_score.data_ptr(), s.row_done.data_ptr(),
               s.length.data_ptr()]
    dev = s.src.device
    with torch.cuda.device(dev):
        st = _lib.load().wt_beam_update_mixed(
            top_s.data_ptr(), top_i.data_ptr(), s.t.data_ptr(), s.pos.data_ptr(), s.sot_pos.data_ptr(),
            ns.data_ptr(), s.no_speech.data_ptr(), s.done.data_ptr(), s.hist.data_ptr(), s.cum.data_ptr(),
            s.src.data_ptr(), s.tokens.data_ptr(), s.forced.data_ptr(), s.h_count.data_ptr(), s.h_score.data_ptr(),
            s.h_len.data_ptr(), s.h_tokens.data_ptr(), s.last_t.data_ptr(), *mix, B, K, c, T, S, s.P,
            s.cfg.vocab_size, s.cfg.eot, torch.cuda.current_stream(dev).cuda_stream)
    _lib.check(st, what)


def sample(s) -> None:
    """Each sampled row's token and its log-probability (``s.samp_tok``, ``s.samp_score``) from the scores
    :func:`scores` wrote (``s.scores``: the sampled rows' log-probabilities), by Gumbel-max on ``log_probs /
    temperature`` with the reference's counter-based random numbers (search.uniform) -- the reference's
    beam_kernels.sample (beam_kernels.py:284-289, kernel :136-167)."""
    what = "beam_sample"
    B, K = s.pos.shape[0], s.K
    n = B * K
    _need(what, s.scores, torch.float32)
    if s.scores.shape[0] != n:
        raise ValueError(f"{what}: scores has {s.scores.shape[0]} rows, expected {n}")
    v = s.scores.shape[1]
    for name, dt, shape in (("t", torch.int64, (B,)), ("done", torch.bool, (B,)), ("row_done", torch.bool, (n,)),
                            ("sampling", torch.bool, (B,)), ("temperature", torch.float32, (B,)),
                            ("seed", torch.int64, (B,)), ("samp_tok", torch.int64, (n,)),
                            ("samp_score", torch.float32, (n,))):
        _need(f"{what}.{name}", getattr(s, name), dt, shape)
    dev = s.scores.device
    with torch.cuda.device(dev):
        st = _lib.load().wt_beam_sample(s.scores.data_ptr(), s.t.data_ptr(), s.done.data_ptr(), s.row_done.data_ptr(),
                                        s.sampling.data_ptr(), s.temperature.data_ptr(), s.seed.data_ptr(),
                                        s.samp_tok.data_ptr(), s.samp_score.data_ptr(), B, K, v,
                                        torch.cuda.current_stream(dev).cuda_stream)
    _lib.check(st, what)


def slot_reset(src: torch.Tensor, slots: torch.Tensor, K: int, prefilled: bool) -> None:
    """Rows of each slot s in ``slots`` read their own cache rows (src[r] = r) or, ``prefilled``, the slot's first
    row (src[r] = s*K), as the reference's Search._start (search.py:440-446)."""
    what = "slot_reset"
    _need(what, src, torch.int32)
    _need(what, slots, torch.int64)
    n, c = src.shape
    dev = src.device
    with torch.cuda.device(dev):
        st = _lib.load().wt_slot_reset(src.data_ptr(), slots.data_ptr(), slots.numel(), n // K, K, c, int(prefilled),
                                       torch.cuda.current_stream(dev).cuda_stream)
    _lib.check(st, what)


def best(s, logits: torch.Tensor, ns: torch.Tensor, out: torch.Tensor | None = None,
         top: tuple[torch.Tensor, torch.Tensor] | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Each window's best 2K candidates (top_s [B, 2K] float32, top_i [B, 2K] int64 = beam * V + token, best
    first) of the scores log_softmax(masked logits) + cum; ``ns`` [B] gets the no-speech probabilities and ``out``
    [N, V] (optional) the scores themselves. ``s`` is a search state with the reference Search's buffers (beam
    mode): suppress / begin [V] bool, t [B], cum [N], hist [N, T], max_initial [1], K, cfg, timestamps."""
    what = "beam_scores"
    B, K = s.t.shape[0], s.K
    n, v = logits.shape
    if n != B * K:
        raise ValueError(f"{what}: logits has {n} rows, expected {B} x {K}")
    _need(what, logits, torch.float32)
    _need(what, ns, torch.float32, (B,))
    if out is not None:
        _need(what, out, torch.float32, (n, v))
    for name, dt, shape in (("suppress", torch.bool, (v,)), ("begin", torch.bool, (v,)), ("t", torch.int64, (B,)),
                            ("cum", torch.float32, (n,)), ("hist", torch.int64, None),
                            ("max_initial", torch.int64, (1,))):
        _need(f"{what}.{name}", getattr(s, name), dt, shape)
    if top is None:
        top = (torch.empty(B, 2 * K, dtype=torch.float32, device=logits.device),
               torch.empty(B, 2 * K, dtype=torch.int64, device=logits.device))
    top_s, top_i = top
    _need(what, top_s, torch.float32, (B, 2 * K))
    _need(what, top_i, torch.int64, (B, 2 * K))
    c = s.cfg
    ts = bool(getattr(s, "timestamps", False))
    sampling = None
    if getattr(s, "mixed", False):  # (sampled windows' rows score their log-probabilities alone)
        _need(f"{what}.sampling", s.sampling, torch.bool, (B,))
        sampling = s.sampling.data_ptr()
    dev = logits.device
    lib = _lib.load()
    nbytes = int(lib.wt_beam_scores_workspace(B, K))
    ws = _workspace(dev, ("scores", B, K), nbytes)
    with torch.cuda.device(dev):
        st = lib.wt_beam_scores_mixed(logits.data_ptr(), s.suppress.data_ptr(), s.begin.data_ptr(), s.t.data_ptr(),
                                s.cum.data_ptr(), sampling, s.hist.data_ptr(), s.max_initial.data_ptr(), _ptr(out),
                                ns.data_ptr(), top_s.data_ptr(), top_i.data_ptr(), B, K, v, s.hist.shape[1], int(ts),
                                c.no_speech, (c.no_timestamps or 0) if ts else 0, (c.timestamp_begin or 0) if ts else 0,
                                c.eot, ws.data_ptr(), nbytes, torch.cuda.current_stream(dev).cuda_stream)
    _lib.check(st, what)
    return top_s, top_i


def scores(s, logits: torch.Tensor, out: torch.Tensor, ns: torch.Tensor) -> None:
    """``out`` [N, V] = log_softmax(masked logits [N, V]) + cum[:, None], ``ns`` [B] the no-speech probabilities --
    the reference's beam_kernels.scores(s, logits, out, ns) (beam mode), as a drop-in."""
    best(s, logits, ns, out=out)


def step_bookkeeping(s, logits: torch.Tensor, ns: torch.Tensor) -> None:
    """One step's bookkeeping from the decoder's logits [N, V]: the best 2K candidates of every window, then
    :func:`update` -- the fused branch of the reference's Search._body (search.py:251-256) without materialising
    the [N, V] scores."""
    top_s, top_i = best(s, logits, ns)
    update(s, top_s, top_i, ns)


def install(module) -> None:
    """Route a reference ``whisper_trt.beam_kernels`` module's bookkeeping (``scores``, ``sample``, ``update``) to
    these kernels (in place), so that the reference's ``Search._body`` (search.py:251-256, ``fused=True``, with or
    without sampled slots) runs on them unchanged."""
    for name in ("scores", "sample", "update"):
        setattr(module, name, globals()[name])
