"""CPU restatement (numpy) of the reference's slot-table bookkeeping -- TEST INFRASTRUCTURE ONLY.

The parity checker for the slot-table kernels of ``whisper_trt_b200`` (integer work: bit-exact). Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs may import it.

Beam search never moves the KV cache. Each decoder row ``r`` (window ``b = r // K``, beam ``r % K``) has a slot
table ``src[r, :]`` naming, for every cache slot, the row whose cache holds it. Per step (reference
``src/whisper_trt/search.py``):

* ``_body`` (search.py:247-258): every row writes its new key/value at its window's position ``pos[b]`` into its
  own cache row, so its table marks that slot as its own: ``src[r, pos[b]] = r``;
* ``_beam`` (search.py:401-409): a new beam with parent ``p`` takes the parent's table and history:
  ``src[b*K + k] = src[b*K + p]``, ``hist[b*K + k] = hist[b*K + p]`` plus its token at index ``t[b]``;
* windows still decoding advance: ``pos += 1`` (search.py:263-265);
* ``_start`` (search.py:440-446): a window loaded into a slot gets ``src[r] = r`` (its own rows), or
  ``src[r] = s*K`` when the prompt was prefilled into the slot's first row (its beams share the prefix).

The fused CUDA path of the reference does all of it per window in ``beam_kernels._update_kernel``
(beam_kernels.py:169-269); :func:`beam_update` restates that kernel's beam mode.
"""

from __future__ import annotations

import numpy as np


def mark_own_slot(src: np.ndarray, offset: np.ndarray) -> None:
    """search.py:258: ``src[r, offset[r]] = r`` in place (slots >= C are left alone, as the fused kernel's
    ``cc < C`` mask does, beam_kernels.py:184)."""
    n, c = src.shape
    for r in range(n):
        o = int(offset[r])
        if 0 <= o < c:
            src[r, o] = r


def beam_reorder(src: np.ndarray, parent: np.ndarray, pos: np.ndarray, hist: np.ndarray | None = None,
                 token: np.ndarray | None = None, t: np.ndarray | None = None, live: np.ndarray | None = None,
                 advance: bool = True) -> None:
    """The slot-table step of beam search with the parents given, in place.

    src [N, C] int32; parent [B, K] (each new beam's parent beam within its window, 0..K-1); pos [B] int64;
    hist [N, T] int64 (optional); token [N] (optional: written into the new history at t[b]); live [B]
    (optional: windows with 0 are left untouched). For each live window b and new beam k with parent p:

        src[b*K+k]         = src_old[b*K+p], then src[b*K+k, pos[b]] = b*K+p   (search.py:258 + :402-409;
                                                                             beam_kernels.py:246-248,264)
        hist[b*K+k]        = hist_old[b*K+p], then hist[b*K+k, t[b]] = token[b*K+k]   (search.py:403-405)
        pos[b] += 1 when ``advance``                                             (search.py:263-264)
    """
    n, c = src.shape
    b_, k_ = parent.shape
    assert b_ * k_ == n
    src_old = src.copy()
    hist_old = hist.copy() if hist is not None else None
    for b in range(b_):
        if live is not None and not live[b]:
            continue
        pb = int(pos[b])
        for k in range(k_):
            r = b * k_ + k
            p = b * k_ + int(parent[b, k])
            src[r] = src_old[p]
            if 0 <= pb < c:
                src[r, pb] = p
            if hist is not None:
                hist[r] = hist_old[p]
                if token is not None and t is not None:
                    tb = int(t[b])
                    if 0 <= tb < hist.shape[1]:
                        hist[r, tb] = token[r]
        if advance:
            pos[b] += 1


def slot_reset(src: np.ndarray, slots: np.ndarray, K: int, prefilled: bool) -> None:
    """search.py:440-446 (``_start``): the rows of each loaded slot s read their own cache rows (``src[r] = r``),
    or, prefilled, all K rows read the slot's first row ``s*K`` (which holds the prompt prefix)."""
    for s in np.asarray(slots).tolist():
        for k in range(K):
            r = s * K + k
            src[r, :] = s * K if prefilled else r


def beam_update(st: dict, top_s: np.ndarray, top_i: np.ndarray, ns: np.ndarray, V: int, EOT: int) -> None:
    """beam_kernels.py:169-269 ``_update_kernel``, beam mode without sampled slots, in place on ``st``.

    ``st`` holds the search state (reference search.py:184-223 names): t, pos, sot_pos [B] int64; no_speech [B]
    f32; done [B] bool; hist [N, T] int64; cum [N] f32; src [N, C] int32; tokens [N] int64; forced [B, P+1]
    int64; h_count [B] int64; h_score [B, S] f32; h_len [B, S] int64; h_tokens [B, S, T] int64; last_t [B]
    int64; and the ints P, K. top_s/top_i [B, 2K]: the best 2K of each window's K*V candidate scores, best first
    (top_i = beam * V + token). ns [B]: this step's no-speech probabilities.
    """
    K, P = st["K"], st["P"]
    B = st["pos"].shape[0]
    C = st["src"].shape[1]
    T = st["hist"].shape[1]
    S = st["h_score"].shape[1]
    for b in range(B):
        rows = b * K + np.arange(K)
        tb, pb, db = int(st["t"][b]), int(st["pos"][b]), bool(st["done"][b])
        if pb == int(st["sot_pos"][b]):  # :181-182
            st["no_speech"][b] = ns[b]
        if tb < 0:  # :186-192 -- in the prompt: next prompt token, mark the new slot, advance
            nxt = st["forced"][b, min(P + tb, P)]
            st["tokens"][rows] = nxt
            if 0 <= pb < C:
                st["src"][rows, pb] = rows
            st["pos"][b] = pb + 1
            st["t"][b] = tb + 1
            continue
        if db:  # done windows are left as they are
            continue
        p_i, p_s = top_i[b, :K].astype(np.int64), top_s[b, :K].astype(np.float32)
        s_i, s_s = top_i[b, K:2 * K].astype(np.int64), top_s[b, K:2 * K].astype(np.float32)
        tok, par = p_i % V, p_i // V  # :226
        s_tok, s_par = s_i % V, s_i // V
        eos = tok == EOT
        last = tb == int(st["last_t"][b])
        finish = eos | last  # :230
        slot = int(st["h_count"][b]) + np.cumsum(finish.astype(np.int64)) - 1
        sec_ok = s_tok != EOT  # :233-240 -- each ended candidate's place: the r-th secondary that does not end
        sec_rank = np.cumsum(sec_ok.astype(np.int64)) - 1
        r = np.cumsum(eos.astype(np.int64)) - 1
        take = eos & (r < sec_ok.sum())
        new_tok, new_par, new_s = tok.copy(), par.copy(), p_s.copy()
        for k in range(K):
            if take[k]:
                j = int(np.nonzero(sec_ok & (sec_rank == r[k]))[0][0])
                new_tok[k], new_par[k], new_s[k] = s_tok[j], s_par[j], s_s[j]
        # every read of the window's state before any write (:241-249)
        par_hist = st["hist"][b * K + par].copy()
        new_hist = st["hist"][b * K + new_par].copy()
        new_src = st["src"][b * K + new_par].copy()
        if 0 <= pb < C:
            new_src[:, pb] = (b * K + new_par).astype(np.int32)
        # finished hypotheses (:250-258): EOS not part of them; at the last step the token is
        with_tok = ~eos
        for k in range(K):
            if finish[k]:
                h_row = par_hist[k].copy()
                if with_tok[k] and 0 <= tb < T:
                    h_row[tb] = tok[k]
                st["h_tokens"][b, slot[k]] = h_row
                st["h_score"][b, slot[k]] = p_s[k]
                st["h_len"][b, slot[k]] = tb + int(with_tok[k])
        count = int(st["h_count"][b]) + int(finish.sum())
        st["h_count"][b] = count
        # the new beams (:259-264)
        if 0 <= tb < T:
            new_hist[:, tb] = new_tok
        st["hist"][rows] = new_hist
        st["cum"][rows] = new_s
        st["tokens"][rows] = new_tok
        st["src"][rows] = new_src
        ended = count >= K or last  # :265-269
        st["done"][b] = ended
        if not ended:
            st["pos"][b] = pb + 1
            st["t"][b] = tb + 1
    assert S >= 1


LOWEST = np.float32(np.finfo(np.float32).min)


def beam_scores(logits: np.ndarray, suppress: np.ndarray, begin: np.ndarray, t: np.ndarray, cum: np.ndarray,
                hist: np.ndarray, max_initial: int, K: int, timestamps: bool, no_speech: int, no_timestamps: int,
                ts_begin: int, eot: int):
    """The candidate scores of a beam step: search.py:283-289 ``_choose`` (suppressed tokens, at a window's first
    step the begin-suppressed ones, set to the lowest float), with ``timestamps`` search.py:313-338
    ``_timestamp_rules`` (CTranslate2's ApplyTimestampRules), log-softmax, plus the row's cumulative
    log-probability (search.py:370); and each window's no-speech probability from its first row's raw logits
    (search.py:259-260). The fused form of the same is beam_kernels.py:36-135 ``_scores_kernel``.

    logits [N, V] f32; suppress/begin [V] bool; t [B] int64; cum [N] f32; hist [N, T] int64.
    Returns (scores [N, V] f32, ns [B] f32)."""
    n, v = logits.shape
    x = logits.astype(np.float32).copy()
    B = n // K
    tr = np.repeat(np.asarray(t, dtype=np.int64), K)  # [N]
    first = tr == 0
    x[np.broadcast_to(suppress[None, :], x.shape)] = LOWEST
    x[np.outer(first, begin)] = LOWEST
    if timestamps:
        tb = ts_begin
        ids = np.arange(v)
        g = np.maximum(tr, 0)
        first_ts = g == 0
        rows = np.arange(n)
        last = hist[rows, np.maximum(g - 1, 0)]
        pen = np.where(g >= 2, hist[rows, np.maximum(g - 2, 0)], last)
        last_ts, pen_ts = last >= tb, pen >= tb
        T = hist.shape[1]
        is_ts = (hist >= tb) & (np.arange(T)[None, :] < g[:, None])
        at = np.where(is_ts, np.arange(T)[None, :], -1).max(1)
        latest = hist[rows, np.maximum(at, 0)]
        mask = (ids[None, :] == no_timestamps) | (first_ts[:, None] & ((ids[None, :] < tb)
                                                                        | (ids[None, :] > tb + max_initial)))
        mask |= (~first_ts & last_ts & pen_ts)[:, None] & (ids[None, :] >= tb)
        pair = ~first_ts & last_ts & ~pen_ts
        mask |= pair[:, None] & ((ids[None, :] < eot) | ((ids[None, :] >= tb) & (ids[None, :] < last[:, None])))
        mask |= (~first_ts & ~last_ts & (at >= 0))[:, None] & (ids[None, :] >= tb) & (ids[None, :] <= latest[:, None])
        x[mask] = LOWEST
        lp = _log_softmax(x)
        with np.errstate(divide="ignore"):
            ts_lse = _logsumexp(lp[:, tb:])
        sample_ts = ts_lse > lp[:, :tb].max(-1)
        check = pair | (~first_ts & ~last_ts)
        x[(check & sample_ts)[:, None] & (ids[None, :] < tb)] = LOWEST
    scores = (_log_softmax(x) + np.asarray(cum, dtype=np.float32)[:, None]).astype(np.float32)
    lg = logits[::K].astype(np.float64)
    ns = np.exp(lg[:, no_speech] - _logsumexp(lg)).astype(np.float32)
    assert ns.shape == (B,)
    return scores, ns


def _logsumexp(x: np.ndarray) -> np.ndarray:
    x = x.astype(np.float64)
    m = x.max(-1)
    return m + np.log(np.exp(x - m[:, None]).sum(-1))


def _log_softmax(x: np.ndarray) -> np.ndarray:
    x64 = x.astype(np.float64)
    return (x64 - _logsumexp(x64)[:, None]).astype(np.float32)


def beam_topk(scores: np.ndarray, K: int):
    """The best 2K of each window's K x V candidate scores (search.py:371 ``topk(2 * K)``), best first; equal
    scores in index order. Returns (top_s [B, 2K] f32, top_i [B, 2K] int64 = beam * V + token)."""
    n, v = scores.shape
    flat = scores.reshape(n // K, K * v)
    order = np.lexsort((np.arange(K * v)[None, :].repeat(flat.shape[0], 0), -flat.astype(np.float64)), axis=1)
    top_i = order[:, : 2 * K].astype(np.int64)
    return np.take_along_axis(flat, top_i, 1).astype(np.float32), top_i
