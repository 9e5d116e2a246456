"""CPU restatement (numpy) of the reference decoder attention ops -- TEST INFRASTRUCTURE ONLY.

This module is the parity checker for the CUDA kernels of ``whisper_trt_b200``. Only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it;
the product path never calls it and has no CPU fallback.

Every function restates the PyTorch reference body of the same name in the reference project's
``src/whisper_trt/attn_plugin.py`` (the op bodies the reference runs on CPU tensors, ``RUNTIME_TRITON=False``).
All arithmetic is float32, as the reference's ``.float()`` upcasts; outputs are float32 (callers round to the
input dtype when they want the op's exact return type). Layouts:

* qkv ``[B, S, 3*H*D]`` -- queries, keys, values, heads in order
* k/v caches ``[B, H, C, D]``; ``offset`` ``[B]`` int64; ``src`` ``[B, C]`` int32 (the row holding each slot)
* cross queries ``[W, S, H*D]``, cross keys/values ``[W, H, T, D]``
* split partials ``[W, H, SPLITS, S, D + 2]`` float32 = (unnormalised output, running max in log2 units, sum)

Pinned against the reference's own outputs by ``tests/golden/make_golden.py`` (fixtures in ``tests/golden/``).
"""

from __future__ import annotations

import math

import numpy as np

SPLITS = 8  # attn_plugin.py:51 -- key slices of the split cross-attention
LOG2E = math.log2(math.e)


def qk_scale(d: int) -> float:
    """attn_plugin.py:458-459 ``_qk_scale``: d^-1/2 * log2(e) (scores in log2 units)."""
    return d**-0.5 * LOG2E


def _f32(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, dtype=np.float32)


def merge_heads(x: np.ndarray) -> np.ndarray:
    """attn_plugin.py:88-89 ``_merge``: [B, H, S, D] -> [B, S, H*D]."""
    b, h, s, d = x.shape
    return np.ascontiguousarray(x.transpose(0, 2, 1, 3)).reshape(b, s, h * d)


def gather_cache(cache: np.ndarray, src: np.ndarray) -> np.ndarray:
    """attn_plugin.py:92-99: the cache [B, H, C, D] as each row sees it -- slot j of row b comes from row
    src[b, j]. Integer indexing only: bit-exact."""
    b, h, c, d = cache.shape
    rows = np.asarray(src, dtype=np.int64)  # [B, C]
    slots = np.arange(c)
    # out[b, h, j, :] = cache[rows[b, j], h, j, :]
    return cache[rows[:, None, :], np.arange(h)[None, :, None], slots[None, None, :], :]


def _softmax_lastdim(x: np.ndarray) -> np.ndarray:
    m = x.max(-1, keepdims=True)
    e = np.exp(x - m, dtype=np.float32)
    return e / e.sum(-1, keepdims=True)


def self_attn(qkv: np.ndarray, k_cache: np.ndarray, v_cache: np.ndarray, offset: np.ndarray,
              src: np.ndarray) -> np.ndarray:
    """attn_plugin.py:102-121 ``self_attn`` (reference body): S new tokens per row over [cache slots <
    offset[b] read through ``src`` | the new tokens, causal]. Returns float32 [B, S, H*D]."""
    b, s, _ = qkv.shape
    h, c, d = k_cache.shape[1:]
    kc = _f32(gather_cache(k_cache, src))
    vc = _f32(gather_cache(v_cache, src))
    qkv5 = _f32(qkv).reshape(b, s, 3, h, d).transpose(2, 0, 3, 1, 4)  # [3, B, H, S, D]
    q, k, v = qkv5[0], qkv5[1], qkv5[2]
    new = np.arange(s)
    cache_ok = np.arange(c)[None, :] < np.asarray(offset, dtype=np.int64)[:, None]  # [B, C]
    mask = np.concatenate([np.broadcast_to(cache_ok[:, None, None, :], (b, 1, s, c)),
                           np.broadcast_to((new[None, :] <= new[:, None])[None, None], (b, 1, s, s))], -1)
    keys = np.concatenate([kc, k], 2)  # [B, H, C+S, D]
    vals = np.concatenate([vc, v], 2)
    scores = (q * np.float32(d**-0.5)) @ keys.transpose(0, 1, 3, 2)  # [B, H, S, C+S]
    scores = np.where(mask, scores, np.float32(-np.inf))
    p = _softmax_lastdim(scores)
    return merge_heads(p @ vals)


def self_attn_step(qkv: np.ndarray, k_cache: np.ndarray, v_cache: np.ndarray, offset: np.ndarray,
                   src: np.ndarray, write_cache: bool = False) -> np.ndarray:
    """attn_plugin.py:309-350 / :488-501 ``self_attn_step_triton`` semantics on the CPU: one new token per row.

    The offset is clamped to [0, C] and each ``src`` entry to [0, B-1] (:321, :338-339). With ``write_cache`` the
    new key/value go into the row's own slot ``offset`` (when < C) of ``k_cache``/``v_cache`` IN PLACE (:327-330);
    the attention itself is unchanged because rows only read slots below their offset. Returns float32 [B, 1, H*D].
    """
    b, s, _ = qkv.shape
    if s != 1:
        raise ValueError("one new token per row")
    h, c, d = k_cache.shape[1:]
    off = np.clip(np.asarray(offset, dtype=np.int64), 0, c)
    rows = np.clip(np.asarray(src, dtype=np.int64), 0, b - 1)
    out = self_attn(qkv, k_cache, v_cache, off, rows)
    if write_cache:
        cache_append(k_cache, v_cache, qkv, off)
    return out


def cache_append(k_cache: np.ndarray, v_cache: np.ndarray, qkv: np.ndarray, offset: np.ndarray) -> None:
    """The append of a decoding step, in place: row b's new key/value (qkv[b, 0, H*D:2*H*D], [2*H*D:]) into its own
    cache slot offset[b] when that is < C. attn_plugin.py:327-330 (``WRITE``), the same as the scatter of
    search.py:249-250 for one token. Bit-exact (copies)."""
    b = qkv.shape[0]
    h, c, d = k_cache.shape[1:]
    hd = h * d
    for r in range(b):
        o = int(offset[r])
        if 0 <= o < c:
            k_cache[r, :, o, :] = qkv[r, 0, hd:2 * hd].reshape(h, d)
            v_cache[r, :, o, :] = qkv[r, 0, 2 * hd:3 * hd].reshape(h, d)


def cross_attn(q: np.ndarray, k: np.ndarray, v: np.ndarray) -> np.ndarray:
    """attn_plugin.py:129-136 ``cross_attn``: q [W, S, H*D] over k/v [W, H, T, D] -> float32 [W, S, H*D]."""
    w, s, _ = q.shape
    h, d = k.shape[1], k.shape[3]
    qh = _f32(q).reshape(w, s, h, d).transpose(0, 2, 1, 3)  # [W, H, S, D]
    scores = (qh * np.float32(d**-0.5)) @ _f32(k).transpose(0, 1, 3, 2)
    return merge_heads(_softmax_lastdim(scores) @ _f32(v))


def log2_scores(q: np.ndarray, k: np.ndarray) -> np.ndarray:
    """attn_plugin.py:144-148 ``_log2_scores``: [W, H, S, T] scores in log2 units."""
    w, s, _ = q.shape
    h, d = k.shape[1], k.shape[3]
    qh = _f32(q).reshape(w, s, h, d).transpose(0, 2, 1, 3)
    return (qh @ _f32(k).transpose(0, 1, 3, 2)) * np.float32(qk_scale(d))


def cross_attn_split(q: np.ndarray, k: np.ndarray, v: np.ndarray, splits: int = SPLITS) -> np.ndarray:
    """attn_plugin.py:151-174 ``cross_attn_split``: per key slice i of chunk = ceil(T / splits): m = max score,
    p = exp2(s - m), acc = p @ v, l = sum(p); an empty slice has m = -inf, acc = l = 0.
    Returns float32 [W, H, splits, S, D + 2]."""
    w, s, _ = q.shape
    h, t, d = k.shape[1:]
    scores = log2_scores(q, k)
    chunk = -(-t // splits)
    out = np.zeros((w, h, splits, s, d + 2), dtype=np.float32)
    vf = _f32(v)
    for i in range(splits):
        lo, hi = i * chunk, min((i + 1) * chunk, t)
        if lo >= hi:
            out[:, :, i, :, d] = -np.inf
            continue
        sc = scores[..., lo:hi]
        m = sc.max(-1, keepdims=True)
        p = np.exp2(sc - m, dtype=np.float32)
        out[:, :, i, :, :d] = p @ vf[:, :, lo:hi]
        out[:, :, i, :, d] = m[..., 0]
        out[:, :, i, :, d + 1] = p.sum(-1)
    return out


def cross_attn_combine(part: np.ndarray) -> np.ndarray:
    """attn_plugin.py:182-194 ``cross_attn_combine``: top = max_i m_i, w_i = exp2(m_i - top) (0 for slices
    without keys), out = sum_i w_i acc_i / sum_i w_i l_i -> float32 [W, S, H*D]."""
    part = _f32(part)
    d = part.shape[-1] - 2
    m = part[..., d]  # [W, H, splits, S]
    top = m.max(2, keepdims=True)
    with np.errstate(invalid="ignore"):
        wgt = np.exp2(m - top, dtype=np.float32)
    wgt = np.where(np.isneginf(m), np.float32(0.0), wgt)
    num = (wgt[..., None] * part[..., :d]).sum(2)  # [W, H, S, D]
    den = (wgt * part[..., d + 1]).sum(2)
    return merge_heads(num / den[..., None])
