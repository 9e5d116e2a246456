"""The decoder-attention plugin surface of whisper-trt, on hand-written sm_100a CUDA kernels.

A drop-in for the launchers of the reference's ``src/whisper_trt/attn_plugin.py``: same function names, argument
meanings, tensor layouts, return shapes and error behaviour, so ``TritonDecoderBackend.step_fn``
(reference runtime.py:134-151) runs unchanged on them -- call :func:`install` on the reference module, or import
the names from here. Every call goes through the C ABI of ``libwhisper_attn_b200.so`` (``include/whisper_attn_b200.h``)
on torch's current CUDA stream; there is no Triton, no CPU path and no fallback: CPU tensors, unsupported dtypes
or a missing library raise.

Layouts (all contiguous): qkv [N, S, 3*H*D] (q | k | v, heads in order), k/v cache [N, H, C, D] (one layer),
offset [N] int64, src [N, C] int32 (the row holding each slot), cross q [W, S, H*D], cross k/v [W, H, T, D],
part [W, H, SPLITS, S, D + 2] float32. fp16 or bf16.

Everything is CUDA-graph capturable (no host synchronisation, no host reads of device data); the kernels that
combine partials in-kernel use a per-device workspace that is allocated (zeroed) on first use outside capture --
run each shape once before capturing it, as the reference's own capture does (search.py:674-685).
"""

from __future__ import annotations

import functools
import math

import torch

from . import _lib

NAMESPACE = "whisper_trt_b200"
SPLITS = 8  # key slices of the split cross-attention, as the reference's (attn_plugin.py:51)
# The reference's Triton tactics (attn_plugin.py:41-46) are accepted as ``config`` arguments for call-compatibility;
# these kernels pick their own launch shapes (one CTA per (row, head[, split]) / (window, head, slice)).
TACTICS = {
    "self_attn": [(16, 64, 4, 2)],
    "cross_attn": [(16, 64, 4, 2)],
    "cross_split": [(16, 64, 4, 2)],
    "cross_combine": [(16, 0, 4, 1)],
}
RUNTIME_TRITON = False  # (reference flag; the ops here never run Triton)

_DTYPES = {torch.float16: _lib.WT_F16, torch.bfloat16: _lib.WT_BF16}
_workspaces: dict[tuple, torch.Tensor] = {}


def _dtype_code(t: torch.Tensor, what: str) -> int:
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise TypeError(f"{what}: {t.dtype} is not supported (float16 or bfloat16)") from None


def _cuda(what: str, *ts: torch.Tensor) -> torch.device:
    dev = ts[0].device
    for t in ts:
        if not t.is_cuda:
            raise ValueError(f"{what}: CUDA tensors only (got a {t.device} tensor; there is no CPU path)")
        if t.device != dev:
            raise ValueError(f"{what}: tensors on different devices ({dev}, {t.device})")
        if not t.is_contiguous():
            raise ValueError(f"{what}: tensors must be contiguous")
    return dev


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _workspace(dev: torch.device, kind: str, shape: tuple, nbytes: int) -> torch.Tensor:
    """The zeroed workspace of one call shape on one device. A workspace holds the in-kernel combine's counters
    (the kernels leave them zeroed) and its partials (left as written), laid out by the shape: a workspace used by
    one shape is not valid for another, so each shape keeps its own."""
    key = (dev.index if dev.index is not None else torch.cuda.current_device(), kind, shape)
    ws = _workspaces.get(key)
    if ws is None or ws.numel() < nbytes:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError(f"{kind} workspace of {nbytes} bytes needed during CUDA-graph capture: run the call "
                               "once before capturing (as warm-up does)")
        ws = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=dev)
        _workspaces[key] = ws
    return ws


def workspace_errors() -> int:
    """The device error words of this process's cross-attention, logits and decoder-linear workspaces, OR-ed (0: no
    kernel gave up a wait).
    Reads device memory: synchronises."""
    err = 0
    for (dev, kind, shape), ws in _workspaces.items():
        if kind in ("cross", "logits", "dec_linear"):
            err |= int(ws[:4].view(torch.int32).item())
    return err


def _qk_scale(d: int) -> float:
    return d**-0.5 * math.log2(math.e)


# --- self-attention ----------------------------------------------------------------------------------------
def self_attn_step_config(rows: int, heads: int = 20, capacity: int = 448, head_dim: int = 64) -> tuple[int, int]:
    """(key splits per (row, head), warps per CTA) this build launches for ``rows`` rows -- the counterpart of the
    reference's (keys per block, warps) choice (attn_plugin.py:482-485). A CTA's 4 warps split its keys."""
    return int(_lib.load().wt_self_attn_step_splits(rows, heads, capacity, head_dim)), 4


def self_attn_step_triton(qkv: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, offset: torch.Tensor,
                          src: torch.Tensor, config=None, write_cache: bool = False, *, kv_splits: int | None = None,
                          out: torch.Tensor | None = None, shared_prefix_group: int | None = None,
                          min_shared: int = 32) -> torch.Tensor:
    """Self-attention of one new token per row (qkv [N, 1, 3*H*D]) over its cache slots < offset, read through
    ``src``, and the new token -> [N, 1, H*D] in qkv's dtype. ``write_cache``: the new keys/values also go into the
    caches at ``offset`` (in place). Reference: attn_plugin.py:488-501 (kernel :309-350).

    ``config`` is accepted for call-compatibility and ignored; ``kv_splits`` (None: chosen from the shape) splits
    every row's cache into that many parts (at least ceil(C / 1024)). ``shared_prefix_group`` (an addition: the
    rows per window, 1-8): the rows of each group of that many consecutive rows that share at least ``min_shared``
    leading slot-table entries with the group's first row have those keys attended once for the whole group
    (``wt_self_attn_step_prefix``); the result is the same attention. Head dim 64, C <= 1024, no key splits."""
    what = "self_attn_step"
    if qkv.dim() != 3:
        raise ValueError(f"{what}: qkv must be [N, S, 3*H*D]")
    n, s, _ = qkv.shape
    if s != 1:
        raise ValueError("one new token per row")
    if k_cache.dim() != 4 or v_cache.shape != k_cache.shape:
        raise ValueError(f"{what}: k_cache/v_cache must be [N, H, C, D] of the same shape")
    h, c, d = k_cache.shape[1:]
    if k_cache.shape[0] != n or qkv.shape[2] != 3 * h * d:
        raise ValueError(f"{what}: qkv {tuple(qkv.shape)} does not match the cache {tuple(k_cache.shape)}")
    if offset.shape != (n,) or offset.dtype != torch.int64:
        raise ValueError(f"{what}: offset must be [N] int64")
    if src.shape != (n, c) or src.dtype != torch.int32:
        raise ValueError(f"{what}: src must be [N, C] int32")
    code = _dtype_code(qkv, what)
    if k_cache.dtype != qkv.dtype or v_cache.dtype != qkv.dtype:
        raise TypeError(f"{what}: the caches must have qkv's dtype")
    dev = _cuda(what, qkv, k_cache, v_cache, offset, src)
    y = qkv.new_empty(n, 1, h * d) if out is None else out
    if y.shape != (n, 1, h * d) or y.dtype != qkv.dtype:
        raise ValueError(f"{what}: out must be [N, 1, H*D] of qkv's dtype")
    lib = _lib.load()
    if shared_prefix_group:
        if kv_splits not in (None, 1):
            raise ValueError(f"{what}: shared_prefix_group takes no key splits")
        ws_bytes = int(lib.wt_self_attn_step_prefix_workspace(n, h, d))
        ws = _workspace(dev, "self_prefix", (n, h, d), ws_bytes)
        with torch.cuda.device(dev):
            st = lib.wt_self_attn_step_prefix(code, qkv.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                                              offset.data_ptr(), src.data_ptr(), y.data_ptr(), n, h, c, d,
                                              int(bool(write_cache)), int(shared_prefix_group), int(min_shared),
                                              ws.data_ptr(), ws_bytes, _stream(dev))
        _lib.check(st, what)
        return y
    splits = int(kv_splits) if kv_splits else int(lib.wt_self_attn_step_splits(n, h, c, d))
    splits = max(splits, -(-c // 1024))  # (at most 1024 cache slots per split)
    ws_ptr, ws_bytes = None, 0
    if splits > 1:
        ws_bytes = int(lib.wt_self_attn_step_workspace(n, h, d, splits))
        ws_ptr = _workspace(dev, "self", (n, h, d, splits), ws_bytes).data_ptr()
    with torch.cuda.device(dev):
        st = lib.wt_self_attn_step(code, qkv.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), offset.data_ptr(),
                                   src.data_ptr(), y.data_ptr(), n, h, c, d, int(bool(write_cache)), splits, ws_ptr,
                                   ws_bytes, _stream(dev))
    _lib.check(st, what)
    return y


def self_attn_triton(qkv: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, offset: torch.Tensor,
                     src: torch.Tensor, config=None, *, out: torch.Tensor | None = None) -> torch.Tensor:
    """Self-attention of S new tokens per row (qkv [N, S, 3*H*D], a prompt) over the row's cache slots < offset,
    read through ``src``, and causally over the new tokens -> [N, S, H*D] in qkv's dtype. The caches are only read
    (the caller stores the new keys/values). Reference: attn_plugin.py:462-479 (kernel :275-307, op :102-121).

    ``config`` is accepted for call-compatibility and ignored (64 queries per CTA; one new token per row goes to
    the decode-step kernel, which computes the same op)."""
    what = "self_attn"
    if qkv.dim() != 3:
        raise ValueError(f"{what}: qkv must be [N, S, 3*H*D]")
    n, s, _ = qkv.shape
    if k_cache.dim() != 4 or v_cache.shape != k_cache.shape:
        raise ValueError(f"{what}: k_cache/v_cache must be [N, H, C, D] of the same shape")
    h, c, d = k_cache.shape[1:]
    if k_cache.shape[0] != n or qkv.shape[2] != 3 * h * d:
        raise ValueError(f"{what}: qkv {tuple(qkv.shape)} does not match the cache {tuple(k_cache.shape)}")
    if offset.shape != (n,) or offset.dtype != torch.int64:
        raise ValueError(f"{what}: offset must be [N] int64")
    if src.shape != (n, c) or src.dtype != torch.int32:
        raise ValueError(f"{what}: src must be [N, C] int32")
    code = _dtype_code(qkv, what)
    if k_cache.dtype != qkv.dtype or v_cache.dtype != qkv.dtype:
        raise TypeError(f"{what}: the caches must have qkv's dtype")
    dev = _cuda(what, qkv, k_cache, v_cache, offset, src)
    y = qkv.new_empty(n, s, h * d) if out is None else out
    if y.shape != (n, s, h * d) or y.dtype != qkv.dtype:
        raise ValueError(f"{what}: out must be [N, S, H*D] of qkv's dtype")
    if s == 0:
        return y
    if s == 1:  # one new token per row (the reference's gemm="triton" decode step calls this op so): the step kernel
        return self_attn_step_triton(qkv, k_cache, v_cache, offset, src, out=y)
    with torch.cuda.device(dev):
        st = _lib.load().wt_self_attn(code, qkv.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), offset.data_ptr(),
                                      src.data_ptr(), y.data_ptr(), n, s, h, c, d, _stream(dev))
    _lib.check(st, what)
    return y


def cache_append(qkv: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, offset: torch.Tensor) -> None:
    """Row r's new key/value (from qkv [N, 1, 3*H*D]) into its own cache slot offset[r] (if < C), in place: the
    scatter of the reference's search.py:249-250 for one layer (the append of attn_plugin.py:327-330 alone)."""
    what = "cache_append"
    n = qkv.shape[0]
    h, c, d = k_cache.shape[1:]
    if qkv.shape != (n, 1, 3 * h * d) or k_cache.shape[0] != n or v_cache.shape != k_cache.shape:
        raise ValueError(f"{what}: shapes do not match")
    if offset.shape != (n,) or offset.dtype != torch.int64:
        raise ValueError(f"{what}: offset must be [N] int64")
    code = _dtype_code(qkv, what)
    dev = _cuda(what, qkv, k_cache, v_cache, offset)
    with torch.cuda.device(dev):
        st = _lib.load().wt_cache_append(code, qkv.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                                         offset.data_ptr(), n, h, c, d, _stream(dev))
    _lib.check(st, what)


def gather_cache(cache: torch.Tensor, src: torch.Tensor) -> torch.Tensor:
    """The cache [N, H, C, D] as each row sees it: slot j of row r from row src[r, j] (reference
    attn_plugin.py:92-99), materialised on the GPU (bit-exact copies)."""
    what = "gather_cache"
    n, h, c, d = cache.shape
    if src.shape != (n, c) or src.dtype != torch.int32:
        raise ValueError(f"{what}: src must be [N, C] int32")
    code = _dtype_code(cache, what)
    dev = _cuda(what, cache, src)
    out = torch.empty_like(cache)
    with torch.cuda.device(dev):
        st = _lib.load().wt_gather_cache(code, cache.data_ptr(), src.data_ptr(), out.data_ptr(), n, h, c, d,
                                         _stream(dev))
    _lib.check(st, what)
    return out


# --- cross-attention ---------------------------------------------------------------------------------------
def _check_cross(what: str, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor):
    if q.dim() != 3 or k.dim() != 4 or v.shape != k.shape:
        raise ValueError(f"{what}: q must be [W, S, H*D] and k/v [W, H, T, D] of the same shape")
    w, s, hd = q.shape
    _, h, t, d = k.shape
    if k.shape[0] != w or hd != h * d:
        raise ValueError(f"{what}: q {tuple(q.shape)} does not match k/v {tuple(k.shape)}")
    code = _dtype_code(q, what)
    if k.dtype != q.dtype or v.dtype != q.dtype:
        raise TypeError(f"{what}: q, k, v must have the same dtype")
    dev = _cuda(what, q, k, v)
    return w, s, h, t, d, code, dev


def cross_attn_split_triton(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, config=None, *,
                            splits: int = SPLITS, out: torch.Tensor | None = None) -> torch.Tensor:
    """Partial attention of q [W, S, H*D] over ``splits`` slices (chunk = ceil(T / splits)) of k/v [W, H, T, D]:
    per slice the unnormalised output, the maximum score (log2 units) and the sum of exponentials ->
    [W, H, splits, S, D + 2] float32. Reference: attn_plugin.py:521-534 (kernel :378-409). Runs on the stream-K TMA
    kernel of :func:`cross_attn_triton` with the (window, head, slice) triples as its units (a per-device
    workspace per shape, as that function's), or, for shapes it does not take, on the per-slice kernel."""
    what = "cross_attn_split"
    w, s, h, t, d, code, dev = _check_cross(what, q, k, v)
    part = q.new_empty(w, h, splits, s, d + 2, dtype=torch.float32) if out is None else out
    if part.shape != (w, h, splits, s, d + 2) or part.dtype != torch.float32:
        raise ValueError(f"{what}: out must be [W, H, splits, S, D+2] float32")
    lib = _lib.load()
    nbytes = int(lib.wt_cross_attn_split_workspace(w, s, h, t, d, splits))  # (0: the per-slice kernel, no workspace)
    ws = _workspace(dev, "cross", (w, s, h, t, d, splits), nbytes).data_ptr() if nbytes else None
    with torch.cuda.device(dev):
        st = lib.wt_cross_attn_split_ws(code, q.data_ptr(), k.data_ptr(), v.data_ptr(), part.data_ptr(), w, s, h, t, d,
                                        splits, ws, nbytes, _stream(dev))
    _lib.check(st, what)
    return part


def cross_attn_combine_triton(part: torch.Tensor, q: torch.Tensor, config=None, *,
                              out: torch.Tensor | None = None) -> torch.Tensor:
    """The slices of :func:`cross_attn_split_triton` combined -> [W, S, H*D] in q's dtype (q only gives the type
    and shape). Reference: attn_plugin.py:537-546 (kernel :411-435)."""
    what = "cross_attn_combine"
    if part.dim() != 5 or part.dtype != torch.float32:
        raise ValueError(f"{what}: part must be [W, H, splits, S, D+2] float32")
    w, h, splits, s, d2 = part.shape
    if q.shape != (w, s, h * (d2 - 2)):
        raise ValueError(f"{what}: q {tuple(q.shape)} does not match part {tuple(part.shape)}")
    code = _dtype_code(q, what)
    dev = _cuda(what, part)
    y = torch.empty_like(q) if out is None else out
    with torch.cuda.device(dev):
        st = _lib.load().wt_cross_attn_combine(code, part.data_ptr(), y.data_ptr(), w, s, h, d2 - 2, splits,
                                               _stream(dev))
    _lib.check(st, what)
    return y


def cross_attn_triton(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, config=None, *,
                      out: torch.Tensor | None = None) -> torch.Tensor:
    """Attention of q [W, S, H*D] to k/v [W, H, T, D] -> [W, S, H*D] in one launch (the split kernel whose last
    CTA per (window, head) combines). Reference: attn_plugin.py:504-518 (kernel :352-376)."""
    what = "cross_attn"
    w, s, h, t, d, code, dev = _check_cross(what, q, k, v)
    y = torch.empty_like(q) if out is None else out
    if y.shape != q.shape or y.dtype != q.dtype:
        raise ValueError(f"{what}: out must be shaped and typed like q")
    lib = _lib.load()
    nbytes = int(lib.wt_cross_attn_workspace(w, s, h, t, d))
    ws = _workspace(dev, "cross", (w, s, h, t, d), nbytes)
    with torch.cuda.device(dev):
        st = lib.wt_cross_attn(code, q.data_ptr(), k.data_ptr(), v.data_ptr(), y.data_ptr(), w, s, h, t, d,
                               ws.data_ptr(), nbytes, _stream(dev))
    _lib.check(st, what)
    return y


# --- vocabulary projection -----------------------------------------------------------------------------------
def logits32_triton(x: torch.Tensor, w: torch.Tensor, config=None, out: torch.Tensor | None = None) -> torch.Tensor:
    """x [B, S, d] (fp16 / bf16) @ w [V, d]^T accumulated and returned in fp32 -> [B, S, V] (into ``out`` if given),
    on the tcgen05 tensor cores. Reference: attn_plugin.py:549-560 (kernel :438-455, op :202-212). ``config`` is
    accepted for call-compatibility and ignored."""
    what = "logits32"
    if x.dim() != 3 or w.dim() != 2 or x.shape[2] != w.shape[1]:
        raise ValueError(f"{what}: x must be [B, S, d] and w [V, d] (got {tuple(x.shape)}, {tuple(w.shape)})")
    b, s, d = x.shape
    v = w.shape[0]
    code = _dtype_code(x, what)
    if w.dtype != x.dtype:
        raise TypeError(f"{what}: x and w must have the same dtype")
    x = x.contiguous()
    dev = _cuda(what, x, w)
    y = torch.empty(b, s, v, dtype=torch.float32, device=dev) if out is None else out
    if y.shape != (b, s, v) or y.dtype != torch.float32 or not y.is_contiguous():
        raise ValueError(f"{what}: out must be a contiguous [B, S, V] float32 tensor")
    if b * s == 0:
        return y
    err = _workspace(dev, "logits", (), 256)
    with torch.cuda.device(dev):
        st = _lib.load().wt_logits32(code, x.data_ptr(), w.data_ptr(), y.data_ptr(), b * s, v, d, err.data_ptr(),
                                     _stream(dev))
    _lib.check(st, what)
    return y


# --- torch custom ops (graph-capturable, with fake kernels for tracing) ------------------------------------
@torch.library.custom_op(f"{NAMESPACE}::logits32", mutates_args=())
def logits32(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """x [B, S, d] @ w [V, d]^T in fp32 (reference op ``whisper_trt::logits32``, attn_plugin.py:202-212)."""
    return logits32_triton(x, w)


@logits32.register_fake
def _(x, w):
    return x.new_empty(x.shape[0], x.shape[1], w.shape[0], dtype=torch.float32)


@torch.library.custom_op(f"{NAMESPACE}::self_attn", mutates_args=())
def self_attn(qkv: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, offset: torch.Tensor,
              src: torch.Tensor) -> torch.Tensor:
    """Self-attention of S new tokens per row through the slot table (reference op ``whisper_trt::self_attn``,
    attn_plugin.py:102-121): the one-token step kernel for S = 1, the prompt kernel otherwise."""
    if qkv.shape[1] == 1:
        return self_attn_step_triton(qkv, k_cache, v_cache, offset, src)
    return self_attn_triton(qkv, k_cache, v_cache, offset, src)


@self_attn.register_fake
def _(qkv, k_cache, v_cache, offset, src):
    return qkv.new_empty(qkv.shape[0], qkv.shape[1], k_cache.shape[1] * k_cache.shape[3])


@torch.library.custom_op(f"{NAMESPACE}::self_attn_step", mutates_args=())
def self_attn_step(qkv: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, offset: torch.Tensor,
                   src: torch.Tensor) -> torch.Tensor:
    """Decode-step self-attention through the slot table (no cache write)."""
    return self_attn_step_triton(qkv, k_cache, v_cache, offset, src)


@self_attn_step.register_fake
def _(qkv, k_cache, v_cache, offset, src):
    return qkv.new_empty(qkv.shape[0], 1, k_cache.shape[1] * k_cache.shape[3])


@torch.library.custom_op(f"{NAMESPACE}::self_attn_step_append", mutates_args=("k_cache", "v_cache"))
def self_attn_step_append(qkv: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, offset: torch.Tensor,
                          src: torch.Tensor) -> torch.Tensor:
    """Decode-step self-attention that also appends the new keys/values at ``offset``."""
    return self_attn_step_triton(qkv, k_cache, v_cache, offset, src, write_cache=True)


@self_attn_step_append.register_fake
def _(qkv, k_cache, v_cache, offset, src):
    return qkv.new_empty(qkv.shape[0], 1, k_cache.shape[1] * k_cache.shape[3])


@torch.library.custom_op(f"{NAMESPACE}::cross_attn", mutates_args=())
def cross_attn(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    return cross_attn_triton(q, k, v)


@cross_attn.register_fake
def _(q, k, v):
    return torch.empty_like(q)


@torch.library.custom_op(f"{NAMESPACE}::cross_attn_split", mutates_args=())
def cross_attn_split(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    return cross_attn_split_triton(q, k, v)


@cross_attn_split.register_fake
def _(q, k, v):
    return q.new_empty(q.shape[0], k.shape[1], SPLITS, q.shape[1], k.shape[3] + 2, dtype=torch.float32)


@torch.library.custom_op(f"{NAMESPACE}::cross_attn_combine", mutates_args=())
def cross_attn_combine(part: torch.Tensor, q: torch.Tensor) -> torch.Tensor:
    return cross_attn_combine_triton(part, q)


@cross_attn_combine.register_fake
def _(part, q):
    return torch.empty_like(q)


def install(module, shared_prefix_group: int | None = None) -> None:
    """Route a reference ``whisper_trt.attn_plugin`` module's launchers to these kernels (in place), so its callers
    -- ``TritonDecoderBackend.step_fn`` (runtime.py:134-151) among them -- run on them unchanged.
    ``shared_prefix_group`` (the caller's rows per window, e.g. its beam or sample count): the decode-step
    self-attention then attends the keys a window's rows share through the slot table once per window."""
    for name in ("self_attn_triton", "self_attn_step_triton", "cross_attn_split_triton",
                 "cross_attn_combine_triton", "cross_attn_triton", "self_attn_step_config", "logits32_triton"):
        setattr(module, name, globals()[name])
    if shared_prefix_group:
        module.self_attn_step_triton = functools.partial(self_attn_step_triton, shared_prefix_group=shared_prefix_group)
