"""The decoder step's linear layers with LayerNorm, bias, GELU and residual fused around them -- the call surface of
the reference's ``whisper_trt.decoder_kernels`` (decoder_kernels.py:127-157: ``layer_norm_bias``, ``ln_linear``,
``linear_residual``), on this package's sm_100a kernels through the C ABI (``wt_layer_norm_bias``,
``wt_ln_linear``, ``wt_linear_residual``).

Numerics as the reference states them: fp32 LayerNorm statistics (the normalized row rounded to the input type),
fp32 accumulation, the GEMM's result rounded before the GELU (computed in fp32) or the residual addition. Tensors:
contiguous CUDA tensors of one 16-bit type (fp16 as the reference; bf16 too); ``w`` in nn.Linear layout [out, in].
There is no CPU path: without the library every call raises.
"""

from __future__ import annotations

import torch

from . import _lib
from .attn_plugin import _cuda, _dtype_code, _stream, _workspace


def _check_linear(what: str, x: torch.Tensor, w: torch.Tensor, b: torch.Tensor) -> tuple[int, int, int]:
    if x.dim() != 2 or w.dim() != 2 or b.dim() != 1:
        raise ValueError(f"{what}: x must be [M, K], w [N, K], b [N]")
    m, k = x.shape
    n = w.shape[0]
    if w.shape[1] != k or b.shape[0] != n:
        raise ValueError(f"{what}: w {tuple(w.shape)} / b {tuple(b.shape)} do not match x {tuple(x.shape)}")
    if w.dtype != x.dtype or b.dtype != x.dtype:
        raise TypeError(f"{what}: x, w and b must have one dtype")
    return m, n, k


def layer_norm_bias(x: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, bias: torch.Tensor,
                    eps: float = 1e-5) -> torch.Tensor:
    """``LN(x)`` [M, K] (fp32 statistics, rounded to x's type), and ``x += bias`` in place (after reading it).
    Reference: decoder_kernels.py:127-135 (kernel :100-115)."""
    what = "layer_norm_bias"
    if x.dim() != 2:
        raise ValueError(f"{what}: x must be [M, K]")
    m, k = x.shape
    for name, t in (("gamma", gamma), ("beta", beta), ("bias", bias)):
        if t.shape != (k,) or t.dtype != x.dtype:
            raise ValueError(f"{what}: {name} must be [{k}] of x's dtype")
    code = _dtype_code(x, what)
    dev = _cuda(what, x, gamma, beta, bias)
    y = torch.empty_like(x)
    with torch.cuda.device(dev):
        st = _lib.load().wt_layer_norm_bias(code, x.data_ptr(), gamma.data_ptr(), beta.data_ptr(), bias.data_ptr(),
                                            y.data_ptr(), m, k, float(eps), _stream(dev))
    _lib.check(st, what)
    return y


def ln_linear(x: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, w: torch.Tensor, b: torch.Tensor,
              gelu: bool = False, eps: float = 1e-5, out: torch.Tensor | None = None) -> torch.Tensor:
    """``LN(x) @ w^T + b`` (GELU'd if ``gelu``): x [M, K], w [N, K] -> [M, N] of x's type.
    Reference: decoder_kernels.py:138-146 (kernel :42-75)."""
    what = "ln_linear"
    m, n, k = _check_linear(what, x, w, b)
    for name, t in (("gamma", gamma), ("beta", beta)):
        if t.shape != (k,) or t.dtype != x.dtype:
            raise ValueError(f"{what}: {name} must be [{k}] of x's dtype")
    code = _dtype_code(x, what)
    dev = _cuda(what, x, gamma, beta, w, b)
    y = torch.empty(m, n, dtype=x.dtype, device=x.device) if out is None else out
    if y.shape != (m, n) or y.dtype != x.dtype or not y.is_contiguous():
        raise ValueError(f"{what}: out must be a contiguous [{m}, {n}] tensor of x's dtype")
    lib = _lib.load()
    nbytes = int(lib.wt_dec_linear_workspace(m, n, k, 1))
    ws = _workspace(dev, "dec_linear", (m, n, k, 1), nbytes)
    with torch.cuda.device(dev):
        st = lib.wt_ln_linear(code, x.data_ptr(), gamma.data_ptr(), beta.data_ptr(), w.data_ptr(), b.data_ptr(),
                              y.data_ptr(), m, n, k, int(bool(gelu)), float(eps), ws.data_ptr(), ws.numel(),
                              _stream(dev))
    _lib.check(st, what)
    return y


def linear_residual(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor, res: torch.Tensor,
                    out: torch.Tensor | None = None) -> torch.Tensor:
    """``res + (x @ w^T + b)``: x [M, K], w [N, K], res [M, N] -> [M, N] (``out`` may be ``res``).
    Reference: decoder_kernels.py:149-157 (kernel :77-97)."""
    what = "linear_residual"
    m, n, k = _check_linear(what, x, w, b)
    if res.shape != (m, n) or res.dtype != x.dtype:
        raise ValueError(f"{what}: res must be [{m}, {n}] of x's dtype")
    code = _dtype_code(x, what)
    dev = _cuda(what, x, w, b, res)
    y = torch.empty_like(res) if out is None else out
    if y.shape != (m, n) or y.dtype != x.dtype or not y.is_contiguous():
        raise ValueError(f"{what}: out must be a contiguous [{m}, {n}] tensor of x's dtype")
    lib = _lib.load()
    nbytes = int(lib.wt_dec_linear_workspace(m, n, k, 0))
    ws = _workspace(dev, "dec_linear", (m, n, k, 0), nbytes)
    with torch.cuda.device(dev):
        st = lib.wt_linear_residual(code, x.data_ptr(), w.data_ptr(), b.data_ptr(), res.data_ptr(), y.data_ptr(), m,
                                    n, k, ws.data_ptr(), ws.numel(), _stream(dev))
    _lib.check(st, what)
    return y


def install(module) -> None:
    """Route a reference ``whisper_trt.decoder_kernels`` module's launchers to these kernels (in place), so that its
    callers -- ``TritonDecoderBackend.step_fn``'s ``run`` and ``run_cublas`` (runtime.py:134-167) -- run on them
    unchanged. The module's other names (its Triton kernels, ``triton``) are left as they are."""
    for name in ("layer_norm_bias", "ln_linear", "linear_residual"):
        setattr(module, name, globals()[name])
