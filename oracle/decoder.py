"""CPU restatement (numpy) of the reference's fused decoder linear layers -- TEST INFRASTRUCTURE ONLY.

The parity checker for ``whisper_trt_b200.decoder_kernels`` (the C ABI's ``wt_layer_norm_bias``, ``wt_ln_linear``,
``wt_linear_residual``). Only ``tests/`` and ``__graft_entry__.smoke()`` may import it; the product path never
calls it and has no CPU fallback.

Each function restates the reference function of the same name in ``src/whisper_trt/decoder_kernels.py``, with the
rounding points its docstring and kernels state (decoder_kernels.py:1-15, :42-115):

* LayerNorm: fp32 statistics -- the mean, then the mean of (x - mean)^2 -- rstd = 1 / sqrt(var + eps), the
  normalized row ``(x - mean) * rstd * gamma + beta`` rounded to the 16-bit type (``modeling.LayerNorm`` with
  ``Precision.ln32``: the row in fp32, rounded at the end);
* GEMM: fp32 accumulation of the 16-bit operands, plus the bias in fp32, rounded to the 16-bit type;
* GELU (``Precision.gelu32``): on the rounded GEMM result, in fp32 (erf form), rounded;
* residual: the rounded GEMM result plus the residual in fp32, rounded.

Inputs are numpy float16 arrays (bf16 inputs are passed as their float32 values with ``dt`` = "bf16" to round to
bfloat16). Pinned against the reference's own PyTorch modules by ``tests/golden/make_golden.py``
(``decoder_golden.npz``).
"""

from __future__ import annotations

import numpy as np
from scipy.special import erf


def _round(x: np.ndarray, dt: str) -> np.ndarray:
    """fp32 -> the 16-bit type (round to nearest even), returned as float32 values."""
    x = np.asarray(x, dtype=np.float32)
    if dt == "f16":
        return x.astype(np.float16).astype(np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32)


def layer_norm(x: np.ndarray, gamma: np.ndarray, beta: np.ndarray, eps: float = 1e-5, dt: str = "f16") -> np.ndarray:
    """LN over the last axis (decoder_kernels.py:100-115, :55-72), rounded to the 16-bit type (float32 values)."""
    xf = np.asarray(x, dtype=np.float32)
    k = xf.shape[-1]
    mean = xf.sum(-1, dtype=np.float32, keepdims=True) / np.float32(k)
    d = xf - mean
    var = (d * d).sum(-1, dtype=np.float32, keepdims=True) / np.float32(k)
    rstd = np.float32(1.0) / np.sqrt(var + np.float32(eps), dtype=np.float32)
    y = d * rstd * np.asarray(gamma, np.float32) + np.asarray(beta, np.float32)
    return _round(y, dt)


def _gemm_bias(x: np.ndarray, w: np.ndarray, b: np.ndarray) -> np.ndarray:
    return (np.asarray(x, np.float32) @ np.asarray(w, np.float32).T + np.asarray(b, np.float32)).astype(np.float32)


def gelu(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, np.float32)
    return (0.5 * x * (1.0 + erf(x / np.sqrt(2.0)))).astype(np.float32)


def layer_norm_bias(x, gamma, beta, bias, eps: float = 1e-5, dt: str = "f16"):
    """(LN(x), round(x + bias)) -- decoder_kernels.py:127-135."""
    y = layer_norm(x, gamma, beta, eps, dt)
    return y, _round(np.asarray(x, np.float32) + np.asarray(bias, np.float32), dt)


def ln_linear(x, gamma, beta, w, b, gelu_: bool = False, eps: float = 1e-5, dt: str = "f16") -> np.ndarray:
    """round(LN(x) . w^T + b), GELU'd on the rounded value if ``gelu_`` -- decoder_kernels.py:138-146, :42-75."""
    h = _round(_gemm_bias(layer_norm(x, gamma, beta, eps, dt), w, b), dt)
    return _round(gelu(h), dt) if gelu_ else h


def linear_residual(x, w, b, res, dt: str = "f16") -> np.ndarray:
    """round(round(x . w^T + b) + res) -- decoder_kernels.py:149-157, :77-97."""
    h = _round(_gemm_bias(x, w, b), dt)
    return _round(h + np.asarray(res, np.float32), dt)
