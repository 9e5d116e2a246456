"""ctypes binding of the C ABI (``include/whisper_attn_b200.h``) in ``libwhisper_attn_b200.so``.

The library is loaded on first use from this package's directory (built in-tree by ``build.py``). There is no
fallback: if the library is missing or fails to load, every op raises.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libwhisper_attn_b200.so"

c_int, c_size, c_void, c_float = ctypes.c_int, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_float
c_char_p = ctypes.c_char_p

# name -> (restype, argtypes); the order of the header
SIGNATURES = {
    "wt_abi_version": (c_int, []),
    "wt_status_string": (c_char_p, [c_int]),
    "wt_last_error": (c_char_p, []),
    "wt_set_launch_flags": (c_int, [c_int]),
    "wt_set_wait_limit": (ctypes.c_uint, [ctypes.c_uint]),
    "wt_set_test_withhold_stage": (c_int, [c_int]),
    "wt_self_attn_step_workspace": (c_size, [c_int, c_int, c_int, c_int]),
    "wt_self_attn_step_splits": (c_int, [c_int, c_int, c_int, c_int]),
    "wt_self_attn_step": (c_int, [c_int, c_void, c_void, c_void, c_void, c_void, c_void, c_int, c_int, c_int, c_int,
                                  c_int, c_int, c_void, c_size, c_void]),
    "wt_self_attn_step_prefix_workspace": (c_size, [c_int, c_int, c_int]),
    "wt_self_attn_step_prefix": (c_int, [c_int, c_void, c_void, c_void, c_void, c_void, c_void, c_int, c_int, c_int,
                                         c_int, c_int, c_int, c_int, c_void, c_size, c_void]),
    "wt_self_attn": (c_int, [c_int, c_void, c_void, c_void, c_void, c_void, c_void, c_int, c_int, c_int, c_int, c_int,
                             c_void]),
    "wt_cross_attn_split": (c_int, [c_int, c_void, c_void, c_void, c_void, c_int, c_int, c_int, c_int, c_int, c_int,
                                    c_void]),
    "wt_cross_attn_split_workspace": (c_size, [c_int] * 6),
    "wt_cross_attn_split_ws": (c_int, [c_int, c_void, c_void, c_void, c_void, c_int, c_int, c_int, c_int, c_int,
                                       c_int, c_void, c_size, c_void]),
    "wt_cross_attn_combine": (c_int, [c_int, c_void, c_void, c_int, c_int, c_int, c_int, c_int, c_void]),
    "wt_cross_attn_workspace": (c_size, [c_int, c_int, c_int, c_int, c_int]),
    "wt_cross_attn": (c_int, [c_int, c_void, c_void, c_void, c_void, c_int, c_int, c_int, c_int, c_int, c_void,
                              c_size, c_void]),
    "wt_cross_attn_noalloc": (c_int, [c_int, c_void, c_void, c_void, c_void, c_int, c_int, c_int, c_int, c_int,
                                      c_void]),
    "wt_cache_append": (c_int, [c_int, c_void, c_void, c_void, c_void, c_int, c_int, c_int, c_int, c_void]),
    "wt_gather_cache": (c_int, [c_int, c_void, c_void, c_void, c_int, c_int, c_int, c_int, c_void]),
    "wt_beam_reorder": (c_int, [c_void, c_void, c_void, c_void, c_void, c_void, c_void, c_void, c_int, c_int, c_int,
                                c_int, c_int, c_void]),
    "wt_beam_update": (c_int, [c_void] * 18 + [c_int] * 8 + [c_void]),
    "wt_slot_reset": (c_int, [c_void, c_void, c_int, c_int, c_int, c_int, c_int, c_void]),
    "wt_beam_update_mixed": (c_int, [c_void] * 23 + [c_int] * 8 + [c_void]),
    "wt_beam_sample": (c_int, [c_void] * 9 + [c_int] * 3 + [c_void]),
    "wt_logits32": (c_int, [c_int, c_void, c_void, c_void, c_int, c_int, c_int, c_void, c_void]),
    "wt_beam_scores_workspace": (c_size, [c_int, c_int]),
    "wt_beam_scores": (c_int, [c_void] * 11 + [c_int] * 9 + [c_void, c_size, c_void]),
    "wt_beam_scores_mixed": (c_int, [c_void] * 12 + [c_int] * 9 + [c_void, c_size, c_void]),
    "wt_dec_linear_workspace": (c_size, [c_int, c_int, c_int, c_int]),
    "wt_layer_norm_bias": (c_int, [c_int, c_void, c_void, c_void, c_void, c_void, c_int, c_int, c_float, c_void]),
    "wt_ln_linear": (c_int, [c_int] + [c_void] * 6 + [c_int] * 4 + [c_float, c_void, c_size, c_void]),
    "wt_linear_residual": (c_int, [c_int] + [c_void] * 5 + [c_int] * 3 + [c_void, c_size, c_void]),
}

# status codes (whisper_attn_b200.h)
WT_OK, WT_ERR_ARG, WT_ERR_ALIGN, WT_ERR_DTYPE, WT_ERR_UNSUPPORTED, WT_ERR_WORKSPACE, WT_ERR_CUDA = range(7)
WT_F16, WT_BF16 = 0, 1
WT_LAUNCH_PDL = 1

_lib = None
_lock = threading.Lock()


def load() -> ctypes.CDLL:
    """The loaded library (raises if it is missing: build it with ``python -m whisper_trt_b200.build``)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(f"{LIB_PATH.name} is not built: run `python -m whisper_trt_b200.build` "
                                   f"(in {LIB_PATH.parent.parent}) -- there is no CPU fallback")
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype, fn.argtypes = res, args
            if lib.wt_abi_version() != 1:
                raise RuntimeError(f"{LIB_PATH.name}: ABI version {lib.wt_abi_version()}, expected 1")
            _lib = lib
    return _lib


class WtError(RuntimeError):
    """A C-ABI call failed (status and message)."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


def check(status: int, what: str) -> None:
    """Raise for a non-zero status: ValueError for argument/shape errors, RuntimeError for launch failures."""
    if status == WT_OK:
        return
    lib = load()
    msg = f"{what}: {lib.wt_status_string(status).decode()}: {lib.wt_last_error().decode()}"
    if status in (WT_ERR_ARG, WT_ERR_ALIGN, WT_ERR_DTYPE, WT_ERR_UNSUPPORTED, WT_ERR_WORKSPACE):
        raise ValueError(msg)
    raise WtError(status, msg)


def set_launch_flags(flags: int) -> int:
    """Process-wide launch flags (``WT_LAUNCH_PDL``); returns the previous value."""
    return load().wt_set_launch_flags(flags)
