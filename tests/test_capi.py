"""The C ABI library on the CPU: it loads, exports every symbol the header declares, and rejects bad arguments
with a status and a message before touching the GPU. Also the Python shim's host-side checks."""

import ctypes
import re
from pathlib import Path

import pytest
import torch

from whisper_trt_b200 import _lib, attn_plugin, slots

HEADER = Path(__file__).resolve().parent.parent / "include" / "whisper_attn_b200.h"


def declared_symbols() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(wt_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_symbols()
    assert len(names) >= 15
    for name in names:
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_signatures_cover_only_declared_symbols():
    assert sorted(_lib.SIGNATURES) == declared_symbols()


def test_version_and_status_strings():
    lib = _lib.load()
    assert lib.wt_abi_version() == 1
    assert lib.wt_status_string(_lib.WT_OK) == b"ok"
    assert lib.wt_status_string(_lib.WT_ERR_ALIGN).startswith(b"pointer")
    assert lib.wt_status_string(99) == b"unknown status"


def test_launch_flags_roundtrip():
    prev = _lib.set_launch_flags(_lib.WT_LAUNCH_PDL)
    assert _lib.set_launch_flags(prev) == _lib.WT_LAUNCH_PDL


def _fake(n):  # host addresses, 16-byte aligned: the checks run before any device access
    buf = (ctypes.c_char * (n + 64))()
    return (ctypes.addressof(buf) + 15) // 16 * 16, buf


def test_bad_arguments_return_status_without_a_gpu():
    lib = _lib.load()
    p, keep = _fake(1024)
    st = lib.wt_self_attn_step(0, p, p, p, p, p, p, 0, 20, 96, 64, 0, 1, None, 0, None)
    assert st == _lib.WT_ERR_ARG and b"sizes" in lib.wt_last_error()
    st = lib.wt_self_attn_step(0, p + 2, p, p, p, p, p, 4, 20, 96, 64, 0, 1, None, 0, None)
    assert st == _lib.WT_ERR_ALIGN and b"qkv" in lib.wt_last_error()
    st = lib.wt_self_attn_step(0, p, p, p, p, p, p, 4, 20, 96, 48, 0, 1, None, 0, None)
    assert st == _lib.WT_ERR_UNSUPPORTED
    st = lib.wt_self_attn_step(7, p, p, p, p, p, p, 4, 20, 96, 64, 0, 1, None, 0, None)
    assert st == _lib.WT_ERR_DTYPE
    st = lib.wt_self_attn_step(0, p, p, p, p, p, p, 4, 20, 96, 64, 0, 4, None, 0, None)
    assert st == _lib.WT_ERR_WORKSPACE
    st = lib.wt_cross_attn(0, p, p, p, p, 2, 5, 20, 1500, 64, None, 0, None)
    assert st == _lib.WT_ERR_WORKSPACE
    pre = lambda dt, c, d, group, ms, ws, nb: lib.wt_self_attn_step_prefix(dt, p, p, p, p, p, p, 10, 20, c, d, 0,
                                                                            group, ms, ws, nb, None)
    assert pre(0, 96, 48, 5, 32, p, 1 << 20) == _lib.WT_ERR_UNSUPPORTED  # head_dim 64 only
    assert pre(0, 96, 64, 0, 32, p, 1 << 20) == _lib.WT_ERR_ARG  # group 1-8
    assert pre(0, 96, 64, 9, 32, p, 1 << 20) == _lib.WT_ERR_ARG
    assert pre(0, 96, 64, 5, 0, p, 1 << 20) == _lib.WT_ERR_ARG  # min_shared >= 1
    assert pre(0, 2000, 64, 5, 32, p, 1 << 20) == _lib.WT_ERR_UNSUPPORTED  # no key splits
    assert pre(7, 96, 64, 5, 32, p, 1 << 20) == _lib.WT_ERR_DTYPE
    assert pre(0, 96, 64, 5, 32, None, 0) == _lib.WT_ERR_WORKSPACE
    assert pre(0, 96, 64, 5, 32, p, 100) == _lib.WT_ERR_WORKSPACE
    st = lib.wt_beam_scores(*([p] * 11), 2, 5, 51866, 16, 0, 50362, 0, 0, 50257, None, 0, None)
    assert st == _lib.WT_ERR_WORKSPACE
    st = lib.wt_beam_scores(*([p] * 11), 2, 9, 51866, 16, 0, 50362, 0, 0, 50257, p, 1 << 20, None)
    assert st == _lib.WT_ERR_UNSUPPORTED  # more than 8 beams
    st = lib.wt_beam_scores(*([p] * 11), 2, 5, 51866, 16, 1, 50362, 50363, 0, 50257, p, 1 << 20, None)
    assert st == _lib.WT_ERR_ARG  # timestamps without a timestamp_begin
    st = lib.wt_logits32(0, p, p, p, 160, 51866, 1280, None, None)
    assert st == _lib.WT_ERR_ARG  # no error word
    st = lib.wt_logits32(0, p, p, p, 160, 51866, 1284, p, None)
    assert st == _lib.WT_ERR_UNSUPPORTED  # d not a multiple of 8
    st = lib.wt_logits32(2, p, p, p, 160, 51866, 1280, p, None)
    assert st == _lib.WT_ERR_DTYPE
    st = lib.wt_self_attn(0, p, p, p, p, p, p, 4, 0, 20, 96, 64, None)
    assert st == _lib.WT_ERR_ARG and b"sizes" in lib.wt_last_error()
    st = lib.wt_self_attn(0, p, p, p, p, p, p + 8, 4, 3, 20, 96, 64, None)
    assert st == _lib.WT_ERR_ALIGN and b"y" in lib.wt_last_error()
    st = lib.wt_self_attn(0, p, p, p, p, p, p, 4, 3, 20, 96, 32, None)
    assert st == _lib.WT_ERR_UNSUPPORTED
    st = lib.wt_self_attn(5, p, p, p, p, p, p, 4, 3, 20, 96, 64, None)
    assert st == _lib.WT_ERR_DTYPE
    st = lib.wt_cross_attn_split(0, p, p, p, p, 2, 5, 20, 1500, 32, 8, None)
    assert st == _lib.WT_ERR_UNSUPPORTED
    st = lib.wt_beam_reorder(p, None, None, None, p, p, None, None, 2, 64, 8, 0, 1, None)
    assert st == _lib.WT_ERR_UNSUPPORTED  # more than 32 beams
    st = lib.wt_beam_update(*([p] * 18), 2, 5, 8, 4, 9, 4, 40, 1, None)
    assert st == _lib.WT_ERR_ARG  # hyp_slots < 2 * beams


def test_workspace_sizes():
    lib = _lib.load()
    assert lib.wt_self_attn_step_workspace(40, 20, 64, 1) == 0
    assert lib.wt_self_attn_step_workspace(5, 20, 64, 4) >= 5 * 20 * 4 * 66 * 4
    assert lib.wt_cross_attn_workspace(8, 5, 20, 1500, 64) == 256  # one CTA per (window, head): the error word only
    assert lib.wt_cross_attn_workspace(8, 16, 20, 1500, 64) > 8 * 20 * 66 * 4  # stream-K: partials and counters
    assert lib.wt_cross_attn_workspace(8, 5, 20, 1500, 32) == 0


def test_split_choice():
    """At least ceil(C / 1024) parts (the staged slot-table slice), more for few rows, never below ~64 slots each."""
    lib = _lib.load()
    for rows, cap in ((160, 228), (320, 448), (40, 228), (5, 448), (1, 16), (1000, 4096)):
        s = lib.wt_self_attn_step_splits(rows, 20, cap, 64)
        assert -(-cap // 1024) <= s <= max(1, -(-cap // 64)), (rows, cap, s)
    assert lib.wt_self_attn_step_splits(5, 20, 448, 64) > lib.wt_self_attn_step_splits(320, 20, 448, 64)


# --- the shim's host checks (the reference's error behaviour) --------------------------------------------------
def _step_inputs(n=4, h=2, c=8, d=64, dtype=torch.float16, device="cpu"):
    qkv = torch.zeros(n, 1, 3 * h * d, dtype=dtype, device=device)
    kc = torch.zeros(n, h, c, d, dtype=dtype, device=device)
    return qkv, kc, kc.clone(), torch.zeros(n, dtype=torch.long, device=device), torch.zeros(n, c, dtype=torch.int32,
                                                                                              device=device)


def test_step_rejects_more_than_one_token():
    qkv, kc, vc, off, src = _step_inputs()
    with pytest.raises(ValueError, match="one new token per row"):
        attn_plugin.self_attn_step_triton(torch.zeros(4, 2, 3 * 2 * 64, dtype=torch.half), kc, vc, off, src)


def test_step_rejects_cpu_tensors_and_bad_types():
    qkv, kc, vc, off, src = _step_inputs()
    with pytest.raises(ValueError, match="no CPU path"):
        attn_plugin.self_attn_step_triton(qkv, kc, vc, off, src)
    with pytest.raises(TypeError, match="not supported"):
        attn_plugin.self_attn_step_triton(qkv.float(), kc.float(), vc.float(), off, src)
    with pytest.raises(ValueError, match="int32"):
        attn_plugin.self_attn_step_triton(qkv, kc, vc, off, src.long())
    with pytest.raises(ValueError, match="does not match"):
        attn_plugin.self_attn_step_triton(qkv[:, :, :-64], kc, vc, off, src)


def test_cross_rejects_mismatched_shapes():
    q = torch.zeros(2, 5, 128, dtype=torch.half)
    k = torch.zeros(2, 2, 10, 64, dtype=torch.half)
    with pytest.raises(ValueError, match="no CPU path"):
        attn_plugin.cross_attn_triton(q, k, k)
    with pytest.raises(ValueError, match="does not match"):
        attn_plugin.cross_attn_split_triton(q[:, :, :64], k, k)
    with pytest.raises(ValueError, match="float32"):
        attn_plugin.cross_attn_combine_triton(torch.zeros(2, 2, 8, 5, 66, dtype=torch.half), q)


def test_slots_reject_bad_types():
    with pytest.raises(TypeError):
        slots.beam_reorder(torch.zeros(6, 4, dtype=torch.long), torch.zeros(2, 3, dtype=torch.long),
                           torch.zeros(2, dtype=torch.long))
    with pytest.raises(ValueError, match="rows"):
        slots.beam_reorder(torch.zeros(5, 4, dtype=torch.int32), torch.zeros(2, 3, dtype=torch.long),
                           torch.zeros(2, dtype=torch.long))


def test_install_routes_a_module():
    import types

    mod = types.SimpleNamespace()
    attn_plugin.install(mod)
    assert mod.self_attn_step_triton is attn_plugin.self_attn_step_triton
    assert mod.self_attn_triton is attn_plugin.self_attn_triton
    assert mod.cross_attn_combine_triton is attn_plugin.cross_attn_combine_triton


def test_decoder_linear_arguments_without_a_gpu():
    """The fused decoder linear layers refuse bad sizes, alignments and workspaces with a status and a message before
    any device access."""
    lib = _lib.load()
    p, keep = _fake(1 << 16)
    assert lib.wt_dec_linear_workspace(160, 1280, 1280, 0) == 256  # (the device error word)
    assert lib.wt_dec_linear_workspace(160, 1280, 1280, 1) == 256 + 160 * 1280 * 2  # (+ the normalized rows)
    assert lib.wt_dec_linear_workspace(0, 1280, 1280, 1) == 0
    st = lib.wt_ln_linear(0, p, p, p, p, p, p, 5, 128, 60, 0, 1e-5, p, 1 << 16, None)
    assert st == _lib.WT_ERR_UNSUPPORTED and b"multiple of 8" in lib.wt_last_error()
    st = lib.wt_ln_linear(0, p, p, p, p, p, None, 5, 128, 64, 0, 1e-5, p, 1 << 16, None)
    assert st == _lib.WT_ERR_ARG and b"null" in lib.wt_last_error()
    st = lib.wt_ln_linear(0, p, p, p, p, p, p, 5, 128, 64, 0, 1e-5, p, 16, None)
    assert st == _lib.WT_ERR_WORKSPACE
    st = lib.wt_linear_residual(2, p, p, p, p, p, 5, 128, 64, p, 1 << 16, None)
    assert st == _lib.WT_ERR_DTYPE
    st = lib.wt_linear_residual(0, p + 4, p, p, p, p, 5, 128, 64, p, 1 << 16, None)
    assert st == _lib.WT_ERR_ALIGN and b"x" in lib.wt_last_error()
    st = lib.wt_layer_norm_bias(0, p, p, p, p, p, 0, 64, 1e-5, None)
    assert st == _lib.WT_ERR_ARG
    st = lib.wt_layer_norm_bias(0, p, p, p, p, p, 4, 60, 1e-5, None)
    assert st == _lib.WT_ERR_UNSUPPORTED


def test_decoder_linear_python_checks():
    from whisper_trt_b200 import decoder_kernels as dk

    x = torch.zeros(5, 64, dtype=torch.half)
    w = torch.zeros(128, 64, dtype=torch.half)
    b = torch.zeros(128, dtype=torch.half)
    with pytest.raises(ValueError, match="CUDA"):
        dk.linear_residual(x, w, b, torch.zeros(5, 128, dtype=torch.half))
    with pytest.raises(ValueError, match="do not match"):
        dk.ln_linear(x, torch.zeros(64, dtype=torch.half), torch.zeros(64, dtype=torch.half), w[:, :32], b)
    with pytest.raises(TypeError, match="one dtype"):
        dk.linear_residual(x, w.float(), b, torch.zeros(5, 128, dtype=torch.half))
    with pytest.raises(ValueError, match="gamma"):
        dk.layer_norm_bias(x, torch.zeros(32, dtype=torch.half), torch.zeros(64, dtype=torch.half),
                           torch.zeros(64, dtype=torch.half))


def test_triton_baseline_without_the_reference(tmp_path):
    """The GPU baseline module reports, and does not fail, when no reference package is staged."""
    import json
    import subprocess
    import sys

    root = Path(__file__).resolve().parent.parent
    out = subprocess.run([sys.executable, str(root / "benchmarks" / "triton_baseline.py"), "--ref", str(tmp_path)],
                         cwd=root, capture_output=True, text=True, timeout=300, check=True)
    assert "unavailable" in json.loads(out.stdout.strip().splitlines()[-1])
