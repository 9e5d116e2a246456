"""GPU parity: the multi-token (prompt) self-attention kernel (C ABI ``wt_self_attn``) against the oracle.

The reference's prompt op (attn_plugin.py:102-121, kernel :275-307) attends S new tokens per row to the row's cache
slots below offset, read through the slot table, and causally to the new tokens. Tolerance: max-abs 2e-3 for fp16
in / fp32 accumulate (tighter than the reference's own 2e-2 for its Triton kernel, test_attn_plugin.py:40-47); bf16
outputs add their rounding, 2^-8 * |ref|. The caches are not written."""

import numpy as np
import pytest
import torch

import cases
from oracle import attn as oa
from whisper_trt_b200 import attn_plugin as ap

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]
ATOL = 2e-3


def assert_close(out: torch.Tensor, ref: np.ndarray, dtype=torch.float16):
    o = out.float().cpu().numpy()
    err = np.abs(o - ref)
    bound = ATOL + (2.0**-8 * np.abs(ref) if dtype == torch.bfloat16 else 0.0)
    assert np.isfinite(o).all()
    assert (err <= bound).all(), f"max err {err.max():.3e} (bound {np.max(bound):.3e})"


def oracle(qkv, kc, vc, off, src):
    """The reference body on the kernel's clamped view of offset and the slot table (attn_plugin.py:284-285,296)."""
    n, c = src.shape
    off = off.clamp(0, c)
    src = src.clamp(0, n - 1)
    return oa.self_attn(qkv.float().cpu().numpy(), kc.float().cpu().numpy(), vc.float().cpu().numpy(),
                        off.cpu().numpy(), src.cpu().numpy())


@pytest.mark.parametrize("name", ["self_s4_f16", "self_s17_f16"])
def test_golden_prompt_cases(attn_golden, name):
    """The reference's own prompt cases (test_attn_plugin.py:40-47: b 10, h 20, c 96, S 4 / 17) against the stored
    reference outputs."""
    inp = cases.make_attn_inputs(*cases.ATTN_CASES[name])
    d = {k: v.cuda() for k, v in inp.items()}
    kc0, vc0 = d["kc"].clone(), d["vc"].clone()
    y = ap.self_attn_triton(d["qkv"], d["kc"], d["vc"], d["offset"], d["src"])
    assert y.shape == (10, inp["qkv"].shape[1], 20 * 64)
    assert_close(y, attn_golden[f"{name}/self"])
    assert torch.equal(d["kc"], kc0) and torch.equal(d["vc"], vc0)  # read only


def test_golden_fp32_case_in_fp16(attn_golden):
    """test_attn_plugin.py:20-34's fp32 case (S 3, h 4, c 32), inputs rounded to fp16, against the oracle on the same
    rounded inputs; the oracle on the fp32 inputs is pinned to the stored reference output by the CPU suite."""
    inp = cases.make_attn_inputs(*cases.ATTN_CASES["self_s3_f32"])
    d = {k: (v.half() if v.is_floating_point() else v).cuda() for k, v in inp.items()}
    y = ap.self_attn_triton(d["qkv"], d["kc"], d["vc"], d["offset"], d["src"])
    assert_close(y, oracle(d["qkv"], d["kc"], d["vc"], d["offset"], d["src"]))


def _case(n, s, h, c, dtype, seed, off=None, scale=1.0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    qkv = (torch.randn(n, s, 3 * h * 64, generator=g) * scale).to(dtype)
    kc = (torch.randn(n, h, c, 64, generator=g) * scale).to(dtype)
    vc = torch.randn(n, h, c, 64, generator=g).to(dtype)
    offset = torch.randint(0, c + 1, (n,), generator=g) if off is None else torch.as_tensor(off, dtype=torch.long)
    src = torch.randint(0, n, (n, c), generator=g).to(torch.int32)
    return [t.cuda() for t in (qkv, kc, vc, offset, src)]


@pytest.mark.parametrize("s", [1, 2, 15, 16, 17, 63, 64, 65, 127, 130, 224])
def test_prompt_lengths(s):
    qkv, kc, vc, off, src = _case(4, s, 3, 96, torch.float16, seed=s)
    y = ap.self_attn_triton(qkv, kc, vc, off, src)
    assert_close(y, oracle(qkv, kc, vc, off, src))


@pytest.mark.parametrize("c,offs", [(1, [0, 1, 1]), (17, [0, 16, 17]), (64, [63, 64, 1]), (65, [65, 64, 0]),
                                    (228, [4, 224, 100]), (448, [448, 0, 300])])
def test_cache_lengths(c, offs):
    """Empty caches, one slot, cache blocks ending exactly at and one past a 64-key block, a full cache."""
    qkv, kc, vc, off, src = _case(3, 40, 2, c, torch.float16, seed=c, off=offs)
    y = ap.self_attn_triton(qkv, kc, vc, off, src)
    assert_close(y, oracle(qkv, kc, vc, off, src))


def test_whisper_prompt_shape():
    """A whisper-large-v3 prompt: 20 heads x 64, a 224-token prompt after 0 / 100 cached positions (C 448)."""
    qkv, kc, vc, off, src = _case(2, 224, 20, 448, torch.float16, seed=7, off=[0, 100], scale=0.5)
    y = ap.self_attn_triton(qkv, kc, vc, off, src)
    assert_close(y, oracle(qkv, kc, vc, off, src))


def test_bf16():
    qkv, kc, vc, off, src = _case(3, 70, 4, 130, torch.bfloat16, seed=3)
    y = ap.self_attn_triton(qkv, kc, vc, off, src)
    assert_close(y, oracle(qkv, kc, vc, off, src), torch.bfloat16)


def test_out_of_range_offsets_and_rows_are_clamped():
    """Offsets below 0 / above C and slot-table rows outside [0, N) are clamped (attn_plugin.py:284-285,296), never
    read out of bounds."""
    qkv, kc, vc, off, src = _case(4, 20, 2, 50, torch.float16, seed=11, off=[-5, 80, 50, 3])
    src[0, :10] = -7
    src[1, 5:20] = 1000
    y = ap.self_attn_triton(qkv, kc, vc, off, src)
    assert_close(y, oracle(qkv, kc, vc, off, src))


def test_one_token_matches_the_step_kernel():
    """S = 1 through the prompt kernel equals the decode-step kernel (same op, reference test_attn_plugin.py:40)."""
    qkv, kc, vc, off, src = _case(10, 1, 20, 96, torch.float16, seed=5)
    a = ap.self_attn_triton(qkv, kc, vc, off, src).float()
    b = ap.self_attn_step_triton(qkv, kc, vc, off, src).float()
    assert (a - b).abs().max().item() < 2e-3


def test_custom_op_and_graph_capture():
    qkv, kc, vc, off, src = _case(4, 33, 2, 64, torch.float16, seed=9)
    ref = oracle(qkv, kc, vc, off, src)
    assert_close(torch.ops.whisper_trt_b200.self_attn(qkv, kc, vc, off, src), ref)
    out = torch.empty(4, 33, 128, dtype=torch.float16, device="cuda")
    ap.self_attn_triton(qkv, kc, vc, off, src, out=out)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        ap.self_attn_triton(qkv, kc, vc, off, src, out=out)
    out.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert_close(out, ref)


def test_argument_errors():
    qkv, kc, vc, off, src = _case(2, 4, 2, 16, torch.float16, seed=1)
    with pytest.raises(ValueError):
        ap.self_attn_triton(qkv, kc, vc, off[:1], src)
    with pytest.raises(ValueError):
        ap.self_attn_triton(qkv, kc, vc, off, src.long().int()[:, :8].contiguous())
    with pytest.raises(TypeError):
        ap.self_attn_triton(qkv.float(), kc.float(), vc.float(), off, src)
    with pytest.raises(ValueError):
        ap.self_attn_triton(qkv.cpu(), kc.cpu(), vc.cpu(), off.cpu(), src.cpu())
