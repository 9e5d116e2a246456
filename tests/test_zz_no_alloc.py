"""The no-allocation cross-attention entry point (``wt_cross_attn_noalloc``) against the workspace one.

``wt_cross_attn_noalloc`` exists for callers that cannot allocate device memory while they run -- a TensorRT-style
plugin enqueue that has to stay inside the memory its engine planned, or an application whose device memory is
owned by its own allocator. It keeps its scratch in a fixed 8 MiB device array inside the library instead of a
caller-given workspace. Each check below calls it through the C ABI (ctypes, raw pointers) twice in a row and
compares its output with ``wt_cross_attn`` (the entry point with a workspace) on the same inputs and with the CPU
oracle (``oracle.attn.cross_attn``, the reference op body restated), both within the attention tolerance of the
other tests (max-abs 2e-3): the two entry points run different kernels, so the oracle catches an error common to
both. This file is collected last on purpose.
"""

import numpy as np
import pytest
import torch

from oracle import attn as oracle
from whisper_trt_b200 import _lib

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]
ATOL = 2e-3


def _inputs(w, s, h, t, seed, dtype=torch.float16):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(w, s, h * 64, generator=g).to(dtype).cuda()
    k = torch.randn(w, h, t, 64, generator=g).to(dtype).cuda()
    v = torch.randn(w, h, t, 64, generator=g).to(dtype).cuda()
    return q, k, v


def _with_workspace(lib, code, q, k, v):
    w, s, hd = q.shape
    h, t = k.shape[1], k.shape[2]
    nbytes = lib.wt_cross_attn_workspace(w, s, h, t, 64)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    y = torch.empty_like(q)
    st = lib.wt_cross_attn(code, q.data_ptr(), k.data_ptr(), v.data_ptr(), y.data_ptr(), w, s, h, t, 64,
                           ws.data_ptr(), nbytes, torch.cuda.current_stream().cuda_stream)
    assert st == _lib.WT_OK, lib.wt_last_error()
    return y


def _no_alloc(lib, code, q, k, v):
    w, s, hd = q.shape
    h, t = k.shape[1], k.shape[2]
    y = torch.full_like(q, float("nan"))
    st = lib.wt_cross_attn_noalloc(code, q.data_ptr(), k.data_ptr(), v.data_ptr(), y.data_ptr(), w, s, h, t, 64,
                                   torch.cuda.current_stream().cuda_stream)
    assert st == _lib.WT_OK, lib.wt_last_error()
    return y


def _oracle(q, k, v):
    return torch.from_numpy(oracle.cross_attn(q.float().cpu().numpy(), k.float().cpu().numpy(),
                                              v.float().cpu().numpy()))


# (windows, queries per window, heads, frames): whisper's 5 beams over 1500 frames; 20 queries (three 8-query tiles);
# 40 queries (two query groups) over frames that are not a multiple of the key slices or of 16; a 17-frame window
@pytest.mark.parametrize("shape", [(8, 5, 20, 1500), (2, 5, 20, 1500), (3, 20, 4, 700), (2, 40, 4, 333),
                                   (1, 5, 20, 17)])
def test_no_alloc_matches_workspace_entry_point_twice(shape):
    lib = _lib.load()
    for call in range(2):  # two calls in a row: the second starts from the array the first left behind
        q, k, v = _inputs(*shape, seed=100 * call + shape[0])
        ref = _with_workspace(lib, _lib.WT_F16, q, k, v)
        out = _no_alloc(lib, _lib.WT_F16, q, k, v)
        torch.cuda.synchronize()
        err = (out.float() - ref.float()).abs().max().item()
        assert np.isfinite(err) and err <= ATOL, (call, err)
        err_oracle = (out.float().cpu() - _oracle(q, k, v)).abs().max().item()
        assert np.isfinite(err_oracle) and err_oracle <= ATOL, (call, err_oracle)


def test_no_alloc_bf16():
    lib = _lib.load()
    for call in range(2):
        q, k, v = _inputs(4, 5, 20, 1500, seed=7 + call, dtype=torch.bfloat16)
        ref = _with_workspace(lib, _lib.WT_BF16, q, k, v)
        out = _no_alloc(lib, _lib.WT_BF16, q, k, v)
        torch.cuda.synchronize()
        bound = ATOL + 2.0**-8 * ref.float().abs()
        assert ((out.float() - ref.float()).abs() <= bound).all()
        exact = _oracle(q, k, v)
        assert ((out.float().cpu() - exact).abs() <= ATOL + 2.0**-8 * exact.abs()).all()


def test_no_alloc_rejects_shapes_beyond_its_scratch():
    lib = _lib.load()
    q, k, v = _inputs(1, 5, 20, 16, seed=1)  # (pointers only; the size check fails before any launch)
    st = lib.wt_cross_attn_noalloc(_lib.WT_F16, q.data_ptr(), k.data_ptr(), v.data_ptr(), q.data_ptr(), 4096, 5,
                                   20, 1500, 64, torch.cuda.current_stream().cuda_stream)
    assert st == _lib.WT_ERR_UNSUPPORTED
    assert b"fixed scratch" in lib.wt_last_error()
