"""The oracle of the fused decoder linear layers (oracle/decoder.py) pinned against the reference's own modules
(decoder_golden.npz, made by tests/golden/make_golden.py from modeling.LayerNorm / modeling.gelu and the rounding
points of decoder_kernels.py). CPU only."""

import numpy as np
import pytest

import cases
from oracle import decoder as od

# fp16 outputs: the oracle's fp32 sums run in another order than torch's, so an output may differ by one unit in
# the last place of fp16 (2^-10 relative); everything else is exact
RTOL, ATOL = 2e-3, 2e-3


def _inputs(name):
    inp = cases.linear_case(**cases.DEC_CASES[name])
    return {k: v.float().numpy() for k, v in inp.items()}, inp


@pytest.mark.parametrize("name", list(cases.DEC_CASES))
def test_inputs_regenerate(name, decoder_golden):
    _, inp = _inputs(name)
    assert cases.digest(*[inp[k] for k in sorted(inp)]) == str(decoder_golden[f"{name}/digest"])


def _close(got, want):
    want = want.astype(np.float32)
    np.testing.assert_allclose(got, want, rtol=RTOL, atol=ATOL)
    assert np.mean(got == want) > 0.97  # (almost all bit-identical after the rounding)


@pytest.mark.parametrize("name", list(cases.DEC_CASES))
def test_oracle_matches_reference(name, decoder_golden):
    f, _ = _inputs(name)
    _close(od.layer_norm(f["x"], f["gamma"], f["beta"]), decoder_golden[f"{name}/layer_norm"])
    _close(od.ln_linear(f["x"], f["gamma"], f["beta"], f["w"], f["b"]), decoder_golden[f"{name}/ln_linear"])
    _close(od.ln_linear(f["x"], f["gamma"], f["beta"], f["w"], f["b"], gelu_=True),
           decoder_golden[f"{name}/ln_linear_gelu"])
    _close(od.linear_residual(f["x"], f["w"], f["b"], f["res"]), decoder_golden[f"{name}/linear_residual"])
    y, xb = od.layer_norm_bias(f["x"], f["gamma"], f["beta"], f["bias"])
    _close(y, decoder_golden[f"{name}/layer_norm"])
    np.testing.assert_array_equal(xb, decoder_golden[f"{name}/x_plus_bias"].astype(np.float32))


def test_bf16_rounding_is_nearest_even():
    x = np.array([1.0, 1.00390625, 1.01171875, -2.5, 3.0e-3], dtype=np.float32)
    import torch

    want = torch.from_numpy(x).bfloat16().float().numpy()
    np.testing.assert_array_equal(od._round(x, "bf16"), want)
