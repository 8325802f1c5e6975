"""The CPU oracle against the reference's own known-answer tests (re-created
in tests/golden) and against an independent float64 PyTorch restatement."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
import torch_ref
from conftest import rel_max


def test_leaky_relu_uses_the_requested_negative_slope(kat):
    # src/models/sovits_decoder.rs:583-589, plus the sign-bit case -0.0.
    y = oracle.leaky_relu(kat["lrelu_in"], 0.1)
    assert np.array_equal(y[:3], np.array([-0.2, 0.0, 3.0], np.float32))
    assert np.signbit(y[3]) and y[3] == 0.0


def test_cpu_transposed_conv_crop_matches_padded_convolution(kat):
    # src/models/sovits_decoder.rs:591-612: full ConvT + crop == padded ConvT.
    y = oracle.conv_transpose1d(kat["convt_x"], kat["convt_w"], stride=2, padding=1)
    assert y.shape == kat["convt_out"].shape
    assert np.abs(y - kat["convt_out"]).max() < 1e-5


@pytest.mark.parametrize("k,d", [(3, 1), (7, 3)])
def test_parallel_im2col_conv_matches_candle(kat, k, d):
    # src/utils/weights.rs:684-710 (16 ch x 4096, affine ramps, 1e-5).
    C, L = 16, 4096
    x = (np.arange(C * L, dtype=np.float64) * 0.001 - 0.5).astype(np.float32).reshape(1, C, L)
    w = (np.arange(C * C * k, dtype=np.float64) * 0.0001 - 0.02).astype(np.float32).reshape(C, C, k)
    y = oracle.conv1d(x, w, padding=d * (k - 1) // 2, dilation=d)
    # The reference's bar is 1e-5 absolute on two fp32 paths; outputs here reach
    # ~600, where one fp32 ulp is 6e-5, so the bar is applied relative to max(1, |y|).
    ref = kat[f"im2col_k{k}d{d}_sub"]
    assert (np.abs(y[..., ::8] - ref) / np.maximum(1.0, np.abs(ref))).max() < 1e-5
    s = kat[f"im2col_k{k}d{d}_sum"]
    y64 = y.astype(np.float64)
    assert abs(y64.sum() - s[0]) <= 1e-5 * s[1]
    assert abs(np.abs(y64).sum() - s[1]) <= 1e-6 * s[1]
    assert abs((y64 * y64).sum() - s[2]) <= 1e-5 * s[2]


def test_weight_norm_fold_recovers_weight(gsv):
    rng = np.random.default_rng(5)
    w = rng.standard_normal((8, 4, 3)).astype(np.float32)
    r = rng.uniform(0.5, 2.0, (8, 1, 1)).astype(np.float32)
    g = np.sqrt((w.astype(np.float64) ** 2).sum(axis=(1, 2))).astype(np.float32)
    folded = oracle.weight_norm(w * r, g)
    assert rel_max(folded, w) < 1e-6


def test_synthetic_weights_are_stable(gsv, tiny):
    for init, bias in (("unit", "rand"), ("n001", "zero")):
        sd = gsv.synth.make_state_dict(0, init=init, bias=bias)
        assert gsv.synth.checksum(sd) == pytest.approx(float(tiny[f"{init}_checksum"]), rel=1e-9)


@pytest.mark.parametrize("T0", [1, 2, 3, 7])
@pytest.mark.parametrize("init,bias", [("unit", "rand"), ("n001", "zero")])
def test_oracle_decoder_matches_golden(gsv, tiny, init, bias, T0):
    sd = gsv.synth.make_state_dict(0, init=init, bias=bias)
    z, g = gsv.synth.make_inputs(2, T0)
    ref = tiny[f"{init}_T{T0}_wav"]
    for acc64 in (True, False):
        wav = oracle.decoder_forward(sd, z, g, acc64=acc64)
        assert wav.shape == ref.shape == (2 * 640 * T0,)
        assert rel_max(wav, ref) < 2e-5


def test_oracle_taps_match_torch(gsv):
    sd = gsv.synth.make_state_dict(1, init="unit", bias="rand")
    z, g = gsv.synth.make_inputs(1, 4, seed_z=7, seed_g=8)
    wav, taps = oracle.decoder_forward(sd, z, g, taps=True)
    wref, tref = torch_ref.decoder_forward(sd, z, g, taps=True)
    assert len(taps) == len(tref) == 12
    for a, b in zip(taps, tref):
        assert a.shape == b.shape
        assert rel_max(a, b) < 1e-5
    assert rel_max(wav, wref) < 1e-5


def test_oracle_without_cond_and_g(gsv):
    sd = gsv.synth.make_state_dict(2, init="unit", bias="rand", with_cond=False)
    z, g = gsv.synth.make_inputs(1, 3)
    a = oracle.decoder_forward(sd, z, g)
    b = oracle.decoder_forward(sd, z, None)
    assert np.array_equal(a, b)  # no dec.cond: g is ignored (sovits_decoder.rs:393-399)
    assert rel_max(a, torch_ref.decoder_forward(sd, z, None)) < 1e-5


def test_oracle_reports_missing_keys(gsv):
    sd = gsv.synth.make_state_dict(0)
    del sd["dec.conv_pre.weight"]
    z, g = gsv.synth.make_inputs(1, 2)
    with pytest.raises(oracle.OracleError, match="dec.conv_pre.weight"):
        oracle.decoder_forward(sd, z, g)
