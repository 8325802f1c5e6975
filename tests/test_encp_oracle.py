"""The EncP chain oracle (C restatement of src/models/sovits_encp.rs:10-40,
:102-109, :371-375, :871-879 and src/models/sovits.rs:378-385) against the
reference crate's own known-answer test and float64 PyTorch fixtures, and the
library's host-side speed-length rule, on CPU."""
from __future__ import annotations

import math

import numpy as np
import pytest

import oracle
from conftest import ENCP_GOLDEN_LAYERS


@pytest.fixture(scope="module")
def sd(gsv):
    return gsv.synth.make_encp_state_dict(layers=ENCP_GOLDEN_LAYERS)


def test_encp_generator_is_stable(gsv, sd, encp_golden):
    assert gsv.synth.checksum(sd) == pytest.approx(float(encp_golden["checksum"]), rel=1e-9)


def test_interpolation_kat_exact(kat):
    # linear_interpolate_last_dim([0, 10], 4) == [0, 2.5, 7.5, 10]
    # (src/models/sovits_encp.rs:928-936), bit for bit.
    out = oracle.interpolate(kat["interp_in"], 4)
    assert out.dtype == np.float32
    assert np.array_equal(out, kat["interp_out"])


@pytest.mark.parametrize("T_out", [30, 50])
def test_oracle_interpolation_matches_torch(encp_golden, T_out):
    # The reference forms the source positions in f32 ((i + 0.5) * (T / T_out)
    # - 0.5): position errors of ~T * 2^-24 move the blend weights, so the f32
    # result sits ~3e-6 (relative) from float64 torch.
    out = oracle.interpolate(encp_golden["T37_x"], T_out)
    ref = encp_golden[f"interp_{T_out}"]
    assert np.abs(out - ref).max() <= 1e-5 * float(np.abs(ref).max())


def test_interpolation_same_length_copies(encp_golden):
    x = encp_golden["T37_x"]
    assert np.array_equal(oracle.interpolate(x, 37), x)


@pytest.mark.parametrize("T", [1, 4, 37])
def test_oracle_add_norm_matches_golden(sd, encp_golden, T):
    p = "enc_p.encoder_text.norm_layers_1.0"
    out = oracle.layer_norm(encp_golden[f"T{T}_x"], sd[p + ".gamma"], sd[p + ".beta"], y=encp_golden[f"T{T}_y"])
    ref = encp_golden[f"T{T}_add_norm"]
    assert np.abs(out - ref).max() <= 1e-5 * max(1.0, float(np.abs(ref).max()))


@pytest.mark.parametrize("T", [1, 4, 37])
def test_oracle_ffn_matches_golden(sd, encp_golden, T):
    ln = encp_golden[f"T{T}_len"]
    out = oracle.encp_ffn(sd, "encoder_ssl", 0, encp_golden[f"T{T}_x"], ln)
    ref = encp_golden[f"T{T}_ffn"]
    assert np.abs(out - ref).max() <= 1e-5 * max(1.0, float(np.abs(ref).max()))
    assert not np.any(out[1, :, int(ln[1]):])  # x * x_mask


@pytest.mark.parametrize("T", [1, 4, 37])
def test_oracle_project_matches_golden(sd, encp_golden, T):
    ln = encp_golden[f"T{T}_len"]
    m, logs, zp = oracle.encp_project(sd, encp_golden[f"T{T}_x"], ln, encp_golden[f"T{T}_noise"], 0.5)
    for name, a in (("m", m), ("logs", logs), ("zp", zp)):
        ref = encp_golden[f"T{T}_{name}"]
        assert np.abs(a - ref).max() <= 1e-5 * max(1.0, float(np.abs(ref).max())), name
    assert logs.min() >= -5.0 and logs.max() <= 2.0
    # padded frames: m = 0, logs = 0, z_p = noise * noise_scale
    n = encp_golden[f"T{T}_noise"]
    tail = slice(int(ln[1]), None)
    assert not np.any(m[1, :, tail]) and not np.any(logs[1, :, tail])
    assert np.allclose(zp[1, :, tail], n[1, :, tail] * 0.5, rtol=0, atol=1e-7)


def test_layer_norm_constant_column_gives_beta():
    x = np.full((1, 8, 3), 2.5, np.float32)
    gamma = np.linspace(0.5, 1.5, 8).astype(np.float32)
    beta = np.linspace(-1, 1, 8).astype(np.float32)
    out = oracle.layer_norm(x, gamma, beta)
    assert np.allclose(out, beta[None, :, None], atol=1e-6)


def _speed_len_formula(T, speed):
    s = np.float32(speed)
    if abs(s - np.float32(1.0)) <= np.finfo(np.float32).eps:
        return T
    return max(1, math.trunc(float(np.float32(T) / s)) + 1)


@pytest.mark.parametrize("T,speed", [(100, 1.0), (100, 1.5), (100, 0.7), (37, 2.0), (1, 3.0),
                                     (250, 1.0000001), (999, 0.33)])
def test_speed_len_oracle_and_library(gsv, T, speed):
    exp = _speed_len_formula(T, speed)
    assert oracle.speed_len(T, speed) == exp
    assert gsv.Decoder.encp_speed_len(T, speed) == exp  # host-only ABI call


@pytest.mark.parametrize("speed", [0.0, -1.0, float("nan"), float("inf")])
def test_speed_len_rejects_bad_speed(gsv, speed):
    with pytest.raises(oracle.OracleError):
        oracle.speed_len(100, speed)
    with pytest.raises(gsv.GsvDecError):
        gsv.Decoder.encp_speed_len(100, speed)
