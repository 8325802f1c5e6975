"""Parity of the CUDA EncP chains (through the C ABI) with the CPU oracle and
the float64 fixtures.

* add + LayerNorm (src/models/sovits_encp.rs:102; src/utils/weights.rs:461-502)
  runs in fp32 in both modes: max |err| / max |ref| <= 1e-5.
* FFN half (:104-109) and projection + prior sample (:871-879;
  src/models/sovits.rs:378-385): FP32 mode max |err| / max |ref| <= 1e-4;
  BF16 mode SNR >= 30 dB.  Masked frames are exactly zero (m, logs) or
  exactly noise * noise_scale (z_p) in both modes.
* interpolation (:10-40) is bit-identical to the oracle (the reference's f32
  operation order), including the crate's own known-answer test.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from conftest import ENCP_GOLDEN_LAYERS, rel_max, snr_db

pytestmark = pytest.mark.gpu

FP32_REL = 1e-4
LN_REL = 1e-5
BF16_SNR_DB = 30.0
LAYERS = {"encoder_ssl": 1, "encoder_text": 2, "encoder2": 1}


@pytest.fixture(scope="module")
def sd_encp(gsv):
    sd = gsv.synth.make_state_dict(0, init="unit", bias="rand")
    sd.update(gsv.synth.make_encp_state_dict(layers=LAYERS))
    return sd


@pytest.fixture(scope="module")
def handles(gsv, sd_encp):
    hs = {m: gsv.Decoder.load(sd_encp, device=0, mode=m) for m in ("fp32", "bf16")}
    yield hs
    for h in hs.values():
        h.close()


@pytest.fixture(scope="module")
def golden_handles(gsv):
    sd = gsv.synth.make_state_dict(0, init="unit", bias="rand")
    sd.update(gsv.synth.make_encp_state_dict(layers=ENCP_GOLDEN_LAYERS))
    hs = {m: gsv.Decoder.load(sd, device=0, mode=m) for m in ("fp32", "bf16")}
    yield hs
    for h in hs.values():
        h.close()


def _x(B, T, seed=7):
    return np.random.default_rng(seed).standard_normal((B, 192, T)).astype(np.float32)


def _check(mode, out, ref):
    if mode == "fp32":
        assert rel_max(out, ref) <= FP32_REL
    else:
        assert snr_db(out, ref) >= BF16_SNR_DB


def test_encp_info(handles):
    info = handles["bf16"].encp_info
    assert info["layers"] == LAYERS
    assert info["channels"] == 192 and info["filter_channels"] == 768 and info["proj_channels"] == 384


@pytest.mark.parametrize("mode", ["fp32", "bf16"])
@pytest.mark.parametrize("T", [1, 4, 37])
def test_golden_fixtures(golden_handles, encp_golden, mode, T):
    h = golden_handles[mode]
    x, y, ln, noise = (encp_golden[f"T{T}_{k}"] for k in ("x", "y", "len", "noise"))
    assert rel_max(h.encp_add_norm("encoder_text", 0, x, y), encp_golden[f"T{T}_add_norm"]) <= LN_REL
    _check(mode, h.encp_ffn("encoder_ssl", 0, x, ln), encp_golden[f"T{T}_ffn"])
    m, logs, zp = h.encp_project(x, ln, noise, 0.5)
    for name, a in (("m", m), ("logs", logs), ("zp", zp)):
        _check(mode, a, encp_golden[f"T{T}_{name}"])


@pytest.mark.parametrize("norm", [1, 2])
@pytest.mark.parametrize("T,lengths", [(1, None), (33, [33, 20, 1]), (300, [300, 171, 64])])
def test_add_norm_matches_oracle(handles, sd_encp, norm, T, lengths):
    B = 3
    x, y = _x(B, T, 1), _x(B, T, 2)
    p = f"enc_p.encoder_text.norm_layers_{norm}.1"
    ref = oracle.layer_norm(x, sd_encp[p + ".gamma"], sd_encp[p + ".beta"], y=y, lengths=lengths)
    for mode in ("fp32", "bf16"):
        out = handles[mode].encp_add_norm("encoder_text", 1, x, y, lengths, norm=norm)
        assert rel_max(out, ref) <= LN_REL
        if lengths is not None:
            assert not np.any(out[1, :, lengths[1]:])
    # y = None: LayerNorm of x alone
    ref0 = oracle.layer_norm(x, sd_encp[p + ".gamma"], sd_encp[p + ".beta"])
    assert rel_max(handles["fp32"].encp_add_norm("encoder_text", 1, x, None, norm=norm), ref0) <= LN_REL


@pytest.mark.parametrize("mode", ["fp32", "bf16"])
@pytest.mark.parametrize("stack,layer", [("encoder_ssl", 0), ("encoder_text", 1), ("encoder2", 0)])
@pytest.mark.parametrize("T,lengths", [(2, [2, 1]), (129, [129, 77]), (500, [500, 233])])
def test_ffn_matches_oracle(handles, sd_encp, mode, stack, layer, T, lengths):
    x = _x(2, T, 3)
    ref = oracle.encp_ffn(sd_encp, stack, layer, x, lengths)
    out = handles[mode].encp_ffn(stack, layer, x, lengths)
    _check(mode, out, ref)
    assert not np.any(out[1, :, lengths[1]:])


def test_ffn_device_equals_host(handles):
    import torch
    x = _x(4, 200, 4)
    ln = [200, 150, 99, 3]
    h = handles["bf16"]
    host = h.encp_ffn("encoder_text", 0, x, ln)
    xd = torch.from_numpy(x).cuda()
    ld = torch.tensor(ln, dtype=torch.int32, device="cuda")
    dev = h.encp_ffn_device("encoder_text", 0, xd, ld)
    torch.cuda.synchronize()
    assert np.array_equal(dev.cpu().numpy(), host)


@pytest.mark.parametrize("mode", ["fp32", "bf16"])
@pytest.mark.parametrize("T,lengths", [(1, None), (61, [61, 30]), (400, [400, 1])])
def test_project_matches_oracle(handles, sd_encp, mode, T, lengths):
    y, noise = _x(2, T, 5), _x(2, T, 6)
    rm, rl, rz = oracle.encp_project(sd_encp, y, lengths, noise, 0.667)
    m, logs, zp = handles[mode].encp_project(y, lengths, noise, 0.667)
    for a, r in ((m, rm), (logs, rl), (zp, rz)):
        _check(mode, a, r)
    assert logs.min() >= -5.0 and logs.max() <= 2.0
    if lengths is not None:
        tail = slice(lengths[1], None)
        assert not np.any(m[1, :, tail]) and not np.any(logs[1, :, tail])
        assert np.array_equal(zp[1, :, tail], (noise[1, :, tail] * np.float32(0.667)).astype(np.float32))


def test_project_without_noise(handles):
    m, logs, zp = handles["fp32"].encp_project(_x(1, 10, 8), None, None)
    assert zp is None and m.shape == (1, 192, 10)


def test_interpolation_kat_bit_exact(handles, kat):
    out = handles["bf16"].encp_interpolate(kat["interp_in"], T_out=4)
    assert np.array_equal(out, kat["interp_out"])


@pytest.mark.parametrize("T,T_out", [(37, 30), (37, 50), (1, 5), (500, 334), (250, 251), (7, 7)])
def test_interpolation_bit_exact(handles, T, T_out):
    y = _x(2, T, 9)
    out = handles["fp32"].encp_interpolate(y, T_out=T_out)
    assert np.array_equal(out, oracle.interpolate(y, T_out))


@pytest.mark.parametrize("speed", [1.0, 0.8, 1.25, 2.0])
def test_interpolation_by_speed(handles, speed):
    y = _x(1, 120, 10)
    To = oracle.speed_len(120, speed)
    out = handles["bf16"].encp_interpolate(y, speed=speed)
    assert out.shape == (1, 192, To)
    assert np.array_equal(out, oracle.interpolate(y, To))


def test_encp_errors(gsv, handles):
    h = handles["fp32"]
    with pytest.raises(gsv.GsvDecError):
        h.encp_ffn("encoder2", 5, _x(1, 4))       # no such layer
    with pytest.raises(gsv.GsvDecError):
        h.encp_add_norm("encoder2", 0, _x(1, 4), norm=3)
    with pytest.raises(gsv.GsvDecError):
        h.encp_ffn(7, 0, _x(1, 4))                # no such stack


def test_handle_without_encp(gsv):
    sd = gsv.synth.make_state_dict(0, init="unit", bias="rand")
    h = gsv.Decoder.load(sd, device=0, mode="bf16")
    try:
        info = h.encp_info
        assert info["layers"] == {"encoder_ssl": 0, "encoder_text": 0, "encoder2": 0}
        with pytest.raises(gsv.GsvDecError):
            h.encp_project(_x(1, 4))
        with pytest.raises(gsv.GsvDecError):
            h.encp_ffn("encoder_ssl", 0, _x(1, 4))
    finally:
        h.close()


@pytest.mark.parametrize("mode", ["fp32", "bf16"])
@pytest.mark.parametrize("with_attn", [True, False])
@pytest.mark.parametrize("T,lengths", [(3, [3, 2]), (250, [250, 97])])
def test_layer_matches_oracle(handles, sd_encp, mode, with_attn, T, lengths):
    x, attn = _x(2, T, 11), (_x(2, T, 12) if with_attn else None)
    p = "enc_p.encoder2.norm_layers_1.0"
    h1 = oracle.layer_norm(x, sd_encp[p + ".gamma"], sd_encp[p + ".beta"], y=attn)
    ref = oracle.encp_ffn(sd_encp, "encoder2", 0, h1, lengths)
    out = handles[mode].encp_layer("encoder2", 0, x, attn, lengths)
    _check(mode, out, ref)
    assert not np.any(out[1, :, lengths[1]:])


def test_layer_device_equals_host(handles):
    import torch
    x, attn = _x(3, 120, 13), _x(3, 120, 14)
    ln = [120, 64, 5]
    h = handles["bf16"]
    host = h.encp_layer("encoder_text", 1, x, attn, ln)
    dev = h.encp_layer_device("encoder_text", 1, torch.from_numpy(x).cuda(), torch.from_numpy(attn).cuda(),
                              torch.tensor(ln, dtype=torch.int32, device="cuda"))
    torch.cuda.synchronize()
    assert np.array_equal(dev.cpu().numpy(), host)


def test_load_file_reads_encp(gsv, sd_encp, handles, tmp_path):
    from safetensors.numpy import save_file
    p = tmp_path / "m.safetensors"
    save_file({k: np.ascontiguousarray(v) for k, v in sd_encp.items()}, str(p))
    d2 = gsv.Decoder.load_file(p, device=0, mode="fp32")
    try:
        assert d2.encp_info == handles["fp32"].encp_info
        x = _x(1, 16, 15)
        assert np.array_equal(d2.encp_ffn("encoder_text", 1, x), handles["fp32"].encp_ffn("encoder_text", 1, x))
    finally:
        d2.close()
