"""GSV_MODE_FP32_TC (mode "fp32tc") through the C ABI: the decoder at fp32
accuracy on the tcgen05 tensor cores.  Every activation and weight is held as
the exact sum of three bf16 pieces and each product is formed from the six
piece products that reach 2^-24 of it, so the mode is held to the FP32 mode's
bars against the oracle (waveform max-abs <= 1e-4 and, since N(0, 0.01)
weights shrink the waveform, max |err| / max |ref| <= 1e-4), and agrees with
the FP32 CUDA-core mode within half of them (the two sum in different orders;
the tensor cores' fp32 accumulation rounds once per instruction).
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from conftest import rel_max

pytestmark = pytest.mark.gpu

FP32_ABS = 1e-4
FP32_REL = 1e-4
AGREE_FP32 = 5e-5  # against the FP32 CUDA-core mode: both within the FP32 bar, summed in different orders


@pytest.fixture(scope="module")
def sd_unit(gsv):
    return gsv.synth.make_state_dict(0, init="unit", bias="rand")


@pytest.fixture(scope="module")
def dec_tc(gsv, sd_unit):
    d = gsv.Decoder.load(sd_unit, device=0, mode="fp32tc")
    yield d
    d.close()


def test_mode_is_reported(dec_tc):
    assert dec_tc.mode == "fp32tc"


@pytest.mark.parametrize("T0", [1, 2, 3, 7])
@pytest.mark.parametrize("init,bias", [("unit", "rand"), ("n001", "zero")])
def test_tiny_matches_golden(gsv, tiny, init, bias, T0):
    sd = gsv.synth.make_state_dict(0, init=init, bias=bias)
    dec = gsv.Decoder.load(sd, device=0, mode="fp32tc")
    try:
        z, g = gsv.synth.make_inputs(2, T0)
        wav = dec.forward(z, g)
        ref = tiny[f"{init}_T{T0}_wav"]
        assert wav.shape == ref.shape
        assert np.abs(wav - ref).max() <= FP32_ABS
        assert rel_max(wav, ref) <= FP32_REL
    finally:
        dec.close()


def test_cfg1_matches_oracle(gsv):
    """The batch-1 5 s workload: z [1,192,250], N(0,0.01) weights, zero bias."""
    sd = gsv.synth.make_state_dict(0, init="n001", bias="zero")
    dec = gsv.Decoder.load(sd, device=0, mode="fp32tc")
    try:
        z, g = gsv.synth.make_inputs(1, 250)
        wav = dec.forward(z, g)
        ref = oracle.decoder_forward(sd, z, g)
        assert wav.shape == (160000,)
        assert np.abs(wav - ref).max() <= FP32_ABS
        assert rel_max(wav, ref) <= FP32_REL
    finally:
        dec.close()


def test_unit_gain_matches_oracle_and_fp32_mode(gsv, dec_tc, sd_unit):
    z, g = gsv.synth.make_inputs(2, 40, seed_z=11, seed_g=12)
    wav = dec_tc.forward(z, g)
    ref = oracle.decoder_forward(sd_unit, z, g)
    assert np.abs(wav - ref).max() <= FP32_ABS
    assert rel_max(wav, ref) <= FP32_REL
    f32 = gsv.Decoder.load(sd_unit, device=0, mode="fp32")
    try:
        assert rel_max(wav, f32.forward(z, g)) <= AGREE_FP32
    finally:
        f32.close()


def test_per_layer_taps(gsv, dec_tc, sd_unit):
    z, g = gsv.synth.make_inputs(1, 9, seed_z=21, seed_g=22)
    wav, taps = dec_tc.forward_debug(z, g)
    rwav, rtaps = oracle.decoder_forward(sd_unit, z, g, taps=True)
    assert len(taps) == len(rtaps) == 12
    for i, (a, b) in enumerate(zip(taps, rtaps)):
        assert a.shape == b.shape, i
        assert rel_max(a, b) <= FP32_REL, i
    assert rel_max(wav, rwav) <= FP32_REL


def test_length_masking(gsv, dec_tc, sd_unit):
    """Each utterance of a right-padded batch decodes as if it were alone."""
    T0 = 12
    lens = [12, 9, 1]
    z, g = gsv.synth.make_inputs(3, T0, seed_z=31, seed_g=32)
    wav = dec_tc.forward(z, g, lengths=lens).reshape(3, -1)
    for b, n in enumerate(lens):
        ref = oracle.decoder_forward(sd_unit, z[b:b + 1, :, :n], g[b:b + 1])
        assert rel_max(wav[b, :640 * n], ref) <= FP32_REL
        assert not wav[b, 640 * n:].any()


def test_chunked_equals_whole(gsv, dec_tc):
    """No launch here splits its K loop by size: a time chunk decoded with its
    halo gives the whole decode's samples bit for bit."""
    T0 = 60
    z, g = gsv.synth.make_inputs(1, T0, seed_z=41, seed_g=42)
    whole = dec_tc.forward(z, g)
    parts = [dec_tc.forward_chunk(z, g, a, b, halo=16) for a, b in ((0, 17), (17, 38), (38, 60))]
    assert np.array_equal(np.concatenate(parts), whole)


def test_device_memory_path(gsv, dec_tc):
    import torch
    z, g = gsv.synth.make_inputs(2, 8, seed_z=51, seed_g=52)
    host = dec_tc.forward(z, g)
    dev = dec_tc.forward_device(torch.from_numpy(z).cuda(), torch.from_numpy(g).cuda())
    torch.cuda.synchronize()
    assert np.array_equal(dev.cpu().numpy(), host)


def test_larger_batch_agrees_with_fp32_mode(gsv, sd_unit, dec_tc):
    """A batch big enough for multi-tile walks and multi-window tiles in every
    stage (4 x 2.5 s: 500 frames give the 64-channel launches four tiles per SM
    to spare), against the FP32 CUDA-core mode."""
    z, g = gsv.synth.make_inputs(4, 125, seed_z=61, seed_g=62)
    wav = dec_tc.forward(z, g)
    f32 = gsv.Decoder.load(sd_unit, device=0, mode="fp32")
    try:
        assert rel_max(wav, f32.forward(z, g)) <= AGREE_FP32
    finally:
        f32.close()
