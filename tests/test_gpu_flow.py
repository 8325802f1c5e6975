"""Parity of the CUDA flow inverse (through the C ABI) with the CPU oracle.

ResidualCouplingBlock::forward(reverse = true) (src/models/sovits_flow.rs:
385-405) then z * y_mask (src/models/sovits.rs:394).  FP32 mode: max |err| /
max |ref| <= 1e-4.  BF16 mode: SNR >= 30 dB.  flow_decode must equal
flow_inverse followed by the decoder.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from conftest import rel_max, snr_db

pytestmark = pytest.mark.gpu

FP32_REL = 1e-4
BF16_SNR_DB = 30.0


@pytest.fixture(scope="module")
def sd_flow(gsv):
    sd = gsv.synth.make_state_dict(0, init="unit", bias="rand")
    sd.update(gsv.synth.make_flow_state_dict(init="unit"))
    return sd


@pytest.fixture(scope="module")
def handles(gsv, sd_flow):
    hs = {m: gsv.Decoder.load(sd_flow, device=0, mode=m) for m in ("fp32", "bf16")}
    yield hs
    for h in hs.values():
        h.close()


def _inputs(B, T0, seed=5):
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((B, 192, T0)).astype(np.float32),
            rng.standard_normal((B, 512, 1)).astype(np.float32))


def test_flow_is_loaded(handles):
    assert handles["fp32"].flow_couplings == 4
    assert handles["bf16"].flow_couplings == 4


@pytest.mark.parametrize("T0,lengths", [(1, None), (5, [5, 3]), (24, [24, 11]), (250, [250, 137])])
def test_flow_fp32_matches_oracle(handles, sd_flow, T0, lengths):
    zp, g = _inputs(2, T0)
    ref = oracle.flow_inverse(sd_flow, zp, g, lengths)
    z = handles["fp32"].flow_inverse(zp, g, lengths)
    assert rel_max(z, ref) <= FP32_REL
    if lengths is not None:
        assert not np.any(z[1, :, lengths[1]:])


def test_flow_fp32_without_g(handles, sd_flow):
    zp, _ = _inputs(2, 40)
    ref = oracle.flow_inverse(sd_flow, zp, None, None)
    z = handles["fp32"].flow_inverse(zp, None, None)
    assert rel_max(z, ref) <= FP32_REL


@pytest.mark.parametrize("T0,lengths", [(5, [5, 2]), (250, [250, 90]), (500, None)])
def test_flow_bf16_snr(handles, sd_flow, T0, lengths):
    zp, g = _inputs(2, T0, seed=7)
    ref = oracle.flow_inverse(sd_flow, zp, g, lengths)
    z = handles["bf16"].flow_inverse(zp, g, lengths)
    assert snr_db(z, ref) >= BF16_SNR_DB
    if lengths is not None:
        assert not np.any(z[1, :, lengths[1]:])


@pytest.mark.parametrize("mode", ["fp32", "bf16"])
def test_flow_decode_equals_flow_then_decoder(handles, mode):
    zp, g = _inputs(2, 30, seed=9)
    h = handles[mode]
    z = h.flow_inverse(zp, g, [30, 17])
    wav_a = h.forward(z, g, lengths=[30, 17])
    wav_b = h.flow_decode(zp, g, [30, 17])
    assert np.array_equal(wav_a, wav_b)


def test_flow_device_pointers(handles, sd_flow):
    import torch
    zp, g = _inputs(2, 64, seed=11)
    h = handles["bf16"]
    ref = h.flow_inverse(zp, g, [64, 40])
    zd = torch.from_numpy(zp).cuda()
    gd = torch.from_numpy(g).cuda()
    ld = torch.tensor([64, 40], dtype=torch.int32).cuda()
    out = h.flow_inverse_device(zd, gd, ld)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), ref)
    wav = h.flow_decode_device(zd, gd, ld)
    torch.cuda.synchronize()
    assert np.array_equal(wav.cpu().numpy(), h.flow_decode(zp, g, [64, 40]))


_NO_PDL_CHILD = r"""
import sys
import numpy as np
sys.path.insert(0, sys.argv[1])
from __graft_entry__ import load_package
gsv = load_package()
sd = gsv.synth.make_state_dict(0, init="unit", bias="rand")
sd.update(gsv.synth.make_flow_state_dict(init="unit"))
d = np.load(sys.argv[2])
outs = {}
for mode in ("fp32", "bf16"):
    h = gsv.Decoder.load(sd, device=0, mode=mode)
    outs[mode] = h.flow_inverse(d["zp"], d["g"], [96, 51])
    h.close()
np.savez(sys.argv[3], **outs)
"""


def test_flow_same_with_and_without_dependent_launch(handles, tmp_path):
    """The flow inverse launches with programmatic dependent launch: each
    kernel may be scheduled before the previous one ends and waits on the
    device for it.  A child process with GSVDEC_NO_PDL=1 (strict stream
    order) must produce bit-identical outputs in both modes."""
    import os
    import subprocess
    import sys
    from conftest import ROOT
    zp, g = _inputs(2, 96, seed=13)
    np.savez(tmp_path / "in.npz", zp=zp, g=g)
    env = dict(os.environ, GSVDEC_NO_PDL="1")
    r = subprocess.run([sys.executable, "-c", _NO_PDL_CHILD, str(ROOT), str(tmp_path / "in.npz"),
                        str(tmp_path / "out.npz")], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    ref = np.load(tmp_path / "out.npz")
    for mode in ("fp32", "bf16"):
        assert np.array_equal(handles[mode].flow_inverse(zp, g, [96, 51]), ref[mode]), mode


def test_handle_without_flow_reports_it(gsv):
    d = gsv.Decoder.load(gsv.synth.make_state_dict(0), device=0, mode="bf16")
    try:
        assert d.flow_couplings == 0
        with pytest.raises(gsv.GsvDecError, match="without flow"):
            d.flow_inverse(np.zeros((1, 192, 4), np.float32))
    finally:
        d.close()
