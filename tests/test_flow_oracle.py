"""The flow-inverse oracle (C restatement of ResidualCouplingBlock reverse,
src/models/sovits_flow.rs:341-415, plus z * y_mask, src/models/sovits.rs:394)
against float64 PyTorch fixtures, on CPU."""
from __future__ import annotations

import numpy as np
import pytest

import oracle


@pytest.mark.parametrize("init", ["unit", "n001"])
def test_flow_generator_is_stable(gsv, flow_golden, init):
    sd = gsv.synth.make_flow_state_dict(init=init)
    assert gsv.synth.checksum(sd) == pytest.approx(float(flow_golden[f"{init}_checksum"]), rel=1e-9)


@pytest.mark.parametrize("init", ["unit", "n001"])
@pytest.mark.parametrize("T0", [1, 5, 24])
def test_oracle_flow_matches_golden(gsv, flow_golden, init, T0):
    sd = gsv.synth.make_flow_state_dict(init=init)
    zp, g, ln = flow_golden[f"T{T0}_zp"], flow_golden[f"T{T0}_g"], flow_golden[f"T{T0}_len"]
    ref = flow_golden[f"{init}_T{T0}_z"]
    z = oracle.flow_inverse(sd, zp, g, ln)
    scale = max(1.0, float(np.abs(ref).max()))
    assert np.abs(z - ref).max() <= 1e-5 * scale
    # masked frames are exactly zero (z * y_mask)
    assert not np.any(z[1, :, int(ln[1]):])
    ref2 = flow_golden[f"{init}_T{T0}_z_nog"]
    z2 = oracle.flow_inverse(sd, zp, None, None)
    assert np.abs(z2 - ref2).max() <= 1e-5 * max(1.0, float(np.abs(ref2).max()))


def test_oracle_flow_float_accumulation_close(gsv, flow_golden):
    sd = gsv.synth.make_flow_state_dict(init="unit")
    zp, g, ln = flow_golden["T24_zp"], flow_golden["T24_g"], flow_golden["T24_len"]
    a = oracle.flow_inverse(sd, zp, g, ln, acc64=True)
    b = oracle.flow_inverse(sd, zp, g, ln, acc64=False)
    assert np.abs(a - b).max() <= 1e-4 * max(1.0, float(np.abs(a).max()))


def test_oracle_flow_reports_missing_keys(gsv):
    sd = gsv.synth.make_flow_state_dict(init="unit")
    del sd["flow.flows.2.enc.res_skip_layers.1.weight_v"]
    with pytest.raises(oracle.OracleError, match="res_skip_layers.1"):
        oracle.flow_inverse(sd, np.zeros((1, 192, 4), np.float32))
    with pytest.raises(oracle.OracleError, match="no flow coupling layers"):
        oracle.flow_inverse({}, np.zeros((1, 192, 4), np.float32))
