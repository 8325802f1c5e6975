"""The allocation-free forward (gsvdec_forward_noalloc) through the C ABI.

Callers such as a real-time audio callback, or a server whose device memory
belongs to its own pool allocator, cannot cudaMalloc while they decode.  The
allocation-free entry point serves them from a static device array; it must
give the same waveform as the regular device-memory forward, call after
call, and refuse requests that do not fit the array.  This file is collected
last so that a stop-at-first-failure run has executed every other test first.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

FP32_REL = 1e-4  # the fp32 parity bar used across the GPU tests


def _rel_max(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.mark.parametrize("mode", ["bf16", "fp32"])
def test_noalloc_matches_forward_on_two_calls(gsv, mode):
    import torch
    sd = gsv.synth.make_state_dict(3, init="unit", bias="rand")
    dec = gsv.Decoder.load(sd, device=0, mode=mode)
    for call, (B, T0, seed) in enumerate(((2, 24, 101), (1, 40, 202))):
        z, g = gsv.synth.make_inputs(B, T0, seed_z=seed, seed_g=seed + 1)
        zt = torch.from_numpy(z).cuda()
        gt = torch.from_numpy(g).cuda()
        ref = dec.forward_device(zt, gt)
        out = torch.full((B * T0 * dec.hop,), float("nan"), device="cuda")
        dec.forward_noalloc(zt, gt, out=out)
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        want = ref.cpu().numpy()
        assert np.isfinite(got).all(), call
        assert _rel_max(got, want) <= FP32_REL, call
    dec.close()


def test_noalloc_lengths_and_limit(gsv):
    import torch
    sd = gsv.synth.make_state_dict(3, init="unit", bias="rand")
    dec = gsv.Decoder.load(sd, device=0, mode="bf16")
    z, g = gsv.synth.make_inputs(3, 16, seed_z=5, seed_g=6)
    lens = torch.tensor([16, 9, 2], dtype=torch.int32, device="cuda")
    zt, gt = torch.from_numpy(z).cuda(), torch.from_numpy(g).cuda()
    ref = dec.forward_device(zt, gt, lengths=lens)
    got = dec.forward_noalloc(zt, gt, lengths=lens)
    torch.cuda.synchronize()
    assert _rel_max(got.cpu().numpy(), ref.cpu().numpy()) <= FP32_REL
    cap = gsv.library().gsvdec_noalloc_scratch_bytes()
    assert cap == 32 << 20
    big = torch.zeros((4, 192, 500), device="cuda")
    with pytest.raises(gsv.GsvDecError) as e:
        dec.forward_noalloc(big, None)
    assert e.value.status == "GSV_E_INVALID_ARG"
    assert "static scratch" in str(e.value)
    dec.close()
