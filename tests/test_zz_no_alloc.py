"""The allocation-free forward (gsvdec_forward_noalloc) through the C ABI.

Callers such as a real-time audio callback, or a server whose device memory
belongs to its own pool allocator, cannot cudaMalloc while they decode.  The
allocation-free entry point serves them from a static device array.  On a
fresh handle it must never give the handle a workspace nor take device memory
(after the library's module, static array included, is resident), and it must
give the waveform of the regular device-memory forward call after call: bit
for bit in BF16 and FP32_TC modes (the same kernels on the same inputs; the
latter's three-piece activations fit about 45 frames), within 1e-5 in
FP32 mode (whose small launches may split their channel loop differently in
the smaller static scratch); requests that do not fit the array are refused.  This file is collected last so that a
stop-at-first-failure run has executed every other test first.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("mode", ["bf16", "fp32", "fp32tc"])
def test_noalloc_matches_forward_on_two_calls(gsv, mode):
    import torch
    sd = gsv.synth.make_state_dict(3, init="unit", bias="rand")
    dec = gsv.Decoder.load(sd, device=0, mode=mode)  # fresh: no workspace yet
    ref_dec = gsv.Decoder.load(sd, device=0, mode=mode)
    try:
        sizes = ((2, 20, 101), (1, 40, 202)) if mode == "fp32tc" else ((2, 24, 101), (1, 40, 202))
        for call, (B, T0, seed) in enumerate(sizes):
            z, g = gsv.synth.make_inputs(B, T0, seed_z=seed, seed_g=seed + 1)
            zt = torch.from_numpy(z).cuda()
            gt = torch.from_numpy(g).cuda()
            out = torch.full((B * T0 * dec.hop,), float("nan"), device="cuda")
            torch.cuda.synchronize()
            free0 = torch.cuda.mem_get_info()[0]
            dec.forward_noalloc(zt, gt, out=out)
            torch.cuda.synchronize()
            if call > 0:  # the first call may still load the library's module
                assert torch.cuda.mem_get_info()[0] == free0, call
            assert dec.workspace_bytes() == 0, call
            want = ref_dec.forward_device(zt, gt)
            torch.cuda.synchronize()
            if mode in ("bf16", "fp32tc"):
                assert torch.equal(out, want), call
            else:
                # FP32 splits small launches over their input channels into
                # scratch; the static array leaves less of it than the regular
                # workspace, so a launch may split differently and round
                # differently (in the last bits).
                got, ref = out.double(), want.double()
                assert float((got - ref).abs().max() / ref.abs().max()) <= 1e-5, call
        dec.sync_status()
    finally:
        dec.close()
        ref_dec.close()


def test_noalloc_lengths_timing_and_limit(gsv):
    import torch
    sd = gsv.synth.make_state_dict(3, init="unit", bias="rand")
    dec = gsv.Decoder.load(sd, device=0, mode="bf16")
    ref_dec = gsv.Decoder.load(sd, device=0, mode="bf16")
    try:
        z, g = gsv.synth.make_inputs(3, 16, seed_z=5, seed_g=6)
        lens = torch.tensor([16, 9, 2], dtype=torch.int32, device="cuda")
        zt, gt = torch.from_numpy(z).cuda(), torch.from_numpy(g).cuda()
        want = ref_dec.forward_device(zt, gt, lengths=lens)
        dec.set_stage_timing(1)
        got = dec.forward_noalloc(zt, gt, lengths=lens)
        times = dec.stage_times()  # this call's own stage timers
        dec.set_stage_timing(0)
        torch.cuda.synchronize()
        assert torch.equal(got, want)
        assert times["total"] > 0 and times["resblocks"] > 0
        assert dec.workspace_bytes() == 0
        cap = gsv.library().gsvdec_noalloc_scratch_bytes()
        assert cap == 32 << 20
        big = torch.zeros((4, 192, 500), device="cuda")
        with pytest.raises(gsv.GsvDecError) as e:
            dec.forward_noalloc(big, None)
        assert e.value.status == "GSV_E_INVALID_ARG"
        assert "static scratch" in str(e.value)
        huge = torch.zeros((1, 192, 1), device="cuda")
        lib = gsv.library()
        import ctypes
        rc = lib.gsvdec_forward_noalloc(dec._h, ctypes.c_void_p(huge.data_ptr()), None, None, 1 << 20, 1 << 20,
                                        ctypes.c_void_p(huge.data_ptr()), None)
        assert rc == -1 and "static scratch" in lib.gsvdec_last_error().decode()
    finally:
        dec.close()
        ref_dec.close()
