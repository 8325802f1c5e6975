"""Failure paths on the GPU, made on purpose without faulting it.

* A bounded device wait that runs out: gsvdec_selftest_wait queues a kernel
  whose wait (the library's own hand-off wait) is on a barrier nothing
  completes, limited to 1 ms; nothing else is in flight in it.  The give-up
  must surface as GSV_E_TIMEOUT from gsvdec_sync_status, from the entry of
  the next call on the handle, or from a host-memory call, and the handle must
  keep working afterwards.
* Device allocation failure through the allocation-failure hook: GSV_E_OOM
  from gsvdec_create and from a forward that needs a workspace, with the
  handle still usable once allocations succeed again.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LIMIT_NS = 1_000_000  # 1 ms


@pytest.fixture(scope="module")
def sd(gsv):
    return gsv.synth.make_state_dict(2, init="unit", bias="rand")


@pytest.fixture(scope="module")
def dec(gsv, sd):
    d = gsv.Decoder.load(sd, device=0, mode="bf16")
    yield d
    d.close()


def test_giveup_reported_by_sync_status(gsv, dec):
    z, g = gsv.synth.make_inputs(2, 6, seed_z=401, seed_g=402)
    ref = dec.forward(z, g)
    dec.selftest_wait(LIMIT_NS)  # stream-async: returns before the kernel ran
    with pytest.raises(gsv.GsvDecError) as e:
        dec.sync_status()
    assert e.value.status == "GSV_E_TIMEOUT"
    dec.sync_status()  # reported once, then cleared
    assert np.array_equal(dec.forward(z, g), ref)


def test_giveup_reported_at_entry_of_next_call(gsv, dec):
    import torch
    z, g = gsv.synth.make_inputs(2, 6, seed_z=403, seed_g=404)
    zt, gt = torch.from_numpy(z).cuda(), torch.from_numpy(g).cuda()
    ref = dec.forward_device(zt, gt).clone()
    dec.selftest_wait(LIMIT_NS)
    torch.cuda.synchronize()
    with pytest.raises(gsv.GsvDecError) as e:
        dec.forward_device(zt, gt)  # reports the earlier call's give-up, does nothing else
    assert e.value.status == "GSV_E_TIMEOUT"
    assert "earlier" in str(e.value)
    out = dec.forward_device(zt, gt)  # proceeds
    dec.sync_status()
    assert torch.equal(out, ref)


def test_giveup_reported_by_host_memory_call(gsv, dec):
    z, g = gsv.synth.make_inputs(1, 5, seed_z=405, seed_g=406)
    ref = dec.forward(z, g)
    dec.selftest_wait(LIMIT_NS)
    with pytest.raises(gsv.GsvDecError) as e:
        dec.forward(z, g)  # at its entry or after its own sync, whichever sees it
    assert e.value.status == "GSV_E_TIMEOUT"
    assert np.array_equal(dec.forward(z, g), ref)


def test_selftest_limit_is_validated(gsv, dec):
    with pytest.raises(gsv.GsvDecError) as e:
        dec.selftest_wait(10)
    assert e.value.status == "GSV_E_INVALID_ARG"


def test_allocation_failure_hook(gsv, sd):
    z, g = gsv.synth.make_inputs(2, 7, seed_z=407, seed_g=408)
    try:
        gsv.set_alloc_fail_after(0)
        with pytest.raises(gsv.GsvDecError) as e:
            gsv.Decoder.load(sd, device=0, mode="bf16")
        assert e.value.status == "GSV_E_OOM"
        gsv.set_alloc_fail_after(2)  # a few weight uploads succeed, then one fails
        with pytest.raises(gsv.GsvDecError) as e:
            gsv.Decoder.load(sd, device=0, mode="bf16")
        assert e.value.status == "GSV_E_OOM"
    finally:
        gsv.set_alloc_fail_after(-1)
    d = gsv.Decoder.load(sd, device=0, mode="bf16")
    try:
        assert d.workspace_bytes() == 0
        gsv.set_alloc_fail_after(0)
        try:
            with pytest.raises(gsv.GsvDecError) as e:
                d.forward(z, g)  # its first call needs a workspace
            assert e.value.status == "GSV_E_OOM"
        finally:
            gsv.set_alloc_fail_after(-1)
        assert d.workspace_bytes() == 0
        ref = gsv.Decoder.load(sd, device=0, mode="bf16")
        try:
            assert np.array_equal(d.forward(z, g), ref.forward(z, g))
        finally:
            ref.close()
        assert d.workspace_bytes() > 0
    finally:
        d.close()
