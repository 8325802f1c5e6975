"""gsvdec_forward_multi through the C ABI.

Several handles -- one per GPU when the box has several, else several handles
on device 0, which run as separate workers on separate streams -- must give
every utterance the waveform of the single-handle forward on it alone: bit for
bit in BF16 mode (the masked and the halo-chunked decodes are exact there),
within 1e-5 relative in FP32 mode, whose small launches split their channel
loop by launch size (so a batch and a lone utterance may round differently).
Samples past an utterance's length are 0.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import rel_max

pytestmark = pytest.mark.gpu

HOP = 640


def _devices(n):
    import torch
    k = torch.cuda.device_count()
    return [i % k for i in range(n)]


@pytest.fixture(scope="module")
def sd(gsv):
    return gsv.synth.make_state_dict(0, init="unit", bias="rand")


def _same(got, want, mode):
    if mode == "bf16":
        return np.array_equal(got, want)
    return rel_max(got, want) <= 1e-5


@pytest.mark.parametrize("mode", ["bf16", "fp32"])
def test_multi_batch_matches_each_utterance_alone(gsv, sd, mode):
    decs = [gsv.Decoder.load(sd, device=d, mode=mode) for d in _devices(3)]
    try:
        B, T0 = 7, 40
        lens = np.array([40, 13, 27, 1, 0, 40, 22], np.int32)
        z, g = gsv.synth.make_inputs(B, T0, seed_z=301, seed_g=302)
        got = gsv.forward_multi(decs, z, g, lengths=lens).reshape(B, -1)
        for b in range(B):
            n = int(lens[b])
            if n:
                alone = decs[0].forward(z[b:b + 1, :, :n], g[b:b + 1])
                assert _same(got[b, :HOP * n], alone, mode), b
            assert not got[b, HOP * n:].any(), b
        # without lengths every utterance is whole
        full = gsv.forward_multi(decs, z, g).reshape(B, -1)
        want = decs[1].forward(z, g).reshape(B, -1)
        assert _same(full, want, mode)
    finally:
        for d in decs:
            d.close()


@pytest.mark.parametrize("mode", ["bf16", "fp32"])
def test_multi_long_utterance_in_time_chunks(gsv, sd, mode):
    decs = [gsv.Decoder.load(sd, device=d, mode=mode) for d in _devices(3)]
    try:
        T0 = 90
        z, g = gsv.synth.make_inputs(1, T0, seed_z=311, seed_g=312)
        whole = decs[0].forward(z, g)
        got = gsv.forward_multi(decs, z, g)
        assert _same(got, whole, mode)
        # with a length: the frames past it are not read, the samples are 0
        n = 61
        part = gsv.forward_multi(decs, z, g, lengths=[n])
        alone = decs[0].forward(z[:, :, :n], g)
        assert _same(part[:HOP * n], alone, mode)
        assert not part[HOP * n:].any()
    finally:
        for d in decs:
            d.close()


def test_multi_device_memory_path(gsv, sd):
    """Device pointers on handles[0]'s device, stream-async: the same samples as
    the host-memory call."""
    import torch
    decs = [gsv.Decoder.load(sd, device=d, mode="bf16") for d in _devices(2)]
    try:
        B, T0 = 5, 24
        lens = np.array([24, 3, 0, 17, 9], np.int32)
        z, g = gsv.synth.make_inputs(B, T0, seed_z=321, seed_g=322)
        host = gsv.forward_multi(decs, z, g, lengths=lens)
        dev0 = decs[0].info["device"]
        zt = torch.from_numpy(z).to(f"cuda:{dev0}")
        gt = torch.from_numpy(g).to(f"cuda:{dev0}")
        lt = torch.from_numpy(lens).to(f"cuda:{dev0}")
        out = torch.full((B * T0 * HOP,), float("nan"), device=f"cuda:{dev0}")
        gsv.forward_multi_device(decs, zt, gt, lt, out=out)
        torch.cuda.synchronize(dev0)
        assert np.array_equal(out.cpu().numpy(), host)
        # one utterance in time chunks, device memory
        z1 = torch.from_numpy(z[:1]).to(f"cuda:{dev0}")
        g1 = torch.from_numpy(g[:1]).to(f"cuda:{dev0}")
        o1 = gsv.forward_multi_device(decs, z1, g1)
        torch.cuda.synchronize(dev0)
        assert np.array_equal(o1.cpu().numpy(), decs[0].forward(z[:1], g[:1]))
        for d in decs:
            d.sync_status()
    finally:
        for d in decs:
            d.close()


def test_multi_rejects_bad_handle_lists(gsv, sd):
    a = gsv.Decoder.load(sd, device=0, mode="bf16")
    b = gsv.Decoder.load(sd, device=0, mode="fp32")
    try:
        z, g = gsv.synth.make_inputs(2, 4)
        with pytest.raises(gsv.GsvDecError) as e:
            gsv.forward_multi([a, a], z, g)
        assert e.value.status == "GSV_E_INVALID_ARG"
        with pytest.raises(gsv.GsvDecError) as e:
            gsv.forward_multi([a, b], z, g)
        assert e.value.status == "GSV_E_INVALID_ARG"
        with pytest.raises(gsv.GsvDecError) as e:
            gsv.forward_multi([a], z, g, lengths=[5, 1])  # longer than T0
        assert e.value.status == "GSV_E_INVALID_ARG"
        # a single handle is a plain forward
        assert np.array_equal(gsv.forward_multi([a], z, g), a.forward(z, g))
    finally:
        a.close()
        b.close()


class _Solo:
    """torch.distributed's calls for one process (no process group)."""

    @staticmethod
    def get_rank(group=None):
        return 0

    @staticmethod
    def get_world_size(group=None):
        return 1

    @staticmethod
    def all_gather(out, t, group=None):
        out[0].copy_(t)

    @staticmethod
    def gather(t, gather_list=None, dst=0, group=None):
        gather_list[0].copy_(t)


def test_sharded_host_arrays_match_device_path(gsv, sd):
    """shard.decode_batch_sharded with host arrays on a CUDA device (one pinned
    H2D per input, device buckets, one D2H) gives the device path's samples,
    also on the next call, which refills the same pinned buffers; the
    one-rank long-utterance path returns the whole decode."""
    import torch
    dec = gsv.Decoder.load(sd, device=0, mode="bf16")
    try:
        B, T0 = 9, 30
        lens = np.array([30, 7, 19, 1, 25, 30, 12, 3, 22], np.int32)
        z, g = gsv.synth.make_inputs(B, T0, seed_z=331, seed_g=332)
        decode = lambda zb, gb, lb: dec.forward_device(zb, gb, lb)  # noqa: E731
        zd, gd = torch.from_numpy(z).cuda(), torch.from_numpy(g).cuda()
        want = [w.cpu().numpy() for w in
                gsv.shard.decode_batch_sharded(decode, zd, gd, lens, dec.hop, _Solo, device="cuda")]
        for call in range(2):
            got = gsv.shard.decode_batch_sharded(decode, z, g, lens, dec.hop, _Solo, device="cuda")
            for b in range(B):
                assert np.array_equal(np.asarray(got[b]), want[b]), (call, b)
        whole = dec.forward(z[:1], g[:1])
        one = gsv.shard.decode_long_chunked(lambda b, e: dec.forward_chunk(z[:1], g[:1], b, e, halo=16),
                                            T0, dec.hop, _Solo, device="cuda")
        assert np.array_equal(one, whole)
    finally:
        dec.close()


class _SeqRank:
    """torch.distributed's calls for rank `r` of `w`, the ranks run one after
    the other in this process: a rank's gather leaves its piece in `sink`,
    and rank 0 (run last) collects every rank's piece from it."""

    def __init__(self, r, w, sink):
        self.r, self.w, self.sink = r, w, sink

    def get_rank(self, group=None):
        return self.r

    def get_world_size(self, group=None):
        return self.w

    def gather(self, t, gather_list=None, dst=0, group=None):
        self.sink[self.r] = t.clone()
        if gather_list is not None:
            for k in range(self.w):
                gather_list[k].copy_(self.sink[k])


def test_long_staged_host_path_matches_whole_decode(gsv, sd):
    """shard.decode_long_staged (each rank's halo window copied in, device
    chunk decode, device gather, one D2H on rank 0) gives the whole-utterance
    decode sample for sample, for 1 and 3 ranks (run in turn in this process),
    also on a second call that refills the same pinned buffers."""
    import torch
    dec = gsv.Decoder.load(sd, device=0, mode="bf16")
    try:
        T0, halo = 100, 16
        z, g = gsv.synth.make_inputs(1, T0, seed_z=341, seed_g=342)
        whole = dec.forward(z, g)
        chunk = lambda zw, gw, b, e: dec.forward_chunk_device(zw, gw, b, e, halo=halo)  # noqa: E731
        for w in (1, 3):
            for call in range(2):
                sink = {}
                got = None
                for r in reversed(range(w)):
                    out = gsv.shard.decode_long_staged(chunk, z, g, dec.hop, _SeqRank(r, w, sink),
                                                       device="cuda", halo=halo)
                    if r == 0:
                        got = np.array(out)
                    else:
                        assert out is None
                torch.cuda.synchronize()
                assert np.array_equal(got, whole), (w, call)
    finally:
        dec.close()
