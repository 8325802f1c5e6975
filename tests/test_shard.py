"""Multi-process decode plumbing on CPU: planners, and world_size-2 gloo runs
of the utterance-sharded batch and the halo-chunked long utterance, with the
CPU oracle standing in for the per-rank decoder.  Also a rank that dies
before the gather: the survivor must fail fast, not hang."""
from __future__ import annotations

import os
import socket
import sys
import traceback
from pathlib import Path

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]
HOP = 640


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_plan_utterances_balances_and_covers(gsv):
    shard = gsv.shard
    rng = np.random.default_rng(0)
    for n, world in ((256, 8), (17, 4), (3, 4), (1, 2)):
        lens = rng.integers(100, 1001, n)
        plan = shard.plan_utterances(lens, world)
        flat = sorted(i for p in plan for i in p)
        assert flat == list(range(n))
        loads = [sum(int(lens[i]) for i in p) for p in plan]
        assert max(loads) - min(loads) <= int(lens.max())
        assert plan == shard.plan_utterances(lens, world)  # deterministic


def test_plan_buckets_cover_and_minimise_padding(gsv):
    import itertools
    shard = gsv.shard
    rng = np.random.default_rng(1)
    for n in (1, 2, 5, 7):
        lens = [int(x) for x in rng.integers(100, 1001, n)]
        for K in (1, 2, 3):
            plan = shard.plan_buckets(lens, K, overhead=300)
            assert sorted(i for b in plan for i in b) == list(range(n))
            assert len(plan) <= K and all(b == sorted(b) for b in plan)
            cost = sum(len(b) * max(lens[i] for i in b) + 300 for b in plan)
            # brute force over cut points of the length-sorted order
            order = sorted(range(n), key=lambda i: (lens[i], i))
            best = None
            for k in range(1, min(K, n) + 1):
                for cuts in itertools.combinations(range(1, n), k - 1):
                    edges = (0,) + cuts + (n,)
                    c = sum((edges[j + 1] - edges[j]) * lens[order[edges[j + 1] - 1]] + 300 for j in range(k))
                    best = c if best is None else min(best, c)
            assert cost == best
    assert shard.plan_buckets([500] * 6, 8) == [list(range(6))]  # equal lengths: one batch
    assert shard.plan_buckets([], 8) == []


def test_plan_chunks_cover_contiguously(gsv):
    shard = gsv.shard
    for T0, world in ((3000, 8), (3000, 1), (5, 8), (11, 3)):
        ch = shard.plan_chunks(T0, world)
        assert ch[0][0] == 0 and ch[-1][1] == T0
        assert all(ch[i][1] == ch[i + 1][0] for i in range(world - 1))
        sizes = [e - b for b, e in ch]
        assert max(sizes) - min(sizes) <= 1
    assert gsv.shard.halo_window(0, 10, 100, 16) == (0, 26)
    assert gsv.shard.halo_window(50, 60, 70, 16) == (34, 70)


def _worker(rank, world, port, mode, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world))
    sys.path[:0] = [str(ROOT), str(ROOT / "tests")]
    import datetime

    import torch.distributed as dist

    import oracle
    from __graft_entry__ import load_package
    gsv = load_package()
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=20))
    try:
        sd = gsv.synth.make_state_dict(5, init="unit", bias="rand")
        if mode == "batch":
            lens = [6, 3, 5, 2, 4]
            z, g = gsv.synth.make_inputs(len(lens), max(lens), seed_z=7, seed_g=8)

            def decode(zb, gb, lb):
                T = zb.shape[2]
                out = np.zeros((zb.shape[0], T * HOP), np.float32)
                for k, n in enumerate(lb):
                    out[k, : n * HOP] = oracle.decoder_forward(sd, zb[k:k + 1, :, :n], gb[k:k + 1])
                return out.reshape(-1)

            res = gsv.shard.decode_batch_sharded(decode, z, g, lens, HOP, dist)
            if rank == 0:
                np.savez(out_dir / "batch.npz", *res)
        elif mode == "chunk":
            T0, halo = 40, 16
            z, g = gsv.synth.make_inputs(1, T0, seed_z=9, seed_g=10)

            def decode_chunk(b, e):
                lo, hi = gsv.shard.halo_window(b, e, T0, halo)
                w = oracle.decoder_forward(sd, z[:, :, lo:hi], g)
                return w[(b - lo) * HOP:(e - lo) * HOP]

            res = gsv.shard.decode_long_chunked(decode_chunk, T0, HOP, dist)
            if rank == 0:
                np.save(out_dir / "chunk.npy", res)
        elif mode == "dead":
            if rank == 1:
                os._exit(0)  # leaves without joining the gather
            try:
                gsv.shard.decode_long_chunked(lambda b, e: np.zeros((e - b) * HOP, np.float32),
                                              8, HOP, dist)
                (out_dir / "dead.txt").write_text("returned")
            except Exception as exc:  # the expected path: a bounded failure
                (out_dir / "dead.txt").write_text("raised " + type(exc).__name__)
            os._exit(0)
    except Exception:
        (out_dir / f"err{rank}.txt").write_text(traceback.format_exc())
        raise
    finally:
        if mode != "dead":
            dist.destroy_process_group()


def _run(mode, tmp_path, world=2):
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, tmp_path)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
        if p.is_alive():
            p.kill()
            pytest.fail(f"{mode}: a rank did not finish")
    for r in range(world):
        f = tmp_path / f"err{r}.txt"
        if f.exists():
            pytest.fail(f.read_text())


def test_batch_sharded_over_two_gloo_ranks(gsv, tmp_path):
    import oracle
    _run("batch", tmp_path)
    got = np.load(tmp_path / "batch.npz")
    sd = gsv.synth.make_state_dict(5, init="unit", bias="rand")
    lens = [6, 3, 5, 2, 4]
    z, g = gsv.synth.make_inputs(len(lens), max(lens), seed_z=7, seed_g=8)
    for i, n in enumerate(lens):
        ref = oracle.decoder_forward(sd, z[i:i + 1, :, :n], g[i:i + 1])
        assert np.array_equal(got[f"arr_{i}"], ref)


def test_long_utterance_chunked_over_two_gloo_ranks(gsv, tmp_path):
    import oracle
    _run("chunk", tmp_path)
    got = np.load(tmp_path / "chunk.npy")
    sd = gsv.synth.make_state_dict(5, init="unit", bias="rand")
    z, g = gsv.synth.make_inputs(1, 40, seed_z=9, seed_g=10)
    ref = oracle.decoder_forward(sd, z, g)
    assert got.shape == ref.shape
    assert np.abs(got - ref).max() <= 1e-6 * np.abs(ref).max()


def test_dead_rank_fails_fast(gsv, tmp_path):
    _run("dead", tmp_path)
    assert (tmp_path / "dead.txt").read_text().startswith("raised")


def test_c_abi_plan_matches_python_planner(gsv):
    """gsvdec_plan_multi (the C++ planner behind gsvdec_forward_multi) makes the
    same utterance shares and length buckets as shard.plan_utterances /
    shard.plan_buckets, and leaves empty utterances out."""
    shard = gsv.shard
    rng = np.random.default_rng(7)
    for n, world in ((256, 8), (256, 1), (33, 4), (5, 8), (1, 1), (40, 3)):
        lens = rng.integers(1, 1001, n).astype(np.int32)
        worker, bucket = gsv.plan_multi(lens, world, T0=1000)
        plan = shard.plan_utterances(lens, world)
        for r, mine in enumerate(plan):
            assert sorted(np.nonzero(worker == r)[0].tolist()) == mine
            bks = shard.plan_buckets([int(lens[i]) for i in mine], 8, overhead=300)
            for k, bk in enumerate(bks):
                assert sorted(np.nonzero((worker == r) & (bucket == k))[0].tolist()) == [mine[i] for i in bk]
            assert int((worker == r).sum()) == len(mine)
    lens = np.array([5, 0, 7, 0], np.int32)
    worker, bucket = gsv.plan_multi(lens, 2, T0=8)
    assert worker[1] == -1 and worker[3] == -1 and bucket[1] == -1
    assert set(worker[[0, 2]].tolist()) == {0, 1}
    with pytest.raises(gsv.GsvDecError):
        gsv.plan_multi(np.array([9], np.int32), 2, T0=8)  # longer than T0
