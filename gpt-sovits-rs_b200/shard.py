"""Multi-GPU decode: one process per GPU, torch.distributed for the plumbing.

The decoder has no exchange step: utterances are independent, and inside one
utterance an output frame depends only on a finite window of input frames
(the receptive field, ``Decoder.info["receptive_halo"]`` frames per side).
So work is partitioned with no collective on the data path, and the single
collective is the gather of finished waveform pieces to the output rank:

* a batch (right-padded, per-utterance lengths) is split by utterance with a
  longest-processing-time greedy balance of the frame counts
  (:func:`plan_utterances`), each rank decoding its share as one masked batch;
* one long utterance is split into contiguous frame ranges
  (:func:`plan_chunks`), each rank decoding its range plus ``halo`` input
  frames per side, clamped at the ends, and keeping only its own samples.

The gather uses ``dist.gather`` of equal-size, zero-padded pieces (NCCL over
NVLink on GPUs, gloo on CPU); rank 0 reassembles.  There is no reference
counterpart: the reference runs one device (src/config/mod.rs:68-80).
"""
from __future__ import annotations

from typing import Callable, List, Optional, Sequence, Tuple

import numpy as np


def plan_utterances(lengths: Sequence[int], nranks: int) -> List[List[int]]:
    """Utterance indices per rank, balancing the summed frame counts (LPT).

    Longest first onto the least-loaded rank; ties go to the lower rank, and
    each rank's list is returned in ascending utterance order.
    """
    if nranks <= 0:
        raise ValueError("nranks must be positive")
    order = sorted(range(len(lengths)), key=lambda i: (-int(lengths[i]), i))
    load = [0] * nranks
    out: List[List[int]] = [[] for _ in range(nranks)]
    for i in order:
        r = min(range(nranks), key=lambda k: (load[k], k))
        out[r].append(i)
        load[r] += int(lengths[i])
    return [sorted(x) for x in out]


def plan_buckets(lengths: Sequence[int], max_buckets: int = 8, overhead: int = 300) -> List[List[int]]:
    """Split utterances into at most `max_buckets` batches of similar length.

    A masked batch costs (its size x its longest length) padded frames plus a
    fixed `overhead` (the per-forward launch cost, in frame units); the split
    minimises the total over contiguous runs of the length-sorted order
    (dynamic programming).  Returns lists of indices into `lengths`, each
    ascending, the buckets ordered by length.
    """
    n = len(lengths)
    if n == 0:
        return []
    order = sorted(range(n), key=lambda i: (int(lengths[i]), i))
    ls = [int(lengths[i]) for i in order]
    K = max(1, min(max_buckets, n))
    INF = float("inf")
    # best[k][j]: min cost of the first j sorted utterances in k buckets
    best = [[INF] * (n + 1) for _ in range(K + 1)]
    cut = [[0] * (n + 1) for _ in range(K + 1)]
    best[0][0] = 0.0
    for k in range(1, K + 1):
        for j in range(1, n + 1):
            for i in range(k - 1, j):
                c = best[k - 1][i] + (j - i) * ls[j - 1] + overhead
                if c < best[k][j]:
                    best[k][j], cut[k][j] = c, i
    k = min(range(1, K + 1), key=lambda kk: best[kk][n])
    out, j = [], n
    while k > 0:
        i = cut[k][j]
        out.append(sorted(order[i:j]))
        j, k = i, k - 1
    return out[::-1]


def plan_chunks(T0: int, nranks: int) -> List[Tuple[int, int]]:
    """Contiguous frame ranges [begin, end) covering [0, T0), one per rank
    (sizes differ by at most one frame; trailing ranks may be empty when
    T0 < nranks)."""
    if nranks <= 0 or T0 < 0:
        raise ValueError("bad arguments")
    base, extra = divmod(T0, nranks)
    out, b = [], 0
    for r in range(nranks):
        n = base + (1 if r < extra else 0)
        out.append((b, b + n))
        b += n
    return out


def halo_window(begin: int, end: int, T0: int, halo: int) -> Tuple[int, int]:
    """Input frames a chunk [begin, end) decodes with: the chunk plus `halo`
    frames each side, clamped to the utterance."""
    return max(0, begin - halo), min(T0, end + halo)


def _gather_to_root(piece, n_valid: int, maxlen: int, dist, group, device, as_numpy: bool = True,
                    sizes: Optional[Sequence[int]] = None):
    """Gather variable-length 1-D float32 pieces to rank 0 (zero-padded to
    `maxlen`); returns the list of trimmed pieces on rank 0 (numpy, or device
    tensors with as_numpy=False), else None.  `sizes` (every rank's n_valid,
    known to all ranks from the plan) spares the size exchange: then the only
    collective is the gather itself and nothing waits on the host."""
    import torch
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    if n_valid == maxlen and piece.numel() == maxlen:
        buf = piece.contiguous()
    else:
        buf = torch.zeros(maxlen, dtype=torch.float32, device=device)
        if n_valid:
            buf[:n_valid] = piece[:n_valid]
    if sizes is None:
        mine = torch.tensor([n_valid], dtype=torch.int64, device=device)
        all_sizes = [torch.zeros(1, dtype=torch.int64, device=device) for _ in range(world)]
        dist.all_gather(all_sizes, mine, group=group)
        sizes = [int(t.item()) for t in all_sizes]
    gl = [torch.empty(maxlen, dtype=torch.float32, device=device) for _ in range(world)] if rank == 0 else None
    dist.gather(buf, gather_list=gl, dst=0, group=group)
    if rank != 0:
        return None
    if not as_numpy:
        return [gl[r][: int(sizes[r])] for r in range(world)]
    return [gl[r][: int(sizes[r])].cpu().numpy() for r in range(world)]


def decode_batch_sharded(decode: Callable, z: np.ndarray, g: Optional[np.ndarray],
                         lengths: Sequence[int], hop: int, dist, group=None, device="cpu",
                         max_buckets: int = 8):
    """Decode a right-padded batch across the ranks of `group`.

    `decode(z_b, g_b, lengths_b)` runs one masked batch and returns its
    flattened waveform [n_b * hop * T_b].  Each rank decodes its share in up
    to `max_buckets` length buckets (plan_buckets), so short utterances are
    not padded to the longest one.  Every rank passes the same z / g /
    lengths.  Rank 0 returns the list of per-utterance waveforms (each
    hop * lengths[i] samples), other ranks return None.

    With z (and g) as CUDA tensors the whole path stays on the device: the
    bucket batches are gathered from z on the device, `decode` receives
    device tensors (lengths as an int32 device tensor) and returns a device
    waveform, the pieces are gathered over the process group as device
    tensors, and rank 0 gets device tensors back.

    With host arrays and a CUDA `device`, `decode` also receives device
    tensors: the rank's share of z / g is staged with ONE host-to-device copy
    (pinned), its buckets run on the device with no host sync between them,
    and rank 0 brings the gathered waveform back with ONE device-to-host copy
    into a pinned buffer and returns numpy views of it.  The buffer is reused
    by the next such call: copy the views to keep them past it.
    """
    import torch
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    plan = plan_utterances(lengths, world)
    mine = plan[rank]
    if not isinstance(z, torch.Tensor) and str(device).startswith("cuda"):
        return _decode_staged(decode, z, g, lengths, hop, dist, group, device, max_buckets, plan)
    on_dev = isinstance(z, torch.Tensor)
    if mine:
        parts = {}
        for bucket in plan_buckets([int(lengths[i]) for i in mine], max_buckets):
            idx = [mine[k] for k in bucket]
            lens = [int(lengths[i]) for i in idx]
            T = max(lens)
            if on_dev:
                it = torch.tensor(idx, device=z.device)
                zb = z.index_select(0, it)[:, :, :T].contiguous()
                gb = None if g is None else g.index_select(0, it).contiguous()
                lb = torch.tensor(lens, dtype=torch.int32, device=z.device)
                wav = decode(zb, gb, lb).reshape(len(idx), T * hop)
            else:
                zb = np.ascontiguousarray(z[idx, :, :T])
                gb = None if g is None else np.ascontiguousarray(g[idx])
                wav = np.asarray(decode(zb, gb, lens), np.float32).reshape(len(idx), T * hop)
            for k, i in enumerate(idx):
                parts[i] = wav[k, : lens[k] * hop]
        piece = torch.cat([parts[i] for i in mine]) if on_dev else np.concatenate([parts[i] for i in mine])
    else:
        piece = torch.zeros(0, device=z.device) if on_dev else np.zeros(0, np.float32)
    sizes = [sum(int(lengths[i]) for i in p) * hop for p in plan]
    maxlen = max(max(sizes), 1)
    n_valid = int(piece.numel()) if on_dev else piece.size
    src = piece if on_dev else torch.from_numpy(piece).to(device)
    got = _gather_to_root(src, n_valid, maxlen, dist, group, device, as_numpy=not on_dev, sizes=sizes)
    if got is None:
        return None
    out: List[Optional[np.ndarray]] = [None] * len(lengths)
    for r, idx in enumerate(plan):
        off = 0
        for i in idx:
            n = int(lengths[i]) * hop
            out[i] = got[r][off:off + n]
            off += n
    return out


_PINNED = {}
_PINNED_COPY = {}  # purpose -> event recorded after the last copy out of that buffer


def _pinned(n: int, dtype, purpose: str):
    """A pinned host buffer of at least n elements for one purpose ("z", "g",
    "wav"), reused across calls (page locking hundreds of MB per call would
    cost more than the copy).  Each purpose has its own buffer, and a buffer
    is handed out again only after the last asynchronous copy out of it (see
    _h2d) has finished, so refilling it never races a copy in flight."""
    import torch
    key = (purpose, str(dtype))
    ev = _PINNED_COPY.pop(purpose, None)
    if ev is not None:
        ev.synchronize()
    buf = _PINNED.get(key)
    if buf is None or buf.numel() < n:
        buf = torch.empty(max(n, 1), dtype=dtype, pin_memory=True)
        _PINNED[key] = buf
    return buf[:n]


def _h2d(buf, device, purpose: str):
    """Asynchronous copy of the pinned buffer `buf` to `device`; the buffer
    stays reserved until the copy has run (_pinned waits for it)."""
    import torch
    out = buf.to(device, non_blocking=True)
    ev = torch.cuda.Event()
    ev.record()
    _PINNED_COPY[purpose] = ev
    return out


def _decode_staged(decode, z, g, lengths, hop, dist, group, device, max_buckets, plan):
    """decode_batch_sharded for host arrays on a CUDA device: one H2D of this
    rank's share, device buckets, device gather, one D2H on rank 0."""
    import torch
    rank = dist.get_rank(group)
    mine = plan[rank]
    T0 = int(z.shape[2])
    if mine:
        # This rank's utterances, gathered straight into the pinned buffer (one
        # multi-threaded copy, no temporary), then one asynchronous H2D.
        sel = torch.as_tensor(mine, dtype=torch.int64)
        zs = _pinned(len(mine) * z.shape[1] * T0, torch.float32, "z").view(len(mine), z.shape[1], T0)
        torch.index_select(torch.from_numpy(np.ascontiguousarray(z, np.float32)), 0, sel, out=zs)
        zd = _h2d(zs, device, "z")
        gd = None
        if g is not None:
            gs = _pinned(len(mine) * int(np.prod(g.shape[1:])), torch.float32, "g").view(len(mine), *g.shape[1:])
            torch.index_select(torch.from_numpy(np.ascontiguousarray(g, np.float32)), 0, sel, out=gs)
            gd = _h2d(gs, device, "g")
        local = [int(lengths[i]) for i in mine]
        parts = {}
        for bucket in plan_buckets(local, max_buckets):
            lens = [local[k] for k in bucket]
            T = max(lens)
            it = torch.tensor(bucket, device=device)
            zb = zd.index_select(0, it)[:, :, :T].contiguous()
            gb = None if gd is None else gd.index_select(0, it).contiguous()
            lb = torch.tensor(lens, dtype=torch.int32, device=device)
            wav = decode(zb, gb, lb).reshape(len(bucket), T * hop)
            for k, i in enumerate(bucket):
                parts[mine[i]] = wav[k, : lens[k] * hop]
        piece = torch.cat([parts[i] for i in mine])
    else:
        piece = torch.zeros(0, device=device)
    sizes = [sum(int(lengths[i]) for i in p) * hop for p in plan]
    maxlen = max(1, max(sizes))
    got = _gather_to_root(piece, int(piece.numel()), maxlen, dist, group, device, as_numpy=False, sizes=sizes)
    if got is None:
        return None
    flat = torch.cat(got)
    host = _pinned(flat.numel(), torch.float32, "wav")
    host.copy_(flat)  # one device-to-host copy of every piece
    arr = host.numpy()
    out: List[Optional[np.ndarray]] = [None] * len(lengths)
    off = 0
    for idx in plan:
        for i in idx:
            n = int(lengths[i]) * hop
            out[i] = arr[off:off + n]
            off += n
    return out


def decode_long_chunked(decode_chunk: Callable, T0: int, hop: int, dist, group=None,
                        device="cpu"):
    """Decode one long utterance split in time across the ranks of `group`.

    `decode_chunk(begin, end)` returns the hop * (end - begin) samples of
    frames [begin, end) (computed with its own halo), as numpy or as a device
    tensor (then the pieces are gathered and joined on the device).  Rank 0
    returns the whole waveform, other ranks None.
    """
    import torch
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    chunks = plan_chunks(T0, world)
    b, e = chunks[rank]
    piece = decode_chunk(b, e) if e > b else None
    on_dev = isinstance(piece, torch.Tensor)
    if piece is None:
        piece = np.zeros(0, np.float32)
    sizes = [(ee - bb) * hop for bb, ee in chunks]
    if world == 1:  # the one chunk is the whole waveform: no gather, no device round trip
        return piece if on_dev else np.asarray(piece, np.float32)
    maxlen = max(1, max(sizes))
    n_valid = int(piece.numel()) if on_dev else int(np.asarray(piece).size)
    src = piece if on_dev else torch.from_numpy(np.asarray(piece, np.float32)).to(device)
    got = _gather_to_root(src, n_valid, maxlen, dist, group, device, as_numpy=not on_dev, sizes=sizes)
    if got is None:
        return None
    return torch.cat(got) if on_dev else np.concatenate(got)


def decode_long_staged(decode_chunk: Callable, z: np.ndarray, g: Optional[np.ndarray], hop: int, dist,
                       group=None, device="cuda", halo: int = 16):
    """decode_long_chunked for a host utterance z [1, C, T0] (g [1, gin, 1] or
    None) on a CUDA device: each rank copies only its chunk's input window
    (the chunk plus `halo` frames per side, clamped) into a reused pinned
    buffer and moves it with ONE asynchronous host-to-device copy, decodes it
    on the device with `decode_chunk(zw, gw, begin, end)` (zw [1, C, w] the
    window on the device, [begin, end) the chunk's frames inside it; e.g.
    ``lambda zw, gw, b, e: dec.forward_chunk_device(zw, gw, b, e, halo)``),
    the device pieces are gathered to rank 0, and rank 0 brings the waveform
    back with ONE device-to-host copy into a pinned buffer.  Rank 0 returns a
    numpy view of that buffer (reused by the next such call: copy it to keep
    it), other ranks None.  The samples equal decode_long_chunked's: a chunk
    decoded from its clamped window sees exactly the frames it would see in
    the whole utterance."""
    import torch
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    if z.ndim != 3 or z.shape[0] != 1:
        raise ValueError("z must be [1, C, T0]")
    T0 = int(z.shape[2])
    chunks = plan_chunks(T0, world)
    b, e = chunks[rank]
    sizes = [(ee - bb) * hop for bb, ee in chunks]
    if e > b:
        lo, hi = halo_window(b, e, T0, halo)
        zs = _pinned(z.shape[1] * (hi - lo), torch.float32, "z").view(1, z.shape[1], hi - lo)
        np.copyto(zs.numpy(), z[:, :, lo:hi], casting="same_kind")
        zd = _h2d(zs, device, "z")
        gd = None
        if g is not None:
            gs = _pinned(int(np.prod(g.shape)), torch.float32, "g").view(*g.shape)
            np.copyto(gs.numpy(), g, casting="same_kind")
            gd = _h2d(gs, device, "g")
        piece = decode_chunk(zd, gd, b - lo, e - lo)
    else:
        piece = torch.zeros(0, device=device)
    if world == 1:
        flat = piece
    else:
        got = _gather_to_root(piece, int(piece.numel()), max(1, max(sizes)), dist, group, device,
                              as_numpy=False, sizes=sizes)
        if got is None:
            return None
        flat = torch.cat(got)
    host = _pinned(flat.numel(), torch.float32, "wav")
    host.copy_(flat)  # the one device-to-host copy
    return host.numpy()
