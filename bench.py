#!/usr/bin/env python
"""Throughput of the SoVITS v2 Generator (vocoder) on B200, one JSON line.

Workload (one "step"): one decoder forward over a batch of 16 utterances of
10 s each -- z [16, 192, 500] ~ N(0,1), speaker g [16, 512, 1] ~ N(0,1),
random-init weights N(0, 0.01) with zero bias (seeded; no checkpoints
offline) -- giving 16 x 320 000 samples at 32 kHz.  Every rank decodes its own
batch (utterances are independent units: weak scaling, no collective on the
data path).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--mode bf16|fp32|fp32tc]
    python bench.py --impl reference ...   # the CPU reference arm

value     audio-seconds per second, whole job, inputs resident in HBM.
e2e       the same metric through the public C-ABI call with host buffers
          (H2D of z/g and D2H of the waveform inside every timed step):
          gsvdec_forward with GSV_MEM_HOST_ASYNC on pinned buffers (one step's
          copies overlap the neighbouring steps' decodes); e2e.blocking is the
          blocking GSV_MEM_HOST call.
extra keys, the other configs of the same job in the same run:
          varlen256  256 utterances of 2-20 s, length-masked, sharded by
                     utterance over the N ranks (strong scaling), with parity;
          long60     one 60 s utterance in N halo time chunks (strong
                     scaling), with parity;
          fp32_cfg1  the fp32 CUDA-core mode on batch 1 x 5 s, with its
                     roofline against the FP32 peak (rank 0);
          fp32tc_cfg1  the same config in the fp32tc mode (fp32 accuracy on
                     the tensor cores, three bf16 pieces per value), against
                     the measured bf16 peak / 6 (rank 0);
          bf16_cfg1  the bf16 mode's latency on batch 1 x 5 s, device-resident
                     and through the blocking host-memory call (rank 0).
          With N > 1 the headline's waveforms are gathered to rank 0 over NCCL
          inside the timed region too.
roofline  the dominant kernel (the 128-channel tap GEMM, every launch of it):
          achieved = algorithmic FLOPs / launch time (CUDA events around
          every launch on the forward's stream); traffic from a single-launch
          ncu capture; layer_roofline adds the
          layer-weighted fraction sum(t_roof) / sum(t_measured), t_roof =
          max(FLOPs / tensor peak, bytes / HBM peak) per conv; roofline_by_bound
          splits the same launches into compute-bound (TF/s against the tensor
          peak) and HBM-bound (GB/s against the HBM peak).
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "decoder audio-sec/sec at B=16×10 s bf16, 1/2/4/8 B200; % layer roofline"
UNIT = "audio-s/s"
SAMPLE_RATE = 32000
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
# FP32 CUDA-core peak, nominal: 148 SMs x 128 lanes x 2 FLOP x 1.965 GHz.
FP32_CORE_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12


def log(*a):
    print(*a, file=sys.stderr, flush=True)


# Where the one JSON result line goes: stdout, or (under torchrun) a saved copy
# of it while file descriptor 1 itself points at stderr, so that banners that
# native libraries print to stdout (NCCL's version line) stay out of it.
_JSON_FD = None


def emit(obj):
    line = json.dumps(obj) + "\n"
    if _JSON_FD is None:
        sys.stdout.write(line)
        sys.stdout.flush()
    else:
        os.write(_JSON_FD, line.encode())


def keep_stdout_for_json():
    global _JSON_FD
    if _JSON_FD is None:
        sys.stdout.flush()
        _JSON_FD = os.dup(1)
        os.dup2(2, 1)


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=5)
        sm, smax, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def audio_seconds(B: int, T0: int, hop: int) -> float:
    return B * T0 * hop / SAMPLE_RATE


def cpu_port_sample(sd, z, g, min_seconds=10.0, max_reps=4):
    """The oracle port (float accumulation, all host threads) on one utterance."""
    import oracle
    oracle.build()
    threads = os.cpu_count() or 1
    oracle.decoder_forward(sd, z[:, :, :8], g, acc64=False, nthreads=threads)  # warm
    reps, t0 = 0, time.perf_counter()
    while True:
        oracle.decoder_forward(sd, z, g, acc64=False, nthreads=threads)
        reps += 1
        el = time.perf_counter() - t0
        if el >= min_seconds or reps >= max_reps:
            break
    return reps, el, threads


def run_reference(args, ws, rank):
    """CPU reference arm: the C restatement of the reference decoder (the
    Candle crate cannot be built here: no Rust toolchain), all host threads,
    each step one 10 s utterance of the same workload."""
    if rank != 0:
        return
    import oracle
    gsv = load_pkg()
    sd = gsv.synth.make_state_dict(0, init="n001", bias="zero")
    z, g = gsv.synth.make_inputs(args.batch, args.frames)
    z1, g1 = z[:1], g[:1]
    oracle.build()
    threads = os.cpu_count() or 1
    for _ in range(args.warmup):
        oracle.decoder_forward(sd, z1, g1, acc64=False, nthreads=threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.decoder_forward(sd, z1, g1, acc64=False, nthreads=threads)
    el = time.perf_counter() - t0
    secs = audio_seconds(1, args.frames, 640) * args.steps
    value = secs / el
    sample = f"1 utterance x {args.frames / 50:g} s (z [1,192,{args.frames}]) per step"
    emit({
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * el / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: seeded N(0,1) z/g, N(0,0.01) random-init weights, zero bias",
        "config": {"workload": f"B={args.batch} x {args.frames / 50:g} s Generator decode, "
                               "sampled one utterance per step on the host CPU",
                   "batch": args.batch, "frames": args.frames},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    })


def load_pkg():
    from __graft_entry__ import load_package
    return load_package()


def layer_roofline(stats, mode, pk):
    """sum(t_roof) / sum(t_meas) over every launch; t_roof of a launch is the
    sum over the reference convs it computes of max(F / P, bytes / BW), each
    conv's F and bytes counted as if it ran alone (unfused layer I/O)."""
    p_tensor = pk.get("bf16_tflops_sustained", pk.get("bf16_tflops")) * 1e12
    # fp32tc: six bf16 tensor-core products per fp32 product
    p_comp = {"bf16": p_tensor, "fp32tc": p_tensor / 6}.get(mode, FP32_CORE_TFLOPS * 1e12)
    bw = pk["hbm_gbs"] * 1e9
    rows, roof, meas = [], 0.0, 0.0
    for s in stats:
        t_meas = s["ms"] / 1e3
        if s["kind"] in (0, 2):
            t_roof = sum(max(f / p_comp, b / bw) for f, b in zip(s["conv_flops"], s["conv_bytes"]))
            comp = s["flops"] / p_comp
        else:
            comp = 0.0
            t_roof = s["bytes"] / bw
        roof += t_roof
        meas += t_meas
        rows.append({"name": s["name"], "ms": round(s["ms"], 4),
                     "roof_ms": round(1e3 * t_roof, 4),
                     "frac": round(t_roof / t_meas, 3) if t_meas > 0 else None,
                     "bound": "hbm" if s["bytes"] / bw >= comp else "compute"})
    return roof, meas, rows


def roofline_by_bound(stats, mode, pk):
    """The tap-GEMM launches split by what bounds each one (algorithmic FLOPs
    against the compute peak vs algorithmic bytes against HBM): compute-bound
    launches report achieved TF/s against the compute peak, HBM-bound ones
    achieved GB/s against the HBM peak."""
    p_tensor = pk.get("bf16_tflops_sustained", pk.get("bf16_tflops"))
    p_comp = {"bf16": p_tensor, "fp32tc": p_tensor / 6}.get(mode, FP32_CORE_TFLOPS) * 1e12
    bw = pk["hbm_gbs"] * 1e9
    acc = {"compute": [0, 0.0, 0.0, 0.0], "hbm": [0, 0.0, 0.0, 0.0]}  # launches, flops, bytes, seconds
    for s in stats:
        if s["kind"] != 0 or s["ms"] <= 0:
            continue
        a = acc["hbm" if s["bytes"] / bw >= s["flops"] / p_comp else "compute"]
        a[0] += 1
        a[1] += s["flops"]
        a[2] += s["bytes"]
        a[3] += s["ms"] / 1e3
    out = {}
    n, f, _, t = acc["compute"]
    if t > 0:
        out["compute"] = {"launches": n, "achieved": f / t / 1e12, "peak": p_comp / 1e12, "unit": "TFLOP/s",
                          "frac": f / t / p_comp, "share_of_time": None}
    n, _, b, t2 = acc["hbm"]
    if t2 > 0:
        out["hbm"] = {"launches": n, "achieved": b / t2 / 1e9, "peak": bw / 1e9, "unit": "GB/s",
                      "frac": b / t2 / bw, "share_of_time": None}
    tot = acc["compute"][3] + acc["hbm"][3]
    for k, v in out.items():
        v["share_of_time"] = acc[k][3] / tot
    return out


def run_sweep(args):
    """Every distinct conv shape of the Generator (conv_pre, the 5 ConvTranspose,
    the 9 (k, d) ResBlock shapes of each of the 5 widths, conv_post), fed
    N(0,1) activations, timed on the device (CUDA events around the conv launch
    only), reported against its own roofline."""
    import torch
    gsv = load_pkg()
    pk, pk_kind = peaks()
    B = 64 if args.batch == 16 else args.batch
    T0 = args.frames
    sd = gsv.synth.make_state_dict(0, init="n001", bias="zero")
    dec = gsv.Decoder.load(sd, device=0, mode=args.mode)
    Ls = [T0]
    for s in (10, 8, 2, 2, 2):
        Ls.append(Ls[-1] * s)
    shapes = [("dec.conv_pre", 192, T0)]
    for i in range(5):
        shapes.append((f"dec.ups.{i}", (512, 256, 128, 64, 32)[i], Ls[i]))
        for r in range(3):
            for j in range(3):
                shapes.append((f"dec.resblocks.{3 * i + r}.convs1.{j}", (256, 128, 64, 32, 16)[i], Ls[i + 1]))
    shapes.append(("dec.conv_post", 16, Ls[5]))
    p_comp = (pk.get("bf16_tflops_sustained", pk["bf16_tflops"]) if args.mode == "bf16"
              else FP32_CORE_TFLOPS) * 1e12
    bw = pk["hbm_gbs"] * 1e9
    rows = []
    gen = torch.Generator(device="cuda").manual_seed(0)
    for name, cin, L in shapes:
        x = torch.randn((B, cin, L), device="cuda", generator=gen)
        if name == "dec.conv_post":
            cout, lout = 1, L
        else:
            cout, lout = dec._layer_out(name, L)
        y = torch.empty((B, cout, lout), device="cuda")
        for _ in range(2):
            dec.layer_forward_device(name, x, y)
        dec.set_stage_timing(2)
        for _ in range(3):
            dec.layer_forward_device(name, x, y)
        st = [s for s in dec.launch_stats() if s["name"] == name][0]
        dec.set_stage_timing(0)
        t = st["ms"] / 1e3
        f, by = st["flops"], st["bytes"]
        t_roof = max(f / p_comp, by / bw)
        bound = "hbm" if by / bw >= f / p_comp else ("tensor" if args.mode == "bf16" else "fp32-core")
        rows.append({"layer": name, "cin": cin, "cout": cout, "L_in": L, "ms": round(1e3 * t, 4),
                     "tflops": round(f / t / 1e12, 2), "gbs": round(by / t / 1e9, 1), "bound": bound,
                     "roof_ms": round(1e3 * t_roof, 4), "frac": round(t_roof / t, 3)})
        log(f"{name:<28s} {cin:4d}->{cout:<4d} L={L:<7d} {1e3 * t:8.3f} ms  {f / t / 1e12:7.1f} TF/s "
            f"{by / t / 1e9:7.0f} GB/s  {bound:<9s} frac {t_roof / t:.3f}")
        del x, y
        torch.cuda.empty_cache()
    tot_roof = sum(r["roof_ms"] for r in rows)
    tot = sum(r["ms"] for r in rows)
    emit({"workload": f"per-layer sweep, B={B} x {T0 / 50:g} s, {args.mode}",
          "peaks": pk_kind, "layers": rows, "sum_ms": tot, "sum_roof_ms": tot_roof,
          "frac": tot_roof / tot})
    dec.close()


def run_flow(args):
    """The flow inverse before the decoder (ResidualCouplingBlock reverse +
    y_mask, src/models/sovits.rs:389-394) at B x T0 frames on one GPU: the flow
    alone and flow + decoder, device-resident inputs, CUDA events around K
    steps; the flow's layer-weighted roofline from per-launch events; the CPU
    oracle on one utterance as the baseline."""
    import torch
    gsv = load_pkg()
    pk, pk_kind = peaks()
    sd = gsv.synth.make_state_dict(0, init="n001", bias="zero")
    sd.update(gsv.synth.make_flow_state_dict(init="n001", bias="zero"))
    B, T0 = args.batch, args.frames
    rng = np.random.default_rng(21)
    zp = rng.standard_normal((B, 192, T0)).astype(np.float32)
    g = rng.standard_normal((B, 512, 1)).astype(np.float32)
    dec = gsv.Decoder.load(sd, device=0, mode=args.mode)
    secs = audio_seconds(B, T0, dec.hop)
    zd, gd = torch.from_numpy(zp).cuda(), torch.from_numpy(g).cuda()
    zo = torch.empty_like(zd)
    wav = torch.empty(B * T0 * dec.hop, device="cuda", dtype=torch.float32)

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / args.steps

    ms_flow = timed(lambda: dec.flow_inverse_device(zd, gd, out=zo))
    ms_both = timed(lambda: dec.flow_decode_device(zd, gd, out=wav))
    dec.set_stage_timing(2)
    for _ in range(3):
        dec.flow_inverse_device(zd, gd, out=zo)
    torch.cuda.synchronize()
    stats = dec.launch_stats()
    dec.set_stage_timing(0)
    roof_s, meas_s, rows = layer_roofline(stats, args.mode, pk)
    if args.layers:
        for r in rows:
            log(f"{r['name']:<22s} {r['ms']:9.4f} ms  roof {r['roof_ms']:9.4f} ms  frac {r['frac']}  {r['bound']}")
    flops = sum(s["flops"] for s in stats if s["kind"] == 0)
    cpu = None
    if not args.no_cpu_baseline:
        import oracle
        one = zp[:1, :, :T0]
        t0 = time.perf_counter()
        oracle.flow_inverse(sd, one, g[:1], None, acc64=False)
        dt = time.perf_counter() - t0
        cpu = {"value": audio_seconds(1, T0, dec.hop) / dt, "unit": UNIT, "cores": oracle.num_threads(),
               "kind": "port", "sample": f"1 utterance of {T0 / 50:g} s (z_p [1,192,{T0}]), C restatement "
                                         "of the reference flow, float accumulation"}
    emit({
        "metric": f"flow inverse audio-sec/sec at B={B}x{T0 / 50:g} s {args.mode}",
        "value": secs / (ms_flow / 1e3), "unit": UNIT, "ms_per_step": ms_flow, "steps": args.steps,
        "warmup": args.warmup, "dtype": args.mode, "data": "synthetic: seeded N(0,1) z_p/g, N(0,0.01) "
        "random-init weights, zero bias",
        "config": {"workload": f"flow inverse + y_mask, z_p [{B},192,{T0}] (4 coupling layers, WN 4 x k5)",
                   "batch": B, "frames": T0, "mode": args.mode},
        "flow_plus_decode": {"value": secs / (ms_both / 1e3), "unit": UNIT, "ms_per_step": ms_both},
        "layer_roofline": {"frac": roof_s / meas_s if meas_s else None, "sum_roof_ms": 1e3 * roof_s,
                           "sum_meas_ms": 1e3 * meas_s, "conv_tflops": flops / meas_s / 1e12 if meas_s else None,
                           "peaks": pk_kind},
        "launches": len(stats), "cpu_baseline": cpu})
    dec.close()


def run_encp(args):
    """The EncP fused chains around the text encoder's convs at B x T frames on
    one GPU (T = 50 frames per second of audio): per encoder layer of the
    v2 stacks (3 + 6 + 3) the attention-side add + LayerNorm (norm1) and the
    FFN half (conv_1 + ReLU, conv_2 + residual, norm2 + x_mask), then the
    output projection + prior sample.  The attention itself is outside these
    chains: a seeded tensor stands in for its output.  Device-resident inputs,
    CUDA events around K steps, layer-weighted roofline from per-launch events,
    the CPU oracle on one utterance as the baseline."""
    import torch
    gsv = load_pkg()
    pk, pk_kind = peaks()
    sd = gsv.synth.make_state_dict(0, init="n001", bias="zero")
    sd.update(gsv.synth.make_encp_state_dict())
    B, T = args.batch, args.frames
    rng = np.random.default_rng(31)
    x = rng.standard_normal((B, 192, T)).astype(np.float32)
    att = rng.standard_normal((B, 192, T)).astype(np.float32)
    noise = rng.standard_normal((B, 192, T)).astype(np.float32)
    lengths = np.full(B, T, np.int32)
    dec = gsv.Decoder.load(sd, device=0, mode=args.mode)
    secs = B * T / 50.0
    xd, ad, nd = (torch.from_numpy(a).cuda() for a in (x, att, noise))
    ld = torch.from_numpy(lengths).cuda()
    h1, h2 = torch.empty_like(xd), torch.empty_like(xd)
    m, logs, zp = torch.empty_like(xd), torch.empty_like(xd), torch.empty_like(xd)
    layers = [(st, i) for st, n in gsv.synth.ENCP_LAYERS.items() for i in range(n)]

    bufs = (h1, h2)

    def step(after=None):
        cur = xd
        for k, (st, i) in enumerate(layers):
            nxt = bufs[k % 2]
            dec.encp_layer_device(st, i, cur, ad, ld, out=nxt)
            if after:
                after()
            cur = nxt
        dec.encp_project_device(cur, ld, nd, 0.5, m, logs, zp)
        if after:
            after()

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / args.steps

    ms_eager = timed(step)  # one API call per layer, launched from Python
    # The same step captured once in a CUDA graph (every call is stream-async
    # and allocation-free after warm-up), replayed: device time without the
    # host's per-call overhead.
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        step()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    ms = timed(graph.replay)
    # per-launch profile of one eager step; each entry point records its own
    # event list, so the stats are read after every call.
    dec.set_stage_timing(2)
    stats = []
    step(after=lambda: stats.extend(dec.launch_stats()))
    dec.set_stage_timing(0)
    roof_s, meas_s, rows = layer_roofline(stats, args.mode, pk)
    if args.layers:
        for r in rows:
            log(f"{r['name']:<34s} {r['ms']:9.4f} ms  roof {r['roof_ms']:9.4f} ms  frac {r['frac']}  {r['bound']}")
    gemm = [s for s in stats if s["kind"] == 0]
    gemm_ms = sum(s["ms"] for s in gemm)
    gemm_flops = sum(s["flops"] for s in gemm)
    cpu = None
    if not args.no_cpu_baseline:
        import oracle
        one, a1, n1 = x[:1], att[:1], noise[:1]
        t0 = time.perf_counter()
        cur = one
        for st, i in layers:
            p = f"enc_p.{st}.norm_layers_1.{i}"
            cur = oracle.layer_norm(cur, sd[p + ".gamma"], sd[p + ".beta"], y=a1)
            cur = oracle.encp_ffn(sd, st, i, cur, [T], acc64=False)
        oracle.encp_project(sd, cur, [T], n1, 0.5, acc64=False)
        dt = time.perf_counter() - t0
        cpu = {"value": (T / 50.0) / dt, "unit": UNIT, "cores": oracle.num_threads(), "kind": "port",
               "sample": f"1 utterance of {T / 50:g} s (x [1,192,{T}]), C restatement of the chains, "
                         "float accumulation"}
    emit({
        "metric": f"EncP chains audio-sec/sec at B={B}x{T / 50:g} s {args.mode}",
        "value": secs / (ms / 1e3), "unit": UNIT, "ms_per_step": ms, "steps": args.steps,
        "warmup": args.warmup, "dtype": args.mode, "timing": "CUDA graph replay of one step",
        "eager": {"value": secs / (ms_eager / 1e3), "unit": UNIT, "ms_per_step": ms_eager,
                  "note": "one gsvdec_encp_layer call per layer from Python"},
        "data": "synthetic: seeded N(0,1) x / attention stand-in / noise, seeded random-init enc_p weights",
        "config": {"workload": f"12 enc_p layers (norm1(x + attn), FFN 192->768->192 k3, norm2 + mask) + proj "
                               f"+ prior sample, x [{B},192,{T}]", "batch": B, "frames": T, "mode": args.mode,
                   "launches_per_step": len(stats)},
        "layer_roofline": {"frac": roof_s / meas_s if meas_s else None, "sum_roof_ms": 1e3 * roof_s,
                           "sum_meas_ms": 1e3 * meas_s, "peaks": pk_kind},
        "ffn_gemm": {"ms": gemm_ms, "tflops": gemm_flops / (gemm_ms / 1e3) / 1e12 if gemm_ms else None,
                     "launches": len(gemm)},
        "launches": len(stats), "cpu_baseline": cpu})
    dec.close()


def run_load(args):
    """Checkpoint load through gsvdec_create_from_file (the C++ safetensors
    reader: mmap, dtype conversion, weight-norm fold, packing, upload) on a
    seeded v2 checkpoint written to a temporary file: the dec.* Generator, the
    flow and the enc_p tensors the chains use, fp32 as the converter writes
    them.  The CPU baseline restates the reference's load path for the same
    file (src/utils/weights.rs:116-162 read + the per-conv weight-norm fold of
    :589-614) with the oracle's fold."""
    import tempfile
    import torch
    from safetensors.numpy import load_file, save_file
    gsv = load_pkg()
    sd = gsv.synth.make_state_dict(0, init="n001", bias="zero")
    sd.update(gsv.synth.make_flow_state_dict(init="n001"))
    sd.update(gsv.synth.make_encp_state_dict())
    with tempfile.TemporaryDirectory() as tmp:
        path = os.path.join(tmp, "sovits_v2_seeded.safetensors")
        save_file({k: np.ascontiguousarray(v, dtype=np.float32) for k, v in sd.items()}, path)
        size = os.path.getsize(path)
        for _ in range(args.warmup):
            gsv.Decoder.load_file(path, device=0, mode=args.mode).close()
        torch.cuda.synchronize()
        times = []
        for _ in range(args.steps):
            t0 = time.perf_counter()
            d = gsv.Decoder.load_file(path, device=0, mode=args.mode)
            torch.cuda.synchronize()
            times.append(time.perf_counter() - t0)
            d.close()
        ms = 1e3 * float(np.median(times))
        cpu = None
        if not args.no_cpu_baseline:
            import oracle
            t0 = time.perf_counter()
            tens = load_file(path)
            n_wn = 0
            for k in [k for k in tens if k.endswith(".weight_v")]:
                pfx = k[: -len(".weight_v")]
                oracle.weight_norm(tens[k], tens[pfx + ".weight_g"])
                n_wn += 1
            dt = time.perf_counter() - t0
            cpu = {"value": size / dt / 1e6, "unit": "MB/s", "cores": oracle.num_threads(), "kind": "port",
                   "sample": f"the same {size / 1e6:.0f} MB file: safetensors read + {n_wn} weight-norm folds"}
    emit({
        "metric": f"checkpoint load MB/s ({args.mode})", "value": size / (ms / 1e3) / 1e6, "unit": "MB/s",
        "ms_per_load": ms, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
        "dtype": args.mode, "data": "synthetic: seeded v2 dec + flow + enc_p tensors, fp32 safetensors",
        "config": {"workload": f"gsvdec_create_from_file of a {size / 1e6:.0f} MB checkpoint "
                               "(mmap, fold, pack, upload; host wall clock incl. device sync)",
                   "file_bytes": size, "tensors": len(sd)},
        "cpu_baseline": cpu})


class _Solo:
    """torch.distributed's calls for a single process (no process group)."""

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


def sharded_result(workload, dec, ws, rank, steps, warmup, mode):
    """One strong-scaling workload over torch.distributed (NCCL): every rank gets
    the same inputs, decodes its share, and the finished waveform pieces are
    gathered to rank 0 inside the timed region; rank 0 then checks the result
    against single-GPU decodes of the same inputs.  Returns the result dict on
    rank 0 (None elsewhere).

    varlen256: 256 utterances with frame counts ~ U[100, 1000] (2-20 s),
    right-padded and length-masked, split by utterance (LPT) with up to 8
    length buckets per rank.  long60: one 60 s utterance (3000 frames) split
    into one contiguous frame range per rank, decoded with a 16-frame halo.
    value: inputs resident in HBM, device-side batching and NCCL gather; e2e:
    host arrays in (one pinned H2D per rank) and the whole waveform back on
    rank 0's host (one D2H), through the same public calls."""
    import torch
    import torch.distributed as dist
    gsv = load_pkg()
    hop = dec.hop
    group = dist.group.WORLD if ws > 1 else None
    dd = dist if ws > 1 else _Solo
    if workload == "varlen256":
        Bn, lo, hi = 256, 100, 1000
        lens = gsv.synth.make_lengths(Bn, lo, hi)
        z, g = gsv.synth.make_inputs(Bn, hi)
        total_s = float(lens.sum()) * hop / SAMPLE_RATE
        zd, gd = torch.from_numpy(z).cuda(), torch.from_numpy(g).cuda()
        dev_decode = lambda zb, gb, lb: dec.forward_device(zb, gb, lb)  # noqa: E731

        def step_dev():  # inputs resident in HBM, device pieces gathered over NCCL
            return gsv.shard.decode_batch_sharded(dev_decode, zd, gd, lens, hop, dd, group, device="cuda")

        def step_host():  # host arrays in, host waveform out on rank 0
            return gsv.shard.decode_batch_sharded(dev_decode, z, g, lens, hop, dd, group, device="cuda")
        desc = (f"{Bn} utterances, frames ~ U[{lo},{hi}] (2-20 s), right-padded to {hi}, length-masked, "
                "sharded by utterance (LPT), up to 8 length buckets per rank")
        h2d = int(z.nbytes + g.nbytes)
        d2h = int(lens.sum()) * hop * 4
    else:
        T0, halo = 3000, 16
        z, g = gsv.synth.make_inputs(1, T0)
        total_s = T0 * hop / SAMPLE_RATE
        zd, gd = torch.from_numpy(z).cuda(), torch.from_numpy(g).cuda()

        def step_dev():
            return gsv.shard.decode_long_chunked(
                lambda b, e: dec.forward_chunk_device(zd, gd, b, e, halo=halo), T0, hop, dd, group, device="cuda")

        def step_host():  # each rank's halo window in (pinned), the waveform out on rank 0
            return gsv.shard.decode_long_staged(
                lambda zw, gw, b, e: dec.forward_chunk_device(zw, gw, b, e, halo=halo), z, g, hop, dd, group,
                device="cuda", halo=halo)
        desc = f"one 60 s utterance (z [1,192,{T0}]) in {ws} time chunks, halo {halo} frames"
        wins = [gsv.shard.halo_window(b, e, T0, halo) for b, e in gsv.shard.plan_chunks(T0, ws) if e > b]
        h2d = int(sum(z.shape[1] * (hi - lo) * 4 + g.nbytes for lo, hi in wins))
        d2h = T0 * hop * 4

    def timed(step):
        for _ in range(warmup):
            step()
        if ws > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            out = step()
        e1.record()
        torch.cuda.synchronize()
        t_ms = e0.elapsed_time(e1)
        if ws > 1:
            t = torch.tensor([t_ms], device="cuda", dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            t_ms = float(t.item())
        return t_ms, out

    ms, res = timed(step_dev)
    ms_host, res_host = timed(step_host)
    if rank != 0:
        return None
    res = [r.cpu().numpy() for r in res] if isinstance(res, list) else res.cpu().numpy()
    # The host path's waveform (views of a reused pinned buffer: compared now)
    # must be the device path's, sample for sample.
    if isinstance(res, list):
        host_same = all(np.array_equal(a, np.asarray(b)) for a, b in zip(res, res_host))
    else:
        host_same = bool(np.array_equal(res, np.asarray(res_host)))
    if workload == "varlen256":
        idx = [0, int(np.argmax(lens)), int(np.argmin(lens))]
        errs, exact = [], True
        for i in idx:
            alone = dec.forward(z[i:i + 1, :, :lens[i]], g[i:i + 1])
            errs.append(float(np.abs(res[i] - alone).max() / max(np.abs(alone).max(), 1e-30)))
            exact = exact and bool(np.array_equal(res[i], alone))
        parity = {"checked_utterances": idx, "max_rel_err": max(errs), "bit_exact": exact,
                  "against": "single-GPU decode of each utterance alone"}
    else:
        whole = dec.forward(z, g)
        parity = {"max_rel_err": float(np.abs(res - whole).max() / max(np.abs(whole).max(), 1e-30)),
                  "bit_exact": bool(np.array_equal(res, whole)), "against": "single-GPU whole-utterance decode"}
    return {
        "value": total_s * steps / (ms / 1e3), "unit": UNIT, "n_gpus": ws, "steps": steps, "warmup": warmup,
        "ms_per_step": ms / steps, "scaling": "strong", "dtype": "bf16" if mode == "bf16" else "f32",
        "workload": desc, "audio_seconds_per_step": total_s,
        "gather": "waveform pieces to rank 0 inside the timed region (NCCL gather)",
        "e2e": {"value": total_s * steps / (ms_host / 1e3), "unit": UNIT, "ms_per_step": ms_host / steps,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "note": "host arrays in (one pinned H2D of each rank's share: its utterances, or its chunk's "
                        "halo window), waveform to rank 0's host (one pinned D2H)",
                "bit_exact_vs_device": bool(host_same)},
        "parity": parity,
    }


def run_sharded(args, ws, rank, local):
    """--workload varlen256 | long60 alone: one JSON line with that workload."""
    import torch
    import torch.distributed as dist
    if ws > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
    torch.cuda.set_device(local)
    gsv = load_pkg()
    sd = gsv.synth.make_state_dict(0, init="n001", bias="zero")
    dec = gsv.Decoder.load(sd, device=local, mode=args.mode)
    r = sharded_result(args.workload, dec, ws, rank, args.steps, args.warmup, args.mode)
    if rank == 0:
        emit({
            "metric": METRIC, "value": r["value"], "unit": UNIT, "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": r["ms_per_step"], "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": r["dtype"],
            "data": "synthetic: seeded N(0,1) z/g, N(0,0.01) random-init weights, zero bias",
            "config": {"workload": r["workload"], "audio_seconds_per_step": r["audio_seconds_per_step"],
                       "mode": args.mode, "gather": r["gather"],
                       "value_path": "inputs resident in HBM, device-side batching and gather"},
            "e2e": r["e2e"], "parity": r["parity"],
        })
    dec.close()
    if ws > 1:
        dist.destroy_process_group()


def bf16_cfg1_result(sd, local, steps, warmup):
    """Latency of one 5 s utterance (batch 1, z [1,192,250]) in the bf16 mode:
    device-resident inputs (CUDA events around K back-to-back forwards), and
    the blocking host-memory call an interactive caller makes (numpy in,
    numpy waveform out, host wall clock per call)."""
    import torch
    gsv = load_pkg()
    dec = gsv.Decoder.load(sd, device=local, mode="bf16")
    z, g = gsv.synth.make_inputs(1, 250)
    zt, gt = torch.from_numpy(z).cuda(), torch.from_numpy(g).cuda()
    out = torch.empty(250 * dec.hop, device="cuda")
    for _ in range(warmup):
        dec.forward_device(zt, gt, out=out)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        dec.forward_device(zt, gt, out=out)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    wav = np.empty(250 * dec.hop, np.float32)
    for _ in range(warmup):
        dec.forward(z, g, out=wav)
    t0 = time.perf_counter()
    for _ in range(steps):
        dec.forward(z, g, out=wav)
    ms_host = (time.perf_counter() - t0) * 1e3 / steps
    dec.close()
    return {"value": 5.0 / (ms / 1e3), "unit": UNIT, "ms_per_step": ms, "steps": steps, "warmup": warmup,
            "dtype": "bf16", "workload": "bf16 mode, B=1 x 5 s (z [1,192,250] -> 160 000 samples), latency",
            "host_call_ms": ms_host,
            "host_call": "gsvdec_forward(GSV_MEM_HOST) per call: numpy z / g in, numpy waveform out, host wall clock"}


def fp32_cfg1_result(sd, local, steps, warmup, pk, cpu=False, mode="fp32"):
    """An fp32-accurate mode on its own config: batch 1 x 5 s (z [1,192,250]),
    device-resident inputs, CUDA events around K steps; the layer-weighted
    roofline and the tap-GEMM launches' achieved TF/s.  mode "fp32": the CUDA
    cores, against the nominal FP32 CUDA-core peak (148 SMs x 128 lanes x 2
    FLOP x 1.965 GHz); "fp32tc": three bf16 pieces per value on the tensor
    cores, against the measured bf16 peak / 6 (six piece products per fp32
    product), its achieved rate also given as a fraction of the FP32 CUDA-core
    peak."""
    import torch
    gsv = load_pkg()
    dec = gsv.Decoder.load(sd, device=local, mode=mode)
    z, g = gsv.synth.make_inputs(1, 250)
    zt, gt = torch.from_numpy(z).cuda(), torch.from_numpy(g).cuda()
    out = torch.empty(250 * dec.hop, device="cuda")
    for _ in range(warmup):
        dec.forward_device(zt, gt, out=out)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        dec.forward_device(zt, gt, out=out)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    dec.set_stage_timing(2)
    for _ in range(steps):
        dec.forward_device(zt, gt, out=out)
    torch.cuda.synchronize()
    stats = dec.launch_stats()
    dec.set_stage_timing(0)
    dec.close()
    roof_s, meas_s, _ = layer_roofline(stats, mode, pk)
    cpu_base = None
    if cpu:  # the same batch-1 5 s input through the oracle port on the host cores
        reps, el, threads = cpu_port_sample(sd, z, g, min_seconds=3.0, max_reps=6)
        cpu_base = {"value": reps * 5.0 / el, "unit": UNIT, "ms_per_utterance": 1e3 * el / reps, "cores": threads,
                    "kind": "port", "sample": f"{reps} x the same 5 s utterance (z [1,192,250]), C restatement of "
                                              "the reference decoder, float accumulation"}
    conv = [s_ for s_ in stats if s_["kind"] == 0]
    f_conv = sum(s_["flops"] for s_ in conv)
    t_conv = sum(s_["ms"] for s_ in conv) / 1e3
    achieved = f_conv / t_conv / 1e12 if t_conv > 0 else None
    if mode == "fp32tc":
        peak = pk.get("bf16_tflops_sustained", pk.get("bf16_tflops")) / 6
        roof = {"bound": "tensor (six bf16 products per fp32 product)", "achieved": achieved, "peak": peak,
                "unit": "TFLOP/s", "frac": achieved / peak if achieved else None,
                "frac_of_fp32_core_peak": achieved / FP32_CORE_TFLOPS if achieved else None,
                "kernel": "tapconv_tc launches of one forward (all 97 convs except conv_post), three-piece operands",
                "peak_source": "measured bf16_tflops_sustained (MEASURED_PEAKS.json) / 6"}
        wl = "fp32tc mode (fp32 accuracy on the tensor cores), B=1 x 5 s (z [1,192,250] -> 160 000 samples)"
    else:
        roof = {"bound": "fp32-core", "achieved": achieved, "peak": FP32_CORE_TFLOPS, "unit": "TFLOP/s",
                "frac": achieved / FP32_CORE_TFLOPS if achieved else None,
                "kernel": "tapconv_f32 launches of one forward (all 97 convs except conv_post)",
                "peak_source": "nominal FP32 CUDA-core peak (not in MEASURED_PEAKS.json)"}
        wl = "fp32 CUDA-core mode, B=1 x 5 s (z [1,192,250] -> 160 000 samples)"
    return {
        "value": 5.0 / (ms / 1e3), "unit": UNIT, "ms_per_step": ms, "steps": steps, "warmup": warmup,
        "dtype": "f32", "workload": wl,
        "roofline": roof,
        "layer_roofline": {"frac": roof_s / meas_s if meas_s else None, "sum_roof_ms": 1e3 * roof_s,
                           "sum_meas_ms": 1e3 * meas_s},
        "gpu_launches": len(stats) * steps,
        "cpu_baseline": cpu_base,
    }


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--mode", choices=("bf16", "fp32", "fp32tc"), default="bf16")
    ap.add_argument("--batch", type=int, default=16)
    ap.add_argument("--frames", type=int, default=500)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--layers", action="store_true", help="print the per-launch table to stderr")
    ap.add_argument("--workload", choices=("batch16", "varlen256", "long60", "flow", "encp", "load"), default="batch16",
                    help="batch16: 16 x 10 s per GPU (weak scaling, the headline); varlen256: "
                         "256 utterances of 2-20 s sharded by utterance (strong scaling); long60: "
                         "one 60 s utterance split in halo time chunks (strong scaling); flow: the "
                         "flow inverse before the decoder (and flow + decoder), one GPU; encp: the "
                         "EncP fused chains (12 encoder layers' norms + FFN, projection + prior), one GPU; "
                         "load: safetensors checkpoint load (gsvdec_create_from_file)")
    ap.add_argument("--sweep", action="store_true",
                    help="per-layer sweep: every distinct conv shape at --batch (64 by default) "
                         "x --frames, in --mode; prints one JSON line per mode")
    ap.add_argument("--no-extra", action="store_true",
                    help="skip the extra keys (varlen256, long60 strong scaling; fp32 batch-1 5 s)")
    ap.add_argument("--once", action="store_true",
                    help="one untimed forward, then exit (a short, fixed launch list for ncu)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    ws, rank, local = dist_setup()
    if ws > 1:
        keep_stdout_for_json()

    if args.impl == "reference":
        run_reference(args, ws, rank)
        return
    if args.sweep:
        run_sweep(args)
        return
    if args.workload == "flow":
        run_flow(args)
        return
    if args.workload == "encp":
        run_encp(args)
        return
    if args.workload == "load":
        run_load(args)
        return
    if args.workload != "batch16":
        run_sharded(args, ws, rank, local)
        return

    import torch
    import torch.distributed as dist
    if ws > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    torch.cuda.set_device(local)
    gsv = load_pkg()
    sd = gsv.synth.make_state_dict(0, init="n001", bias="zero")
    B, T0 = args.batch, args.frames
    z, g = gsv.synth.make_inputs(B, T0, seed_z=1 + 1000 * rank, seed_g=2 + 1000 * rank)
    dec = gsv.Decoder.load(sd, device=local, mode=args.mode)
    hop = dec.hop
    secs_per_step = audio_seconds(B, T0, hop)
    stream = torch.cuda.current_stream()

    def barrier():
        if ws > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if ws == 1:
            return x
        t = torch.tensor([x], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- device-resident throughput (value) --------------------------------
    zt = torch.from_numpy(z).cuda()
    gt = torch.from_numpy(g).cuda()
    out = torch.empty(B * T0 * hop, device="cuda", dtype=torch.float32)
    if args.once:
        dec.forward_device(zt, gt, out=out)
        torch.cuda.synchronize()
        log(f"one forward: {dec.launch_count()} launches, finite={bool(torch.isfinite(out).all())}")
        dec.close()
        return
    # With N > 1 every step's waveform is gathered to rank 0 over NCCL inside
    # the timed region (the north star's one collective).  The gather of step
    # i runs on a second stream while step i + 1 decodes into the other of two
    # output buffers; a buffer is overwritten only after its gather has read it.
    outs = [out, torch.empty_like(out)]
    comm = torch.cuda.Stream() if ws > 1 else None
    ev_done = [torch.cuda.Event(), torch.cuda.Event()]
    ev_sent = [torch.cuda.Event(), torch.cuda.Event()]
    gathered = [[torch.empty_like(out) for _ in range(ws)] for _ in range(2)] if (ws > 1 and rank == 0) else None

    def step(i):
        k = i % 2
        if comm is not None:
            stream.wait_event(ev_sent[k])
        dec.forward_device(zt, gt, out=outs[k])
        if comm is not None:
            ev_done[k].record(stream)
            with torch.cuda.stream(comm):
                comm.wait_event(ev_done[k])
                dist.gather(outs[k], gather_list=gathered[k] if rank == 0 else None, dst=0)
                ev_sent[k].record(comm)

    for i in range(args.warmup):
        step(i)
    if comm is not None:
        stream.wait_stream(comm)
    torch.cuda.synchronize()
    launches_per_step = dec.launch_count()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        step(i)
    if comm is not None:
        stream.wait_stream(comm)  # every gather has landed before the clock stops
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    ms = max_over_ranks(e0.elapsed_time(e1))
    value = ws * secs_per_step * args.steps / (ms / 1e3)
    assert torch.isfinite(out).all().item()
    gather_check = None
    if gathered is not None:
        # rank r's last waveform arrived intact: rank 0 decodes rank r's inputs itself
        last = gathered[(args.steps - 1) % 2]
        zr, gr = gsv.synth.make_inputs(B, T0, seed_z=1 + 1000 * (ws - 1), seed_g=2 + 1000 * (ws - 1))
        mine = dec.forward_device(torch.from_numpy(zr).cuda(), torch.from_numpy(gr).cuda())
        torch.cuda.synchronize()
        gather_check = {"rank_checked": ws - 1, "bit_exact": bool(torch.equal(last[ws - 1], mine))}
    # ---- end to end through the public call with host buffers (e2e) --------
    # Every step copies its z / g in from pinned host memory and its waveform
    # back out.  Headline: gsvdec_forward with GSV_MEM_HOST_ASYNC, the call a
    # serving loop makes -- the copies of one step run while the steps next to
    # it decode.  Also reported: the blocking GSV_MEM_HOST call, one step at a
    # time (copy in, decode, copy out, stream sync).
    zh = torch.from_numpy(z).pin_memory()
    gh = torch.from_numpy(g).pin_memory()
    wh = torch.empty(B * T0 * hop, dtype=torch.float32).pin_memory()
    zn, gn, wn = zh.numpy(), gh.numpy(), wh.numpy()

    # Same protocol as the device-resident loop above (warm-up, the same short
    # idle while the clock sampler starts, then K steps), so both start from
    # the same power state: under the 1 kW cap the SM clock falls after
    # ~0.5 s of back-to-back decoding, and a loop timed straight after the
    # others would measure that instead of the host path.
    def timed_host(call):
        for _ in range(args.warmup):
            call()
        torch.cuda.synchronize()
        cs = ClockSampler(local)
        cs.start()
        time.sleep(0.3)
        barrier()
        torch.cuda.synchronize()
        h0, h1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        h0.record(stream)
        for _ in range(args.steps):
            call()
        h1.record(stream)
        torch.cuda.synchronize()
        barrier()
        return max_over_ranks(h0.elapsed_time(h1)), cs.stop()

    ms_e2e, clk_e2e = timed_host(lambda: dec.forward_async(zh, gh, out=wh, stream=stream.cuda_stream))
    dec.sync_status(stream.cuda_stream)
    wav_async = wn.copy()
    ms_block, _ = timed_host(lambda: dec.forward(zn, gn, out=wn, stream=stream.cuda_stream))
    assert np.array_equal(wav_async, wn), "overlapped and blocking host calls disagree"
    e2e = {"value": ws * secs_per_step * args.steps / (ms_e2e / 1e3), "unit": UNIT,
           "h2d_bytes_per_step": int(zn.nbytes + gn.nbytes), "d2h_bytes_per_step": int(wn.nbytes),
           "ms_per_step": ms_e2e / args.steps,
           "call": "gsvdec_forward(GSV_MEM_HOST_ASYNC) on pinned host buffers, one call per step",
           "clocks": clk_e2e,
           "blocking": {"value": ws * secs_per_step * args.steps / (ms_block / 1e3),
                        "ms_per_step": ms_block / args.steps,
                        "call": "gsvdec_forward(GSV_MEM_HOST): copy in, decode, copy out, sync, per step"}}

    # Per-launch profile (roofline) from the same K steps run again with an
    # event pair around every launch; kept out of the timed loop above, which
    # runs the launches exactly as a caller does (no event records between
    # them, so each kernel may start during the tail of the one before).
    dec.set_stage_timing(2)
    for _ in range(args.steps):
        dec.forward_device(zt, gt, out=out)
    torch.cuda.synchronize()
    stats = dec.launch_stats()
    dec.set_stage_timing(0)

    # ---- roofline of the dominant kernel + layer-weighted fraction ----------
    pk, pk_kind = peaks()
    conv = [s for s in stats if s["kind"] == 0]
    f_conv = sum(s["flops"] for s in conv)
    t_conv = sum(s["ms"] for s in conv) / 1e3
    if args.mode == "bf16":
        peak = pk.get("bf16_tflops_sustained", pk["bf16_tflops"])
        bound = "tensor"
    elif args.mode == "fp32tc":  # six bf16 tensor-core products per fp32 product
        peak = pk.get("bf16_tflops_sustained", pk["bf16_tflops"]) / 6
        bound = "tensor (three-piece fp32)"
    else:
        peak = FP32_CORE_TFLOPS
        bound = "fp32-core"
    achieved_all = f_conv / t_conv / 1e12 if t_conv > 0 else None
    # The dominant kernel: tapconv_tc_kernel<64, 128, ...>, every launch of it
    # (conv_pre, rb1's conv1 / conv2 groups and branch sum, and ups2: the largest share
    # of the forward in the ncu launch list).  achieved = their algorithmic
    # FLOPs / their CUDA-event time; traffic = DRAM bytes of one rb1.step1.conv1
    # launch from a single-launch ncu capture.
    dom_names = ("conv_pre", "rb1.step0.conv1", "rb1.step0.conv2", "rb1.step1.conv1", "rb1.step1.conv2",
                 "rb1.step2.conv1", "rb1.final", "ups2")
    dom = [s for s in conv if s["name"] in dom_names]
    f_dom = sum(s["flops"] for s in dom)
    t_dom = sum(s["ms"] for s in dom) / 1e3
    achieved = f_dom / t_dom / 1e12 if t_dom > 0 else None
    traffic = None
    prof = ROOT / "profiles" / "tapconv_tc_64x128_rb1_conv1_traffic.json"
    if args.mode == "bf16" and prof.exists():
        try:
            traffic = json.loads(prof.read_text()).get("dram_bytes_per_launch")
        except (ValueError, OSError):
            traffic = None
    roof_s, meas_s, rows = layer_roofline(stats, args.mode, pk)
    roofline = {"bound": bound, "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak if achieved else None, "traffic": traffic,
                "traffic_unit": "DRAM bytes per launch (ncu, one rb1.step1.conv1 launch)",
                "kernel": "tapconv_tc_kernel<64, 128, ...>, every launch of it (" + str(len(dom_names)) +
                          " per forward: " + ", ".join(dom_names) + ")",
                "launches_per_step": len(dom),
                "peak_source": f"{pk_kind} " + {"bf16": "bf16_tflops_sustained",
                                                "fp32tc": "bf16_tflops_sustained / 6"}.get(args.mode,
                                                                                           "nominal fp32 CUDA-core"),
                "all_tap_gemm": {"achieved": achieved_all, "frac": achieved_all / peak if achieved_all else None,
                                 "note": "every tap-GEMM launch (tapconv_tc + fused rbstep_tc), HBM-bound ones "
                                         "included, against the tensor peak"}}
    by_bound = roofline_by_bound(stats, args.mode, pk)
    layer = {"frac": roof_s / meas_s if meas_s else None, "sum_roof_ms": 1e3 * roof_s,
             "sum_meas_ms": 1e3 * meas_s, "hbm_gbs": pk["hbm_gbs"],
             "compute_tflops": peak, "peaks": pk_kind}
    if args.layers and rank == 0:
        for r in rows:
            log(f"{r['name']:<22s} {r['ms']:9.4f} ms  roof {r['roof_ms']:9.4f} ms  "
                f"frac {r['frac']}  {r['bound']}")

    # ---- CPU baseline (rank 0, N = 1 only) ----------------------------------
    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        reps, el, threads = cpu_port_sample(sd, z[:1], g[:1])
        cpu = {"value": reps * audio_seconds(1, T0, hop) / el, "unit": UNIT, "cores": threads,
               "kind": "port",
               "sample": f"{reps} x 1 utterance of {T0 / 50:g} s (z [1,192,{T0}]) of the same "
                         "workload, C restatement of the reference decoder, float accumulation"}

    # ---- the other configs of the same job, as extra keys of the line -------
    extra = {}
    if not args.no_extra:
        xs, xw = max(1, min(args.steps, 5)), 3
        for wl in ("varlen256", "long60"):
            r = sharded_result(wl, dec, ws, rank, xs, xw, args.mode)
            if rank == 0:
                extra[wl] = r
        if rank == 0:
            extra["fp32_cfg1"] = fp32_cfg1_result(sd, local, max(3, min(args.steps, 10)), 3, pk,
                                                  cpu=ws == 1 and not args.no_cpu_baseline)
            extra["fp32tc_cfg1"] = fp32_cfg1_result(sd, local, max(3, min(args.steps, 10)), 3, pk, mode="fp32tc")
            extra["bf16_cfg1"] = bf16_cfg1_result(sd, local, max(10, args.steps), 5)
        barrier()

    if rank == 0:
        emit({
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16" if args.mode == "bf16" else "f32",
            "data": "synthetic: seeded N(0,1) z/g, N(0,0.01) random-init weights, zero bias",
            "config": {"workload": f"B={B} x {T0 / 50:g} s Generator decode per GPU "
                                   f"(z [{B},192,{T0}] -> [{B},1,{T0 * hop}])",
                       "batch": B, "frames": T0, "mode": args.mode,
                       "l2": "no flush: one step moves several GB of activations through "
                             "buffers of 164 MB each (> 126 MB L2)",
                       "parallelism": f"utterance-sharded x{ws}" + (
                           ", every step's waveform gathered to rank 0 over NCCL inside the timed region "
                           "(overlapped with the next step's decode)" if ws > 1 else "")},
            "e2e": e2e, "gpu_launches": launches_per_step * args.steps, "roofline": roofline,
            "layer_roofline": layer, "roofline_by_bound": by_bound, "cpu_baseline": cpu, "clocks": clk,
            "gather_check": gather_check, **extra,
        })
    dec.close()
    if ws > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
