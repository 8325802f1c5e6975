"""Seeded synthetic Generator weights and inputs in the reference's layout.

There are no checkpoints offline, so every workload runs on random-init
weights with the SoVITS v2 Generator architecture, stored under the exact
safetensors keys the reference loads (src/models/sovits_decoder.rs:231-293):

* ``dec.conv_pre.{weight [512,192,7], bias [512]}``
* ``dec.cond.{weight [512,gin,1], bias [512]}``
* ``dec.ups.{i}.{weight_g [Cin,1,1], weight_v [Cin,Cout,k], bias [Cout]}``
* ``dec.resblocks.{r}.convs{1,2}.{j}.{weight_g [C,1,1], weight_v [C,C,k], bias [C]}``
* ``dec.conv_post.weight [1,16,7]`` (no bias, as in v2)

Weight-norm pairs are generated so the fold ``g * v / ||v||`` recovers the
intended weight w exactly: ``v = w * r`` for a random positive per-slice
scale r and ``g = ||w||``.  ``init="n001"`` draws every weight from
N(0, 0.01) (the benchmark workload); ``init="unit"`` uses std
1/sqrt(fan_in) so activations stay O(1) through the stack (stronger parity
checks, since N(0, 0.01) shrinks the waveform to ~1e-6).
"""
from __future__ import annotations

import numpy as np

UPSAMPLE_RATES = (10, 8, 2, 2, 2)
UPSAMPLE_KERNELS = (16, 16, 8, 2, 2)
CHANNELS = (512, 256, 128, 64, 32, 16)
RES_KERNELS = (3, 7, 11)
RES_DILATIONS = (1, 3, 5)
IN_CHANNELS = 192
HOP = 640


def _std(init: str, fan_in: int) -> float:
    if init == "n001":
        return 0.01
    if init == "unit":
        return 1.0 / np.sqrt(fan_in)
    raise ValueError(init)


def make_state_dict(seed: int = 0, gin: int = 512, init: str = "n001", bias: str = "zero",
                    with_cond: bool = True, n_stages: int = 5) -> dict:
    """The ``dec.*`` tensors (float32) of a seeded random Generator."""
    rng = np.random.default_rng(seed)
    sd = {}

    def w(shape, fan_in):
        return (rng.standard_normal(shape, dtype=np.float32) * np.float32(_std(init, fan_in)))

    def b(n):
        if bias == "zero":
            return np.zeros(n, np.float32)
        return (rng.standard_normal(n, dtype=np.float32) * np.float32(0.05))

    def wn(prefix, weight):
        r = rng.uniform(0.5, 2.0, size=(weight.shape[0], 1, 1)).astype(np.float32)
        norm = np.sqrt((weight.astype(np.float64) ** 2).sum(axis=(1, 2))).astype(np.float32)
        sd[prefix + ".weight_v"] = (weight * r).astype(np.float32)
        sd[prefix + ".weight_g"] = norm.reshape(-1, 1, 1)

    sd["dec.conv_pre.weight"] = w((CHANNELS[0], IN_CHANNELS, 7), IN_CHANNELS * 7)
    sd["dec.conv_pre.bias"] = b(CHANNELS[0])
    if with_cond:
        sd["dec.cond.weight"] = w((CHANNELS[0], gin, 1), gin)
        sd["dec.cond.bias"] = b(CHANNELS[0])
    for i in range(n_stages):
        cin, cout, k, s = CHANNELS[i], CHANNELS[i + 1], UPSAMPLE_KERNELS[i], UPSAMPLE_RATES[i]
        wn(f"dec.ups.{i}", w((cin, cout, k), cin * max(1, k // s)))
        sd[f"dec.ups.{i}.bias"] = b(cout)
        for rr in range(3):
            r = 3 * i + rr
            kk = RES_KERNELS[rr]
            for c in (1, 2):
                for j in range(3):
                    p = f"dec.resblocks.{r}.convs{c}.{j}"
                    wn(p, w((cout, cout, kk), cout * kk))
                    sd[p + ".bias"] = b(cout)
    sd["dec.conv_post.weight"] = w((1, CHANNELS[n_stages], 7), CHANNELS[n_stages] * 7)
    return sd


FLOW_HALF = 96      # inter_channels / 2
FLOW_HIDDEN = 192
FLOW_KERNEL = 5
FLOW_WN_LAYERS = 4
FLOW_COUPLINGS = 4  # at indices 0, 2, 4, 6 (the flips between them hold no weights)


def make_flow_state_dict(seed: int = 10, gin: int = 512, init: str = "unit", bias: str = "rand",
                         with_cond: bool = True, n_couplings: int = FLOW_COUPLINGS) -> dict:
    """The ``flow.flows.*`` tensors (float32) of a seeded random SoVITS v2 flow,
    under the keys ResidualCouplingBlock::load reads (reference
    src/models/sovits_flow.rs:346-368, 186-335, 10-108): per coupling layer
    ``pre.{weight [192,96,1], bias}`` and ``post.{weight [96,192,1], bias}``
    (plain weights), ``enc.in_layers.{j}`` [384,192,5], ``enc.res_skip_layers.{j}``
    [384 or 192 (last),192,1] and ``enc.cond_layer`` [1536,gin,1] as weight-norm
    pairs (v, g) with biases."""
    rng = np.random.default_rng(seed)
    sd = {}
    h, half, k, nl = FLOW_HIDDEN, FLOW_HALF, FLOW_KERNEL, FLOW_WN_LAYERS

    def w(shape, fan_in):
        return (rng.standard_normal(shape, dtype=np.float32) * np.float32(_std(init, fan_in)))

    def b(n):
        if bias == "zero":
            return np.zeros(n, np.float32)
        return (rng.standard_normal(n, dtype=np.float32) * np.float32(0.05))

    def wn(prefix, weight):
        r = rng.uniform(0.5, 2.0, size=(weight.shape[0], 1, 1)).astype(np.float32)
        norm = np.sqrt((weight.astype(np.float64) ** 2).sum(axis=(1, 2))).astype(np.float32)
        sd[prefix + ".weight_v"] = (weight * r).astype(np.float32)
        sd[prefix + ".weight_g"] = norm.reshape(-1, 1, 1)

    for li in range(n_couplings):
        p = f"flow.flows.{2 * li}"
        sd[p + ".pre.weight"] = w((h, half, 1), half)
        sd[p + ".pre.bias"] = b(h)
        for j in range(nl):
            wn(f"{p}.enc.in_layers.{j}", w((2 * h, h, k), h * k))
            sd[f"{p}.enc.in_layers.{j}.bias"] = b(2 * h)
            ro = 2 * h if j < nl - 1 else h
            wn(f"{p}.enc.res_skip_layers.{j}", w((ro, h, 1), h))
            sd[f"{p}.enc.res_skip_layers.{j}.bias"] = b(ro)
        if with_cond:
            wn(f"{p}.enc.cond_layer", w((2 * h * nl, gin, 1), gin))
            sd[f"{p}.enc.cond_layer.bias"] = b(2 * h * nl)
        sd[p + ".post.weight"] = w((half, h, 1), h)
        sd[p + ".post.bias"] = b(half)
    return sd


ENCP_HIDDEN = 192
ENCP_FILTER = 768
ENCP_KERNEL = 3
ENCP_LAYERS = {"encoder_ssl": 3, "encoder_text": 6, "encoder2": 3}  # n_layers // 2, n_layers, n_layers // 2
ENCP_OUT = 192


def make_encp_state_dict(seed: int = 20, layers=None, hidden: int = ENCP_HIDDEN,
                         filter_channels: int = ENCP_FILTER, kernel: int = ENCP_KERNEL,
                         out_channels: int = ENCP_OUT, with_proj: bool = True) -> dict:
    """The ``enc_p.*`` tensors (float32) the EncP chains read, seeded, under the
    keys of EncoderLayer::load / FeedForward::load (reference
    src/models/sovits_encp.rs:54-96, 348-369, 752-771): per layer i of each
    stack ``ffn_layers.{i}.conv_1`` [F, C, k] and ``conv_2`` [C, F, k] with
    biases, ``norm_layers_{1,2}.{i}.{gamma, beta}`` [C]; and ``enc_p.proj``
    [2 out, C, 1] with bias.  Attention weights are not generated (the
    attention itself is not part of these chains)."""
    rng = np.random.default_rng(seed)
    layers = ENCP_LAYERS if layers is None else layers
    sd = {}
    C, F, k = hidden, filter_channels, kernel
    for stack, n in layers.items():
        p = f"enc_p.{stack}"
        for i in range(n):
            f = f"{p}.ffn_layers.{i}"
            sd[f + ".conv_1.weight"] = rng.standard_normal((F, C, k), dtype=np.float32) * np.float32((C * k) ** -0.5)
            sd[f + ".conv_1.bias"] = rng.standard_normal(F, dtype=np.float32) * np.float32(0.05)
            sd[f + ".conv_2.weight"] = rng.standard_normal((C, F, k), dtype=np.float32) * np.float32((F * k) ** -0.5)
            sd[f + ".conv_2.bias"] = rng.standard_normal(C, dtype=np.float32) * np.float32(0.05)
            for nl in (1, 2):
                sd[f"{p}.norm_layers_{nl}.{i}.gamma"] = (
                    1.0 + 0.1 * rng.standard_normal(C, dtype=np.float32)).astype(np.float32)
                sd[f"{p}.norm_layers_{nl}.{i}.beta"] = rng.standard_normal(C, dtype=np.float32) * np.float32(0.1)
    if with_proj:
        sd["enc_p.proj.weight"] = rng.standard_normal((2 * out_channels, C, 1), dtype=np.float32) * np.float32(C ** -0.5)
        sd["enc_p.proj.bias"] = rng.standard_normal(2 * out_channels, dtype=np.float32) * np.float32(0.5)
    return sd


def make_inputs(B: int, T0: int, gin: int = 512, seed_z: int = 1, seed_g: int = 2):
    """z [B,192,T0] ~ N(0,1) and g [B,gin,1] ~ N(0,1), seeded."""
    z = np.random.default_rng(seed_z).standard_normal((B, IN_CHANNELS, T0), dtype=np.float32)
    g = np.random.default_rng(seed_g).standard_normal((B, gin, 1), dtype=np.float32)
    return z, g


def make_lengths(B: int, lo: int, hi: int, seed: int = 3) -> np.ndarray:
    """Per-utterance frame counts ~ U[lo, hi] (seeded), int32."""
    return np.random.default_rng(seed).integers(lo, hi + 1, size=B).astype(np.int32)


def checksum(sd: dict) -> float:
    """Order-independent float64 checksum of a state dict (fixture drift check)."""
    return float(sum(np.asarray(v, np.float64).sum() + np.abs(np.asarray(v, np.float64)).sum()
                     for v in sd.values()))
