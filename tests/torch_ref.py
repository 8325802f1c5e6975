"""Independent float64 PyTorch restatement of the reference Generator forward.

Used only to cross-check the C oracle (and to generate golden fixtures): it
shares no code with the oracle or the CUDA library.  Follows
src/models/sovits_decoder.rs:386-458 of the reference crate, with
torch.nn.functional conv semantics (the PyTorch semantics the reference was
aligned to, IMPLEMENTATION.md:3).
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

RATES = (10, 8, 2, 2, 2)


def lrelu(x, slope):
    # Sign-bit LeakyReLU of the reference's CPU op (sovits_decoder.rs:46-53).
    return torch.where(torch.signbit(x), x * slope, x)


def fold(sd, p):
    v = torch.as_tensor(np.asarray(sd[p + ".weight_v"]), dtype=torch.float64)
    g = torch.as_tensor(np.asarray(sd[p + ".weight_g"]), dtype=torch.float64).reshape(-1, 1, 1)
    return v / v.pow(2).sum(dim=(1, 2), keepdim=True).sqrt() * g


def t64(sd, k):
    return torch.as_tensor(np.asarray(sd[k]), dtype=torch.float64) if k in sd else None


def decoder_forward(sd, z, g=None, taps=False):
    z = torch.as_tensor(np.asarray(z), dtype=torch.float64)
    out_taps = []
    x = F.conv1d(z, t64(sd, "dec.conv_pre.weight"), t64(sd, "dec.conv_pre.bias"), padding=3)
    if g is not None and "dec.cond.weight" in sd:
        gg = torch.as_tensor(np.asarray(g), dtype=torch.float64)
        x = x + F.conv1d(gg, t64(sd, "dec.cond.weight"), t64(sd, "dec.cond.bias"))
    out_taps.append(x)
    n_up = 0
    ups = [i for i in range(10) if f"dec.ups.{i}.weight_v" in sd]
    rbs = [r for r in range(15) if f"dec.resblocks.{r}.convs1.0.weight_v" in sd]
    for i, u in enumerate(ups):
        x = lrelu(x, 0.1)
        w = fold(sd, f"dec.ups.{u}")
        s = RATES[i] if i < 5 else 2
        k = w.shape[2]
        x = F.conv_transpose1d(x, w, t64(sd, f"dec.ups.{u}.bias"), stride=s, padding=(k - s) // 2)
        out_taps.append(x)
        acc = None
        sel = rbs[3 * i:3 * i + 3]
        for rr, r in enumerate(sel):
            kk = (3, 7, 11)[r % 3]
            xo = x
            for j in range(3):
                p1 = f"dec.resblocks.{r}.convs1.{j}"
                if p1 + ".weight_v" not in sd:
                    continue
                d = (1, 3, 5)[j]
                t = F.conv1d(lrelu(xo, 0.1), fold(sd, p1), t64(sd, p1 + ".bias"),
                             padding=d * (kk - 1) // 2, dilation=d)
                p2 = f"dec.resblocks.{r}.convs2.{j}"
                t = F.conv1d(lrelu(t, 0.1), fold(sd, p2), t64(sd, p2 + ".bias"), padding=(kk - 1) // 2)
                xo = xo + t
            acc = xo if acc is None else acc + xo
        if acc is not None:
            x = acc / len(sel)
            out_taps.append(x)
    x = lrelu(x, 0.01)
    x = F.conv1d(x, t64(sd, "dec.conv_post.weight"), t64(sd, "dec.conv_post.bias"), padding=3)
    out_taps.append(x)
    wav = torch.tanh(x).flatten().numpy()
    if taps:
        return wav, [t.numpy() for t in out_taps]
    return wav


def flow_inverse(sd, z_p, g=None, lengths=None, prefix="flow.flows"):
    """z = flow^-1(z_p) * y_mask in float64: ResidualCouplingBlock::forward with
    reverse = true (src/models/sovits_flow.rs:341-415; coupling layer :286-335,
    WN :119-168) and src/models/sovits.rs:394, with torch conv semantics."""
    x = torch.as_tensor(np.asarray(z_p), dtype=torch.float64)
    B, C, T = x.shape
    ln = torch.full((B,), T) if lengths is None else torch.as_tensor(np.asarray(lengths))
    mask = (torch.arange(T)[None, :] < ln[:, None]).to(torch.float64)[:, None, :]
    gg = torch.as_tensor(np.asarray(g), dtype=torch.float64) if g is not None else None
    idx = [i for i in range(8) if f"{prefix}.{i}.pre.weight" in sd]

    def conv(p, inp):
        w = fold(sd, p) if p + ".weight_v" in sd else t64(sd, p + ".weight")
        return F.conv1d(inp, w, t64(sd, p + ".bias"), padding=(w.shape[2] - 1) // 2)

    for i in reversed(idx):
        p = f"{prefix}.{i}"
        x = torch.flip(x, dims=[1])
        half = sd[p + ".pre.weight"].shape[1]
        x0, x1 = x[:, :half], x[:, half:]
        h = conv(p + ".pre", x0) * mask
        nl = len([j for j in range(16) if f"{p}.enc.in_layers.{j}.weight_v" in sd])
        hid = h.shape[1]
        gp = conv(p + ".enc.cond_layer", gg) if gg is not None and p + ".enc.cond_layer.weight_v" in sd else None
        out = torch.zeros_like(h)
        xw = h
        for j in range(nl):
            xin = conv(f"{p}.enc.in_layers.{j}", xw * mask)
            if gp is not None:
                xin = xin + gp[:, j * 2 * hid:(j + 1) * 2 * hid]
            acts = torch.tanh(xin[:, :hid]) * torch.sigmoid(xin[:, hid:])
            rs = conv(f"{p}.enc.res_skip_layers.{j}", acts)
            if j < nl - 1:
                xw = (xw + rs[:, :hid]) * mask
                out = out + rs[:, hid:]
            else:
                out = out + rs
        stats = conv(p + ".post", out * mask) * mask
        if stats.shape[1] >= 2 * half:
            m, logs = stats[:, :half], stats[:, half:]
        else:
            m, logs = stats, torch.zeros_like(stats)
        x = torch.cat([x0, (x1 - m) * torch.exp(-logs)], dim=1)
    return (x * mask).numpy()


def _mask(B, T, lengths):
    ln = torch.full((B,), T) if lengths is None else torch.as_tensor(np.asarray(lengths))
    return (torch.arange(T)[None, :] < ln[:, None]).to(torch.float64)[:, None, :]


def layer_norm(x, gamma, beta, y=None, lengths=None, eps=1e-5):
    """LayerNorm over channels of x (+ y) [B, C, T] in float64, times x_mask
    (src/utils/weights.rs:461-502; src/models/sovits_encp.rs:102-109), via
    F.layer_norm on the channel-last view."""
    v = torch.as_tensor(np.asarray(x), dtype=torch.float64)
    if y is not None:
        v = v + torch.as_tensor(np.asarray(y), dtype=torch.float64)
    g = torch.as_tensor(np.asarray(gamma), dtype=torch.float64)
    b = torch.as_tensor(np.asarray(beta), dtype=torch.float64)
    o = F.layer_norm(v.transpose(1, 2), (v.shape[1],), g, b, eps).transpose(1, 2)
    if lengths is not None:
        o = o * _mask(v.shape[0], v.shape[2], lengths)
    return o.numpy()


def encp_ffn(sd, stack, layer, x, lengths=None):
    """norm2(x + conv_2(relu(conv_1(x)))) * x_mask (src/models/sovits_encp.rs:104-109)."""
    f = f"enc_p.{stack}.ffn_layers.{layer}"
    xt = torch.as_tensor(np.asarray(x), dtype=torch.float64)
    w1, w2 = t64(sd, f + ".conv_1.weight"), t64(sd, f + ".conv_2.weight")
    h = torch.relu(F.conv1d(xt, w1, t64(sd, f + ".conv_1.bias"), padding=(w1.shape[2] - 1) // 2))
    y = F.conv1d(h, w2, t64(sd, f + ".conv_2.bias"), padding=(w2.shape[2] - 1) // 2)
    p = f"enc_p.{stack}.norm_layers_2.{layer}"
    return layer_norm(xt.numpy(), sd[p + ".gamma"], sd[p + ".beta"], y=y.numpy(), lengths=lengths)


def interpolate(x, T_out):
    """Half-pixel linear interpolation along time (F.interpolate, mode
    'linear', align_corners False), the PyTorch op linear_interpolate_last_dim
    restates (src/models/sovits_encp.rs:10-40)."""
    xt = torch.as_tensor(np.asarray(x), dtype=torch.float64)
    return F.interpolate(xt, size=T_out, mode="linear", align_corners=False).numpy()


def encp_project(sd, y, lengths=None, noise=None, noise_scale=0.5):
    """(m, logs, z_p) of src/models/sovits_encp.rs:871-879 and
    src/models/sovits.rs:378-385 in float64."""
    yt = torch.as_tensor(np.asarray(y), dtype=torch.float64)
    stats = F.conv1d(yt, t64(sd, "enc_p.proj.weight"), t64(sd, "enc_p.proj.bias"))
    stats = stats * _mask(yt.shape[0], yt.shape[2], lengths)
    co = stats.shape[1] // 2
    m, logs = stats[:, :co], stats[:, co:].clamp(-5.0, 2.0)
    zp = None
    if noise is not None:
        zp = (m + torch.as_tensor(np.asarray(noise), dtype=torch.float64) * torch.exp(logs) * noise_scale).numpy()
    return m.numpy(), logs.numpy(), zp
