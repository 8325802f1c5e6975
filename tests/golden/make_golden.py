"""Regenerates the golden fixtures in this folder (run from the repo root:
``python tests/golden/make_golden.py``).

Expected values come from PyTorch CPU in float64 -- an implementation
independent of both the C oracle and the CUDA library.  Inputs:

* ``kat_ref.npz`` -- the reference crate's own known-answer tests, re-created
  from their closed-form inputs:
  - leaky_relu([-2, 0, 3], 0.1) == [-0.2, 0, 3]  (src/models/sovits_decoder.rs:583-589)
  - padded ConvTranspose1d == full ConvTranspose1d cropped, x = arange(8)
    [1,2,4], w = arange(24)*0.01-0.1 [2,3,4], stride 2, pad 1
    (src/models/sovits_decoder.rs:591-612)
  - im2col conv1d == conv1d, 16 ch x 4096, x = arange*0.001-0.5,
    w = arange*0.0001-0.02, (k, d) in {(3, 1), (7, 3)}, pad d(k-1)/2
    (src/utils/weights.rs:684-710); stored subsampled every 8th sample plus
    float64 checksums of the full output.
* ``decoder_tiny.npz`` -- whole-Generator outputs for seeded weights
  (synth.make_state_dict) at T0 in {1, 2, 3, 7}, B = 2, two inits; the
  state-dict checksum is stored to detect generator drift.
* ``encp_tiny.npz`` -- the EncP chains for seeded enc_p weights
  (synth.make_encp_state_dict with one layer per stack): add + LayerNorm,
  the FFN half, the output projection + prior sample, B = 2, T in {1, 4, 37}
  with lengths (T, ceil(T/2)); interpolation 37 -> 30 and 37 -> 50 frames.
* ``flow_tiny.npz`` -- flow inverse (ResidualCouplingBlock reverse, then
  z * y_mask) for seeded flow weights (synth.make_flow_state_dict), B = 2,
  T0 in {1, 5, 24} with lengths (T0, ceil(T0/2)), with and without g; the
  state-dict checksum again guards the generator.
"""
from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT / "tests"))


def load_pkg():
    pkg = ROOT / "gpt-sovits-rs_b200"
    spec = importlib.util.spec_from_file_location("gsv_b200", pkg / "__init__.py",
                                                  submodule_search_locations=[str(pkg)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["gsv_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def kats():
    out = {}
    out["lrelu_in"] = np.array([-2.0, 0.0, 3.0, -0.0], np.float32)
    out["lrelu_out"] = np.array([-0.2, 0.0, 3.0, -0.0], np.float32)
    # linear_interpolate_last_dim([0, 10], 4) (src/models/sovits_encp.rs:928-936)
    out["interp_in"] = np.array([[[0.0, 10.0]]], np.float32)
    out["interp_out"] = np.array([[[0.0, 2.5, 7.5, 10.0]]], np.float32)
    x = torch.arange(8, dtype=torch.float64).reshape(1, 2, 4)
    w = (torch.arange(24, dtype=torch.float64) * 0.01 - 0.1).reshape(2, 3, 4)
    out["convt_x"] = x.float().numpy()
    out["convt_w"] = w.float().numpy()
    out["convt_out"] = F.conv_transpose1d(x, w, stride=2, padding=1).float().numpy()
    C, L = 16, 4096
    xi = (torch.arange(C * L, dtype=torch.float64) * 0.001 - 0.5).reshape(1, C, L)
    for k, d in ((3, 1), (7, 3)):
        wi = (torch.arange(C * C * k, dtype=torch.float64) * 0.0001 - 0.02).reshape(C, C, k)
        y = F.conv1d(xi, wi, padding=d * (k - 1) // 2, dilation=d)
        out[f"im2col_k{k}d{d}_sub"] = y[..., ::8].float().numpy()
        out[f"im2col_k{k}d{d}_sum"] = np.array([y.sum().item(), y.abs().sum().item(),
                                                (y * y).sum().item()])
    return out


def decoders():
    gsv = load_pkg()
    import torch_ref
    out = {}
    for init, bias in (("unit", "rand"), ("n001", "zero")):
        sd = gsv.synth.make_state_dict(0, init=init, bias=bias)
        out[f"{init}_checksum"] = np.array(gsv.synth.checksum(sd))
        for T0 in (1, 2, 3, 7):
            z, g = gsv.synth.make_inputs(2, T0)
            out[f"{init}_T{T0}_wav"] = torch_ref.decoder_forward(sd, z, g).astype(np.float32)
    return out


def flows():
    gsv = load_pkg()
    import torch_ref
    out = {}
    for init in ("unit", "n001"):
        sd = gsv.synth.make_flow_state_dict(init=init)
        out[f"{init}_checksum"] = np.array(gsv.synth.checksum(sd))
        for T0 in (1, 5, 24):
            rng = np.random.default_rng(100 + T0)
            zp = rng.standard_normal((2, 192, T0)).astype(np.float32)
            g = rng.standard_normal((2, 512, 1)).astype(np.float32)
            lengths = np.array([T0, (T0 + 1) // 2], np.int32)
            out[f"T{T0}_zp"] = zp
            out[f"T{T0}_g"] = g
            out[f"T{T0}_len"] = lengths
            out[f"{init}_T{T0}_z"] = torch_ref.flow_inverse(sd, zp, g, lengths).astype(np.float32)
            out[f"{init}_T{T0}_z_nog"] = torch_ref.flow_inverse(sd, zp, None, None).astype(np.float32)
    return out


ENCP_LAYERS = {"encoder_ssl": 1, "encoder_text": 1, "encoder2": 1}


def encps():
    gsv = load_pkg()
    import torch_ref
    sd = gsv.synth.make_encp_state_dict(layers=ENCP_LAYERS)
    out = {"checksum": np.array(gsv.synth.checksum(sd))}
    for T in (1, 4, 37):
        rng = np.random.default_rng(200 + T)
        x = rng.standard_normal((2, 192, T)).astype(np.float32)
        y = rng.standard_normal((2, 192, T)).astype(np.float32)
        noise = rng.standard_normal((2, 192, T)).astype(np.float32)
        lengths = np.array([T, (T + 1) // 2], np.int32)
        out[f"T{T}_x"], out[f"T{T}_y"], out[f"T{T}_noise"], out[f"T{T}_len"] = x, y, noise, lengths
        p = "enc_p.encoder_text.norm_layers_1.0"
        out[f"T{T}_add_norm"] = torch_ref.layer_norm(x, sd[p + ".gamma"], sd[p + ".beta"], y=y).astype(np.float32)
        out[f"T{T}_ffn"] = torch_ref.encp_ffn(sd, "encoder_ssl", 0, x, lengths).astype(np.float32)
        m, logs, zp = torch_ref.encp_project(sd, x, lengths, noise, 0.5)
        out[f"T{T}_m"], out[f"T{T}_logs"], out[f"T{T}_zp"] = (a.astype(np.float32) for a in (m, logs, zp))
    x = out["T37_x"]
    for To in (30, 50):
        out[f"interp_{To}"] = torch_ref.interpolate(x, To).astype(np.float32)
    return out


if __name__ == "__main__":
    np.savez_compressed(HERE / "kat_ref.npz", **kats())
    np.savez_compressed(HERE / "decoder_tiny.npz", **decoders())
    np.savez_compressed(HERE / "flow_tiny.npz", **flows())
    np.savez_compressed(HERE / "encp_tiny.npz", **encps())
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")))
