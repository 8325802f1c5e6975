"""ctypes front-end of the CPU oracle (test infrastructure only).

The oracle is a C restatement of the gpt-sovits-rs SoVITS v2 Generator
(src/models/sovits_decoder.rs, src/utils/weights.rs of the reference crate).
Only tests/, ``__graft_entry__.smoke()`` and the CPU-baseline leg of bench.py
import this module, and only as the checker or the timed CPU baseline.  The
product path never routes through it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "_build" / "libgsv_oracle.so"
_lib = None


class OracleError(RuntimeError):
    pass


def build(force: bool = False) -> Path:
    """Compile the oracle shared library with its Makefile (gcc + OpenMP)."""
    src = _HERE / "gsv_oracle.c"
    if force or not _LIB_PATH.exists() or _LIB_PATH.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)
    return _LIB_PATH


class _Tensor(ctypes.Structure):
    _fields_ = [
        ("name", ctypes.c_char_p),
        ("data", ctypes.POINTER(ctypes.c_float)),
        ("ndim", ctypes.c_int),
        ("shape", ctypes.c_int64 * 4),
    ]


def _load():
    global _lib
    if _lib is None:
        build()
        lib = ctypes.CDLL(str(_LIB_PATH))
        fp = ctypes.POINTER(ctypes.c_float)
        lib.gsvo_last_error.restype = ctypes.c_char_p
        lib.gsvo_leaky_relu.argtypes = [fp, ctypes.c_int64, ctypes.c_float]
        lib.gsvo_weight_norm.argtypes = [fp, fp, ctypes.c_int, ctypes.c_int, ctypes.c_int, fp]
        lib.gsvo_conv1d.argtypes = [fp, ctypes.c_int, ctypes.c_int, ctypes.c_int, fp, ctypes.c_int,
                                    ctypes.c_int, ctypes.c_int, ctypes.c_int, fp, fp, ctypes.c_int]
        lib.gsvo_conv_transpose1d.argtypes = [fp, ctypes.c_int, ctypes.c_int, ctypes.c_int, fp,
                                              ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                              ctypes.c_int, fp, fp, ctypes.c_int]
        lib.gsvo_decoder_forward.argtypes = [ctypes.POINTER(_Tensor), ctypes.c_int, fp, fp,
                                             ctypes.c_int, ctypes.c_int, fp,
                                             ctypes.POINTER(fp), ctypes.c_int, ctypes.c_int]
        lib.gsvo_flow_inverse.argtypes = [ctypes.POINTER(_Tensor), ctypes.c_int, ctypes.c_char_p, fp,
                                          fp, ctypes.POINTER(ctypes.c_int), ctypes.c_int,
                                          ctypes.c_int, fp, ctypes.c_int, ctypes.c_int]
        ip = ctypes.POINTER(ctypes.c_int)
        lib.gsvo_layer_norm.argtypes = [fp, fp, fp, fp, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                        ctypes.c_float, ip, fp]
        lib.gsvo_encp_ffn.argtypes = [fp, ctypes.c_int, ctypes.c_int, ctypes.c_int, fp, fp, ctypes.c_int,
                                      ctypes.c_int, fp, fp, ctypes.c_int, fp, fp, ip, fp, ctypes.c_int]
        lib.gsvo_interpolate.argtypes = [fp, ctypes.c_int64, ctypes.c_int, ctypes.c_int, fp]
        lib.gsvo_encp_project.argtypes = [fp, ctypes.c_int, ctypes.c_int, ctypes.c_int, fp, fp, ctypes.c_int,
                                          ip, fp, ctypes.c_float, fp, fp, fp, ctypes.c_int]
        _lib = lib
    return _lib


def _fp(a):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float)) if a is not None else None


def _f32(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def _check(rc):
    if rc != 0:
        raise OracleError(_load().gsvo_last_error().decode())


def leaky_relu(x, slope: float):
    """Sign-bit LeakyReLU (reference src/models/sovits_decoder.rs:46-53)."""
    y = _f32(x).copy()
    _load().gsvo_leaky_relu(_fp(y), y.size, slope)
    return y


def weight_norm(v, g):
    """w = g * v / ||v|| per dim-0 slice (reference src/utils/weights.rs:589-614)."""
    v = _f32(v)
    g = _f32(g).reshape(-1)
    w = np.empty_like(v)
    _load().gsvo_weight_norm(_fp(v), _fp(g), v.shape[0], v.shape[1], v.shape[2], _fp(w))
    return w


def conv1d(x, w, bias=None, padding=0, dilation=1, acc64=True):
    """Conv1d, x [B,Cin,L], w [Cout,Cin,K] (reference src/utils/weights.rs:78-113)."""
    x, w = _f32(x), _f32(w)
    B, Cin, L = x.shape
    Cout, _, K = w.shape
    Lout = L + 2 * padding - dilation * (K - 1)
    y = np.empty((B, Cout, Lout), np.float32)
    b = _f32(bias) if bias is not None else None
    _check(_load().gsvo_conv1d(_fp(x), B, Cin, L, _fp(w), Cout, K, padding, dilation, _fp(b),
                               _fp(y), int(acc64)))
    return y


def conv_transpose1d(x, w, bias=None, stride=1, padding=0, acc64=True):
    """ConvTranspose1d as full conv + crop (reference src/models/sovits_decoder.rs:88-98)."""
    x, w = _f32(x), _f32(w)
    B, Cin, L = x.shape
    _, Cout, K = w.shape
    Lout = (L - 1) * stride + K - 2 * padding
    y = np.empty((B, Cout, Lout), np.float32)
    b = _f32(bias) if bias is not None else None
    _check(_load().gsvo_conv_transpose1d(_fp(x), B, Cin, L, _fp(w), Cout, K, stride, padding,
                                         _fp(b), _fp(y), int(acc64)))
    return y


def _tap_shapes(sd, B, T0):
    """Shapes of the forward_debug taps (reference src/models/sovits_decoder.rs:473-526)."""
    C = sd["dec.conv_pre.weight"].shape[0] if "dec.conv_pre.weight" in sd else 0
    L = T0
    shapes = [(B, C, L)]
    rates = [10, 8, 2, 2, 2]
    n_ups = 0
    for i in range(10):
        if f"dec.ups.{i}.weight_v" not in sd:
            continue
        s = rates[n_ups] if n_ups < 5 else 2
        k = sd[f"dec.ups.{i}.weight_v"].shape[2]
        L = (L - 1) * s + k - 2 * ((k - s) // 2)
        C = sd[f"dec.ups.{i}.weight_v"].shape[1]
        shapes += [(B, C, L), (B, C, L)]
        n_ups += 1
    post = sd.get("dec.conv_post.weight")
    shapes.append((B, post.shape[0] if post is not None else 1, L))
    return shapes


def decoder_forward(state_dict, z, g=None, acc64=True, taps=False, nthreads=0):
    """Decoder::forward (reference src/models/sovits_decoder.rs:386-458).

    state_dict maps safetensors ``dec.*`` keys to arrays (any float dtype; they
    are upcast to f32 like the reference's F32 SoVITS path).  Returns the
    flattened waveform (utterances concatenated) and, with ``taps``, the list
    [conv_pre+cond, ups0, rb0, ..., ups4, rb4, conv_post-before-tanh].
    """
    lib = _load()
    keep = []
    arr = (_Tensor * len(state_dict))()
    for i, (k, v) in enumerate(state_dict.items()):
        a = _f32(np.asarray(v, dtype=np.float32))
        keep.append(a)
        arr[i].name = k.encode()
        arr[i].data = _fp(a)
        arr[i].ndim = a.ndim
        for d in range(a.ndim):
            arr[i].shape[d] = a.shape[d]
    z = _f32(z)
    B, _, T0 = z.shape
    gg = _f32(g) if g is not None else None
    tap_bufs = None
    tap_ptrs = None
    out_len = _tap_shapes(state_dict, B, T0)[-1]
    if taps:
        tap_bufs = [np.empty(s, np.float32) for s in _tap_shapes(state_dict, B, T0)]
        tap_ptrs = (ctypes.POINTER(ctypes.c_float) * len(tap_bufs))(*[_fp(t) for t in tap_bufs])
    wav = np.empty(int(np.prod(out_len)), np.float32)
    _check(lib.gsvo_decoder_forward(arr, len(state_dict), _fp(z), _fp(gg), B, T0, _fp(wav),
                                    tap_ptrs, int(acc64), int(nthreads)))
    if taps:
        return wav, tap_bufs
    return wav


def _tensor_array(state_dict, prefix=None):
    items = [(k, v) for k, v in state_dict.items() if prefix is None or k.startswith(prefix)]
    keep = []
    arr = (_Tensor * max(1, len(items)))()
    for i, (k, v) in enumerate(items):
        a = _f32(np.asarray(v, dtype=np.float32))
        keep.append(a)
        arr[i].name = k.encode()
        arr[i].data = _fp(a)
        arr[i].ndim = a.ndim
        for d in range(a.ndim):
            arr[i].shape[d] = a.shape[d]
    return arr, len(items), keep


def flow_inverse(state_dict, z_p, g=None, lengths=None, prefix="flow.flows", acc64=True,
                 nthreads=0):
    """z = flow^-1(z_p) * y_mask: ResidualCouplingBlock::forward(reverse = true)
    (reference src/models/sovits_flow.rs:341-415) then src/models/sovits.rs:394.

    z_p [B, 192, T0]; g [B, gin, 1] or None; lengths [B] (valid frames) or None.
    """
    lib = _load()
    arr, n, keep = _tensor_array(state_dict, prefix + ".")
    z_p = _f32(z_p)
    B, C, T0 = z_p.shape
    gg = _f32(g) if g is not None else None
    ln = None
    if lengths is not None:
        la = np.ascontiguousarray(np.asarray(lengths, dtype=np.int32))
        keep.append(la)
        ln = la.ctypes.data_as(ctypes.POINTER(ctypes.c_int))
    z = np.empty((B, C, T0), np.float32)
    _check(lib.gsvo_flow_inverse(arr, n, prefix.encode(), _fp(z_p), _fp(gg), ln, B, T0, _fp(z),
                                 int(acc64), int(nthreads)))
    return z


def num_threads() -> int:
    return os.cpu_count() or 1


def _lengths(lengths, B, keep):
    if lengths is None:
        return None
    la = np.ascontiguousarray(np.asarray(lengths, dtype=np.int32))
    if la.shape != (B,):
        raise ValueError("lengths must hold one value per utterance")
    keep.append(la)
    return la.ctypes.data_as(ctypes.POINTER(ctypes.c_int))


def layer_norm(x, gamma, beta, y=None, lengths=None, eps: float = 1e-5):
    """LayerNorm over channels of x (+ y) [B, C, T], times x_mask with lengths
    (reference src/utils/weights.rs:461-502; src/models/sovits_encp.rs:102-109)."""
    x = _f32(x)
    B, C, T = x.shape
    yy = _f32(y) if y is not None else None
    keep = []
    out = np.empty_like(x)
    _check(_load().gsvo_layer_norm(_fp(x), _fp(yy), _fp(_f32(gamma)), _fp(_f32(beta)), B, C, T, eps,
                                   _lengths(lengths, B, keep), _fp(out)))
    return out


def encp_ffn(state_dict, stack: str, layer: int, x, lengths=None, acc64=True):
    """norm_layers_2[layer](x + conv_2(relu(conv_1(x)))) * x_mask of one enc_p
    encoder layer (reference src/models/sovits_encp.rs:104-109, 371-375)."""
    p = f"enc_p.{stack}"
    f = f"{p}.ffn_layers.{layer}"
    w1, w2 = _f32(state_dict[f + ".conv_1.weight"]), _f32(state_dict[f + ".conv_2.weight"])
    b1, b2 = _f32(state_dict[f + ".conv_1.bias"]), _f32(state_dict[f + ".conv_2.bias"])
    g = _f32(state_dict[f"{p}.norm_layers_2.{layer}.gamma"])
    be = _f32(state_dict[f"{p}.norm_layers_2.{layer}.beta"])
    x = _f32(x)
    B, C, T = x.shape
    keep = []
    out = np.empty_like(x)
    _check(_load().gsvo_encp_ffn(_fp(x), B, C, T, _fp(w1), _fp(b1), w1.shape[0], w1.shape[2], _fp(w2),
                                 _fp(b2), w2.shape[2], _fp(g), _fp(be), _lengths(lengths, B, keep),
                                 _fp(out), int(acc64)))
    return out


def speed_len(T: int, speed: float) -> int:
    """Frames after the speed change (reference src/models/sovits_encp.rs:857-867)."""
    s = np.float32(speed)
    if abs(s - np.float32(1.0)) <= np.finfo(np.float32).eps:
        return T
    if not np.isfinite(s) or s <= 0:
        raise OracleError(f"speed must be finite and positive, got {speed}")
    return max(1, int(np.float32(T) / s) + 1)


def interpolate(x, T_out: int):
    """linear_interpolate_last_dim (reference src/models/sovits_encp.rs:10-40)."""
    x = _f32(x)
    T = x.shape[-1]
    rows = int(np.prod(x.shape[:-1]))
    out = np.empty(x.shape[:-1] + (T_out,), np.float32)
    _check(_load().gsvo_interpolate(_fp(x), rows, T, T_out, _fp(out)))
    return out


def encp_project(state_dict, y, lengths=None, noise=None, noise_scale: float = 0.5, acc64=True):
    """(m, logs, z_p) of the EncP output projection and the prior sample
    (reference src/models/sovits_encp.rs:871-879; src/models/sovits.rs:378-385)."""
    w = _f32(state_dict["enc_p.proj.weight"])
    b = _f32(state_dict["enc_p.proj.bias"]) if "enc_p.proj.bias" in state_dict else None
    y = _f32(y)
    B, C, T = y.shape
    co = w.shape[0] // 2
    keep = []
    nz = _f32(noise) if noise is not None else None
    m = np.empty((B, co, T), np.float32)
    logs = np.empty_like(m)
    zp = np.empty_like(m) if nz is not None else None
    _check(_load().gsvo_encp_project(_fp(y), B, C, T, _fp(w), _fp(b), w.shape[0], _lengths(lengths, B, keep),
                                     _fp(nz), noise_scale, _fp(m), _fp(logs), _fp(zp), int(acc64)))
    return m, logs, zp
