"""gsvdec -- B200 (sm_100a) SoVITS v2 Generator of gpt-sovits-rs, Python side.

This module is the host-side mirror of the reference's decoder interface,
``impl Decoder { fn load(&StateDict, &Device, DType); fn forward(&self, x,
Option<&Tensor>) -> Result<Vec<f32>> }`` (src/models/sovits_decoder.rs:231,
386 of the reference crate), over the C ABI of ``libgsvdec.so``
(include/gsvdec.h).  The CUDA library is the only compute path: if it is
missing, importing ``Decoder`` raises instead of falling back to anything.

Reference errors (``crate::Error`` values, src/lib.rs:76-97) surface as
:class:`GsvDecError` carrying the library's status code and message.
"""
from __future__ import annotations

import ctypes
from pathlib import Path
from typing import Mapping, Optional, Sequence

import numpy as np

from . import shard, synth  # noqa: F401  (multi-GPU plumbing, seeded weights / inputs)

PKG_DIR = Path(__file__).resolve().parent
LIB_PATH = PKG_DIR / "_build" / "libgsvdec.so"

GSV_OK = 0
STATUS = {
    -1: "GSV_E_INVALID_ARG", -2: "GSV_E_MISSING_KEY", -3: "GSV_E_SHAPE", -4: "GSV_E_DTYPE",
    -5: "GSV_E_CUDA", -6: "GSV_E_OOM", -7: "GSV_E_UNSUPPORTED", -8: "GSV_E_TIMEOUT",
}
MODES = {"fp32": 0, "bf16": 1, "fp32tc": 2}  # fp32tc: fp32 accuracy on tensor cores (three bf16 pieces)
MEM_HOST, MEM_DEVICE, MEM_HOST_ASYNC = 0, 1, 2
DT_F32, DT_F16, DT_BF16 = 0, 1, 2

# Every symbol include/gsvdec.h declares (checked by the CPU test suite).
EXPORTS = (
    "gsvdec_create", "gsvdec_create_from_file", "gsvdec_destroy", "gsvdec_get_info",
    "gsvdec_forward", "gsvdec_forward_chunk", "gsvdec_forward_taps", "gsvdec_set_stage_timing",
    "gsvdec_get_stage_times", "gsvdec_launch_count", "gsvdec_get_launch_stats",
    "gsvdec_forward_noalloc", "gsvdec_noalloc_scratch_bytes", "gsvdec_layer_forward",
    "gsvdec_layer_names", "gsvdec_last_error", "gsvdec_flow_info", "gsvdec_flow_inverse",
    "gsvdec_flow_decode", "gsvdec_encp_info", "gsvdec_encp_add_norm", "gsvdec_encp_ffn", "gsvdec_encp_layer",
    "gsvdec_encp_speed_len", "gsvdec_encp_interpolate", "gsvdec_encp_project",
    "gsvdec_forward_multi", "gsvdec_plan_multi", "gsvdec_sync_status", "gsvdec_selftest_wait",
    "gsvdec_set_alloc_fail_after", "gsvdec_workspace_bytes",
)

# EncP encoder stacks (GSV_ENCP_SSL / _TEXT / _2), by their enc_p.* names.
ENCP_STACKS = {"encoder_ssl": 0, "encoder_text": 1, "encoder2": 2}


class GsvDecError(RuntimeError):
    """A non-zero status from libgsvdec."""

    def __init__(self, code: int, message: str):
        super().__init__(f"{STATUS.get(code, code)}: {message}")
        self.code = code
        self.status = STATUS.get(code, str(code))


class _Tensor(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("dtype", ctypes.c_int), ("ndim", ctypes.c_int),
                ("shape", ctypes.c_int64 * 4), ("data", ctypes.c_void_p)]


class _Info(ctypes.Structure):
    _fields_ = [("mode", ctypes.c_int), ("device", ctypes.c_int), ("in_channels", ctypes.c_int),
                ("gin_channels", ctypes.c_int), ("n_upsamples", ctypes.c_int),
                ("n_resblocks", ctypes.c_int), ("hop", ctypes.c_int),
                ("receptive_halo", ctypes.c_int), ("weight_bytes", ctypes.c_int64)]


class _LaunchStat(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 48), ("kind", ctypes.c_int), ("n_convs", ctypes.c_int),
                ("flops", ctypes.c_double), ("bytes", ctypes.c_double),
                ("conv_flops", ctypes.c_double * 6), ("conv_bytes", ctypes.c_double * 6),
                ("ms", ctypes.c_float)]


_lib = None


def library(path: Optional[Path] = None) -> ctypes.CDLL:
    """Load libgsvdec.so (built in-tree by build.py).  Raises if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise ImportError(f"libgsvdec.so not built at {p}; run gpt-sovits-rs_b200/build.py "
                          "(there is no CPU fallback)")
    lib = ctypes.CDLL(str(p))
    vp, i, fp = ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_float)
    lib.gsvdec_last_error.restype = ctypes.c_char_p
    lib.gsvdec_create.argtypes = [ctypes.POINTER(_Tensor), i, i, i, ctypes.POINTER(vp)]
    lib.gsvdec_create_from_file.argtypes = [ctypes.c_char_p, i, i, ctypes.POINTER(vp)]
    lib.gsvdec_destroy.argtypes = [vp]
    lib.gsvdec_get_info.argtypes = [vp, ctypes.POINTER(_Info)]
    lib.gsvdec_forward.argtypes = [vp, vp, vp, vp, i, i, vp, i, vp]
    lib.gsvdec_forward_chunk.argtypes = [vp, vp, vp, i, i, i, i, vp, i, vp]
    lib.gsvdec_forward_taps.argtypes = [vp, vp, vp, i, i, vp, ctypes.POINTER(fp), i]
    lib.gsvdec_set_stage_timing.argtypes = [vp, i]
    lib.gsvdec_get_stage_times.argtypes = [vp, fp]
    lib.gsvdec_launch_count.argtypes = [vp, i, i, ctypes.POINTER(i)]
    lib.gsvdec_get_launch_stats.argtypes = [vp, ctypes.POINTER(_LaunchStat), i, ctypes.POINTER(i)]
    lib.gsvdec_forward_noalloc.argtypes = [vp, vp, vp, vp, i, i, vp, vp]
    lib.gsvdec_noalloc_scratch_bytes.restype = ctypes.c_int64
    lib.gsvdec_layer_forward.argtypes = [vp, ctypes.c_char_p, vp, i, i, vp, i, vp]
    lib.gsvdec_layer_names.argtypes = [vp, ctypes.c_char_p, ctypes.c_size_t,
                                       ctypes.POINTER(ctypes.c_size_t)]
    lib.gsvdec_flow_info.argtypes = [vp, ctypes.POINTER(i), ctypes.POINTER(i)]
    lib.gsvdec_flow_inverse.argtypes = [vp, vp, vp, vp, i, i, vp, i, vp]
    lib.gsvdec_flow_decode.argtypes = [vp, vp, vp, vp, i, i, vp, i, vp]
    lib.gsvdec_encp_info.argtypes = [vp, ctypes.POINTER(i), ctypes.POINTER(i), ctypes.POINTER(i),
                                     ctypes.POINTER(i)]
    lib.gsvdec_encp_add_norm.argtypes = [vp, i, i, i, vp, vp, vp, i, i, vp, i, vp]
    lib.gsvdec_encp_ffn.argtypes = [vp, i, i, vp, vp, i, i, vp, i, vp]
    lib.gsvdec_encp_layer.argtypes = [vp, i, i, vp, vp, vp, i, i, vp, i, vp]
    lib.gsvdec_encp_speed_len.argtypes = [i, ctypes.c_float, ctypes.POINTER(i)]
    lib.gsvdec_encp_interpolate.argtypes = [vp, vp, i, i, i, i, vp, i, vp]
    lib.gsvdec_encp_project.argtypes = [vp, vp, vp, i, i, vp, ctypes.c_float, vp, vp, vp, i, vp]
    lib.gsvdec_forward_multi.argtypes = [ctypes.POINTER(vp), i, vp, vp, vp, i, i, vp, i, vp]
    lib.gsvdec_plan_multi.argtypes = [vp, i, i, i, vp, vp]
    lib.gsvdec_sync_status.argtypes = [vp, vp]
    lib.gsvdec_selftest_wait.argtypes = [vp, ctypes.c_int64, vp]
    lib.gsvdec_set_alloc_fail_after.argtypes = [i]
    lib.gsvdec_workspace_bytes.argtypes = [vp, ctypes.POINTER(ctypes.c_int64)]
    _lib = lib
    return lib


def _check(rc: int) -> None:
    if rc != GSV_OK:
        raise GsvDecError(rc, library().gsvdec_last_error().decode())


def _as_weight(v):
    """(array kept alive, dtype code) for a state-dict value (numpy or torch)."""
    try:
        import torch
        if isinstance(v, torch.Tensor):
            t = v.detach().cpu().contiguous()
            if t.dtype == torch.bfloat16:
                return t.view(torch.int16).numpy(), DT_BF16
            if t.dtype == torch.float16:
                return t.numpy(), DT_F16
            return t.float().numpy(), DT_F32
    except ImportError:  # pragma: no cover
        pass
    a = np.ascontiguousarray(np.asarray(v))
    if a.dtype == np.float16:
        return a, DT_F16
    return np.ascontiguousarray(a, dtype=np.float32), DT_F32


def _host_f32(a):
    if a is None:
        return None
    try:
        import torch
        if isinstance(a, torch.Tensor):
            a = a.detach().cpu().float().numpy()
    except ImportError:  # pragma: no cover
        pass
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


class Decoder:
    """The Generator on one B200: ``Decoder.load(...)`` then ``forward(z, g)``."""

    def __init__(self, handle: ctypes.c_void_p):
        self._h = handle
        info = _Info()
        _check(library().gsvdec_get_info(self._h, ctypes.byref(info)))
        self.info = {f: getattr(info, f) for f, _ in _Info._fields_}
        self.mode = {v: k for k, v in MODES.items()}[info.mode]
        self.hop = info.hop

    # -- Decoder::load ------------------------------------------------------
    @classmethod
    def load(cls, state_dict: Mapping[str, object], device: int = 0, mode: str = "bf16") -> "Decoder":
        """Decoder::load (src/models/sovits_decoder.rs:231-293) from ``dec.*`` tensors."""
        if mode not in MODES:
            raise ValueError(f"mode must be one of {sorted(MODES)}")
        keep = []
        items = list(state_dict.items())
        arr = (_Tensor * max(1, len(items)))()
        for idx, (k, v) in enumerate(items):
            a, dt = _as_weight(v)
            if a.ndim < 1 or a.ndim > 4:
                raise ValueError(f"{k}: unsupported rank {a.ndim}")
            name = k.encode()
            keep += [a, name]
            arr[idx].name = name
            arr[idx].dtype = dt
            arr[idx].ndim = a.ndim
            for d in range(a.ndim):
                arr[idx].shape[d] = a.shape[d]
            arr[idx].data = a.ctypes.data
        h = ctypes.c_void_p()
        _check(library().gsvdec_create(arr, len(items), MODES[mode], device, ctypes.byref(h)))
        return cls(h)

    @classmethod
    def load_file(cls, path: str, device: int = 0, mode: str = "bf16") -> "Decoder":
        """Decoder::load straight from a safetensors checkpoint (dec.* keys)."""
        h = ctypes.c_void_p()
        _check(library().gsvdec_create_from_file(str(path).encode(), MODES[mode], device,
                                                 ctypes.byref(h)))
        return cls(h)

    def close(self) -> None:
        if getattr(self, "_h", None):
            library().gsvdec_destroy(self._h)
            self._h = None

    def __del__(self):  # pragma: no cover - best effort
        try:
            self.close()
        except Exception:
            pass

    def out_len(self, T0: int) -> int:
        return T0 * self.hop

    # -- Decoder::forward ---------------------------------------------------
    def forward(self, x, g=None, lengths: Optional[Sequence[int]] = None, out=None,
                stream: Optional[int] = None) -> np.ndarray:
        """Decoder::forward (src/models/sovits_decoder.rs:386-458) on host arrays.

        x [B, C_in, T0], g [B, gin, 1] or None; returns the flattened fp32
        waveform (utterances concatenated), like the reference's Vec<f32>.
        ``out`` may be a preallocated (e.g. pinned) float32 array of B*hop*T0;
        ``stream`` a cudaStream_t handle as an int (default: legacy stream).
        """
        z = _host_f32(x)
        if z.ndim != 3:
            raise ValueError("x must be [B, C, T]")
        B, _, T0 = z.shape
        gg = _host_f32(g)
        ln = None if lengths is None else np.ascontiguousarray(np.asarray(lengths, np.int32))
        if ln is not None and ln.shape != (B,):
            raise ValueError("lengths must hold one value per utterance")
        if out is None:
            out = np.empty(B * self.out_len(T0), np.float32)
        elif out.dtype != np.float32 or out.size != B * self.out_len(T0) or not out.flags.c_contiguous:
            raise ValueError("out must be a contiguous float32 array of B*hop*T0 samples")
        _check(library().gsvdec_forward(self._h, _ptr(z), _ptr(gg), _ptr(ln), B, T0, _ptr(out),
                                        MEM_HOST, None if stream is None else ctypes.c_void_p(stream)))
        return out

    def forward_device(self, z, g=None, lengths=None, out=None, stream=None):
        """Stream-async forward on CUDA tensors (torch) already on the device."""
        import torch
        B, _, T0 = z.shape
        assert z.is_cuda and z.dtype == torch.float32 and z.is_contiguous()
        if out is None:
            out = torch.empty(B * self.out_len(T0), device=z.device, dtype=torch.float32)
        st = stream if stream is not None else torch.cuda.current_stream(z.device).cuda_stream
        _check(library().gsvdec_forward(
            self._h, ctypes.c_void_p(z.data_ptr()),
            None if g is None else ctypes.c_void_p(g.data_ptr()),
            None if lengths is None else ctypes.c_void_p(lengths.data_ptr()),
            B, T0, ctypes.c_void_p(out.data_ptr()), MEM_DEVICE, ctypes.c_void_p(st)))
        return out

    def forward_async(self, z, g=None, lengths=None, out=None, stream=None):
        """Overlapped host-memory forward (GSV_MEM_HOST_ASYNC) on CPU tensors --
        pinned for the copies to overlap: the copies in, the decode and the copy
        out are queued and the call returns; ``out`` is complete once
        ``stream`` (default: torch's current stream) has passed the call.
        Consecutive calls overlap one call's copies with the next decode.  The
        tensors must stay alive and untouched until then."""
        import torch
        B, _, T0 = z.shape
        assert not z.is_cuda and z.dtype == torch.float32 and z.is_contiguous()
        if out is None:
            out = torch.empty(B * self.out_len(T0), dtype=torch.float32, pin_memory=True)
        assert not out.is_cuda and out.numel() == B * self.out_len(T0) and out.is_contiguous()
        if stream is None:
            stream = torch.cuda.current_stream(self.info["device"]).cuda_stream
        p = lambda t: None if t is None else ctypes.c_void_p(t.data_ptr())  # noqa: E731
        _check(library().gsvdec_forward(self._h, p(z), p(g), p(lengths), B, T0, p(out), MEM_HOST_ASYNC,
                                        ctypes.c_void_p(stream)))
        return out

    def forward_noalloc(self, z, g=None, lengths=None, out=None, stream=None):
        """Allocation-free forward on CUDA tensors: the layers' scratch comes from
        the library's static device array (for callers that cannot allocate
        device memory at call time), so only small requests fit; ``out`` must
        then be preallocated by the caller to stay allocation-free."""
        import torch
        B, _, T0 = z.shape
        assert z.is_cuda and z.dtype == torch.float32 and z.is_contiguous()
        if out is None:
            out = torch.empty(B * self.out_len(T0), device=z.device, dtype=torch.float32)
        st = stream if stream is not None else torch.cuda.current_stream(z.device).cuda_stream
        _check(library().gsvdec_forward_noalloc(
            self._h, ctypes.c_void_p(z.data_ptr()),
            None if g is None else ctypes.c_void_p(g.data_ptr()),
            None if lengths is None else ctypes.c_void_p(lengths.data_ptr()),
            B, T0, ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(st)))
        return out

    # -- status of stream-async calls, failure hooks --------------------------
    def sync_status(self, stream=None) -> None:
        """Wait for ``stream`` (default: torch's current stream on this device)
        and raise GsvDecError(GSV_E_TIMEOUT) if a device wait of a
        stream-async call on this handle gave up (gsvdec_sync_status)."""
        if stream is None:
            import torch
            stream = torch.cuda.current_stream(self.info["device"]).cuda_stream
        _check(library().gsvdec_sync_status(self._h, ctypes.c_void_p(stream)))

    def selftest_wait(self, limit_ns: int = 1_000_000, stream=None) -> None:
        """Queue the give-up self-test (gsvdec_selftest_wait): one bounded wait
        that nothing completes, reported like a decode kernel's give-up."""
        if stream is None:
            import torch
            stream = torch.cuda.current_stream(self.info["device"]).cuda_stream
        _check(library().gsvdec_selftest_wait(self._h, int(limit_ns), ctypes.c_void_p(stream)))

    def workspace_bytes(self) -> int:
        """Device bytes held for per-call workspaces (not the weights)."""
        n = ctypes.c_int64()
        _check(library().gsvdec_workspace_bytes(self._h, ctypes.byref(n)))
        return n.value

    # -- ResidualCouplingBlock::forward(reverse = true) ----------------------
    @property
    def flow_couplings(self) -> int:
        """Coupling layers of the flow loaded with this handle (0: none)."""
        n, c = ctypes.c_int(), ctypes.c_int()
        _check(library().gsvdec_flow_info(self._h, ctypes.byref(n), ctypes.byref(c)))
        return n.value

    def flow_inverse(self, z_p, g=None, lengths: Optional[Sequence[int]] = None) -> np.ndarray:
        """z = flow^-1(z_p) * y_mask (src/models/sovits_flow.rs:385-405 with
        reverse = true, src/models/sovits.rs:391-394) on host arrays:
        z_p [B, 192, T0], g [B, gin, 1] or None, lengths [B] or None."""
        zp = _host_f32(z_p)
        if zp.ndim != 3:
            raise ValueError("z_p must be [B, C, T]")
        B, C, T0 = zp.shape
        gg = _host_f32(g)
        ln = None if lengths is None else np.ascontiguousarray(np.asarray(lengths, np.int32))
        if ln is not None and ln.shape != (B,):
            raise ValueError("lengths must hold one value per utterance")
        z = np.empty((B, C, T0), np.float32)
        _check(library().gsvdec_flow_inverse(self._h, _ptr(zp), _ptr(gg), _ptr(ln), B, T0, _ptr(z),
                                             MEM_HOST, None))
        return z

    def flow_decode(self, z_p, g=None, lengths: Optional[Sequence[int]] = None, out=None) -> np.ndarray:
        """Flow inverse then Decoder::forward with the same g and lengths
        (src/models/sovits.rs:389-400): the flattened fp32 waveform."""
        zp = _host_f32(z_p)
        B, _, T0 = zp.shape
        gg = _host_f32(g)
        ln = None if lengths is None else np.ascontiguousarray(np.asarray(lengths, np.int32))
        if out is None:
            out = np.empty(B * self.out_len(T0), np.float32)
        _check(library().gsvdec_flow_decode(self._h, _ptr(zp), _ptr(gg), _ptr(ln), B, T0, _ptr(out),
                                            MEM_HOST, None))
        return out

    def flow_inverse_device(self, z_p, g=None, lengths=None, out=None, stream=None):
        """Stream-async flow inverse on CUDA tensors (torch)."""
        import torch
        B, C, T0 = z_p.shape
        assert z_p.is_cuda and z_p.dtype == torch.float32 and z_p.is_contiguous()
        if out is None:
            out = torch.empty((B, C, T0), device=z_p.device, dtype=torch.float32)
        st = stream if stream is not None else torch.cuda.current_stream(z_p.device).cuda_stream
        _check(library().gsvdec_flow_inverse(
            self._h, ctypes.c_void_p(z_p.data_ptr()), None if g is None else ctypes.c_void_p(g.data_ptr()),
            None if lengths is None else ctypes.c_void_p(lengths.data_ptr()), B, T0,
            ctypes.c_void_p(out.data_ptr()), MEM_DEVICE, ctypes.c_void_p(st)))
        return out

    def flow_decode_device(self, z_p, g=None, lengths=None, out=None, stream=None):
        """Stream-async flow inverse + decoder on CUDA tensors (torch)."""
        import torch
        B, _, T0 = z_p.shape
        assert z_p.is_cuda and z_p.dtype == torch.float32 and z_p.is_contiguous()
        if out is None:
            out = torch.empty(B * self.out_len(T0), device=z_p.device, dtype=torch.float32)
        st = stream if stream is not None else torch.cuda.current_stream(z_p.device).cuda_stream
        _check(library().gsvdec_flow_decode(
            self._h, ctypes.c_void_p(z_p.data_ptr()), None if g is None else ctypes.c_void_p(g.data_ptr()),
            None if lengths is None else ctypes.c_void_p(lengths.data_ptr()), B, T0,
            ctypes.c_void_p(out.data_ptr()), MEM_DEVICE, ctypes.c_void_p(st)))
        return out

    # -- EncP fused elementwise chains (src/models/sovits_encp.rs) -----------
    @property
    def encp_info(self) -> dict:
        """Layers per enc_p stack, hidden / FFN filter / projection widths."""
        n = (ctypes.c_int * 3)()
        c, f, p = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        _check(library().gsvdec_encp_info(self._h, n, ctypes.byref(c), ctypes.byref(f), ctypes.byref(p)))
        return {"layers": {k: n[v] for k, v in ENCP_STACKS.items()}, "channels": c.value,
                "filter_channels": f.value, "proj_channels": p.value}

    @staticmethod
    def _stack(stack) -> int:
        return ENCP_STACKS[stack] if isinstance(stack, str) else int(stack)

    @staticmethod
    def _lengths(lengths, B):
        if lengths is None:
            return None
        ln = np.ascontiguousarray(np.asarray(lengths, np.int32))
        if ln.shape != (B,):
            raise ValueError("lengths must hold one value per utterance")
        return ln

    def encp_add_norm(self, stack, layer: int, x, y=None, lengths=None, norm: int = 1) -> np.ndarray:
        """norm_layers_<norm>[layer](x + y) (src/models/sovits_encp.rs:102, :107),
        times x_mask when lengths are given; x, y [B, C, T]."""
        xa, ya = _host_f32(x), _host_f32(y)
        B, C, T = xa.shape
        if ya is not None and ya.shape != xa.shape:
            raise ValueError("x and y must have the same shape")
        ln = self._lengths(lengths, B)
        out = np.empty_like(xa)
        _check(library().gsvdec_encp_add_norm(self._h, self._stack(stack), layer, norm, _ptr(xa), _ptr(ya),
                                              _ptr(ln), B, T, _ptr(out), MEM_HOST, None))
        return out

    def encp_ffn(self, stack, layer: int, x, lengths=None) -> np.ndarray:
        """norm_layers_2[layer](x + FFN(x)) * x_mask (src/models/sovits_encp.rs:104-109)."""
        xa = _host_f32(x)
        B, C, T = xa.shape
        ln = self._lengths(lengths, B)
        out = np.empty_like(xa)
        _check(library().gsvdec_encp_ffn(self._h, self._stack(stack), layer, _ptr(xa), _ptr(ln), B, T,
                                         _ptr(out), MEM_HOST, None))
        return out

    def encp_layer(self, stack, layer: int, x, attn=None, lengths=None) -> np.ndarray:
        """EncoderLayer::forward after the attention (src/models/sovits_encp.rs:98-110):
        norm2(h + FFN(h)) * x_mask, h = norm1(x + attn)."""
        xa, aa = _host_f32(x), _host_f32(attn)
        B, C, T = xa.shape
        if aa is not None and aa.shape != xa.shape:
            raise ValueError("x and attn must have the same shape")
        ln = self._lengths(lengths, B)
        out = np.empty_like(xa)
        _check(library().gsvdec_encp_layer(self._h, self._stack(stack), layer, _ptr(xa), _ptr(aa), _ptr(ln), B,
                                           T, _ptr(out), MEM_HOST, None))
        return out

    def encp_layer_device(self, stack, layer: int, x, attn=None, lengths=None, out=None, stream=None):
        """Stream-async encp_layer on CUDA tensors (torch)."""
        import torch
        B, C, T = x.shape
        assert x.is_cuda and x.dtype == torch.float32 and x.is_contiguous()
        if out is None:
            out = torch.empty_like(x)
        st = stream if stream is not None else torch.cuda.current_stream(x.device).cuda_stream
        p = lambda t: None if t is None else ctypes.c_void_p(t.data_ptr())  # noqa: E731
        _check(library().gsvdec_encp_layer(self._h, self._stack(stack), layer, p(x), p(attn), p(lengths), B, T,
                                           p(out), MEM_DEVICE, ctypes.c_void_p(st)))
        return out

    def encp_ffn_device(self, stack, layer: int, x, lengths=None, out=None, stream=None):
        """Stream-async FFN half on CUDA tensors (torch): x, out [B, C, T] fp32."""
        import torch
        B, C, T = x.shape
        assert x.is_cuda and x.dtype == torch.float32 and x.is_contiguous()
        if out is None:
            out = torch.empty_like(x)
        st = stream if stream is not None else torch.cuda.current_stream(x.device).cuda_stream
        _check(library().gsvdec_encp_ffn(
            self._h, self._stack(stack), layer, ctypes.c_void_p(x.data_ptr()),
            None if lengths is None else ctypes.c_void_p(lengths.data_ptr()), B, T,
            ctypes.c_void_p(out.data_ptr()), MEM_DEVICE, ctypes.c_void_p(st)))
        return out

    def encp_add_norm_device(self, stack, layer: int, x, y=None, lengths=None, out=None, norm: int = 1,
                             stream=None):
        """Stream-async add + LayerNorm on CUDA tensors (torch): x, y, out [B, C, T] fp32."""
        import torch
        B, C, T = x.shape
        assert x.is_cuda and x.dtype == torch.float32 and x.is_contiguous()
        if out is None:
            out = torch.empty_like(x)
        st = stream if stream is not None else torch.cuda.current_stream(x.device).cuda_stream
        _check(library().gsvdec_encp_add_norm(
            self._h, self._stack(stack), layer, norm, ctypes.c_void_p(x.data_ptr()),
            None if y is None else ctypes.c_void_p(y.data_ptr()),
            None if lengths is None else ctypes.c_void_p(lengths.data_ptr()), B, T,
            ctypes.c_void_p(out.data_ptr()), MEM_DEVICE, ctypes.c_void_p(st)))
        return out

    def encp_project_device(self, y, lengths=None, noise=None, noise_scale: float = 0.5, m=None, logs=None,
                            z_p=None, stream=None):
        """Stream-async projection + prior sample on CUDA tensors (torch); any of
        m / logs / z_p may be None (not written)."""
        import torch
        B, C, T = y.shape
        assert y.is_cuda and y.dtype == torch.float32 and y.is_contiguous()
        st = stream if stream is not None else torch.cuda.current_stream(y.device).cuda_stream
        p = lambda t: None if t is None else ctypes.c_void_p(t.data_ptr())  # noqa: E731
        _check(library().gsvdec_encp_project(self._h, p(y), p(lengths), B, T, p(noise), noise_scale, p(m),
                                             p(logs), p(z_p), MEM_DEVICE, ctypes.c_void_p(st)))
        return m, logs, z_p

    @staticmethod
    def encp_speed_len(T: int, speed: float) -> int:
        """Frames after the speed change (src/models/sovits_encp.rs:857-867)."""
        n = ctypes.c_int()
        _check(library().gsvdec_encp_speed_len(T, speed, ctypes.byref(n)))
        return n.value

    def encp_interpolate(self, y, speed: float = None, T_out: int = None) -> np.ndarray:
        """linear_interpolate_last_dim (src/models/sovits_encp.rs:10-40) of
        y [B, C, T] to T_out frames (or the length `speed` gives)."""
        ya = _host_f32(y)
        B, C, T = ya.shape
        if T_out is None:
            T_out = self.encp_speed_len(T, 1.0 if speed is None else speed)
        out = np.empty((B, C, T_out), np.float32)
        _check(library().gsvdec_encp_interpolate(self._h, _ptr(ya), B, C, T, T_out, _ptr(out),
                                                 MEM_HOST, None))
        return out

    def encp_project(self, y, lengths=None, noise=None, noise_scale: float = 0.5):
        """(m, logs, z_p): stats = proj(y) * y_mask, logs clamped to [-5, 2]
        (src/models/sovits_encp.rs:871-879), z_p = m + noise * exp(logs) *
        noise_scale (src/models/sovits.rs:378-385); z_p is None without noise."""
        ya = _host_f32(y)
        B, C, T = ya.shape
        ln = self._lengths(lengths, B)
        co = self.encp_info["proj_channels"] // 2
        na = _host_f32(noise)
        if na is not None and na.shape != (B, co, T):
            raise ValueError(f"noise must be [{B}, {co}, {T}]")
        m = np.empty((B, co, T), np.float32)
        logs = np.empty_like(m)
        zp = np.empty_like(m) if na is not None else None
        _check(library().gsvdec_encp_project(self._h, _ptr(ya), _ptr(ln), B, T, _ptr(na), noise_scale,
                                             _ptr(m), _ptr(logs), _ptr(zp), MEM_HOST, None))
        return m, logs, zp

    def forward_chunk(self, x, g, frame_begin: int, frame_end: int, halo: int = 16) -> np.ndarray:
        """Frames [frame_begin, frame_end) of one utterance with a recomputed halo."""
        z = _host_f32(x)
        if z.ndim != 3 or z.shape[0] != 1:
            raise ValueError("x must be [1, C, T]")
        gg = _host_f32(g)
        wav = np.empty(max(1, frame_end - frame_begin) * self.hop, np.float32)
        _check(library().gsvdec_forward_chunk(self._h, _ptr(z), _ptr(gg), z.shape[2], frame_begin,
                                              frame_end, halo, _ptr(wav), MEM_HOST, None))
        return wav

    def forward_chunk_device(self, z, g, frame_begin: int, frame_end: int, halo: int = 16, out=None,
                             stream=None):
        """forward_chunk on CUDA tensors (z [1, C, T0], g [1, gin, 1]): frames
        [frame_begin, frame_end) with a recomputed halo, into a device tensor."""
        import torch
        assert z.is_cuda and z.dtype == torch.float32 and z.is_contiguous() and z.shape[0] == 1
        n = max(1, frame_end - frame_begin) * self.hop
        if out is None:
            out = torch.empty(n, device=z.device, dtype=torch.float32)
        st = stream if stream is not None else torch.cuda.current_stream(z.device).cuda_stream
        _check(library().gsvdec_forward_chunk(
            self._h, ctypes.c_void_p(z.data_ptr()), None if g is None else ctypes.c_void_p(g.data_ptr()),
            z.shape[2], frame_begin, frame_end, halo, ctypes.c_void_p(out.data_ptr()), MEM_DEVICE,
            ctypes.c_void_p(st)))
        return out

    def forward_debug(self, x, g=None):
        """Decoder::forward_debug (src/models/sovits_decoder.rs:473-526): the
        waveform plus the per-layer taps [conv_pre(+cond), ups0, rb0, ...,
        conv_post before tanh] in the reference's [B, C, T] layout."""
        z = _host_f32(x)
        B, _, T0 = z.shape
        gg = _host_f32(g)
        shapes = self.tap_shapes(B, T0)
        taps = [np.empty(s, np.float32) for s in shapes]
        fp = ctypes.POINTER(ctypes.c_float)
        ptrs = (fp * len(taps))(*[t.ctypes.data_as(fp) for t in taps])
        wav = np.empty(B * self.out_len(T0), np.float32)
        _check(library().gsvdec_forward_taps(self._h, _ptr(z), _ptr(gg), B, T0, _ptr(wav), ptrs,
                                             len(taps)))
        return wav, taps

    def layer_names(self) -> list:
        """dec.* prefixes of the Generator's conv layers, in forward order."""
        n = ctypes.c_size_t()
        _check(library().gsvdec_layer_names(self._h, None, 0, ctypes.byref(n)))
        buf = ctypes.create_string_buffer(n.value)
        _check(library().gsvdec_layer_names(self._h, buf, n.value, ctypes.byref(n)))
        return [x for x in buf.value.decode().split("\n") if x]

    def layer_forward(self, name: str, x, out_len: Optional[int] = None) -> np.ndarray:
        """One conv layer on host x [B, Cin, L] -> [B, Cout, Lout] (bias, no activation)."""
        xx = _host_f32(x)
        B, _, L = xx.shape
        if name == "dec.conv_post":
            cout, lout = 1, L
        else:
            cout, lout = self._layer_out(name, L)
        y = np.empty((B, cout, lout), np.float32)
        _check(library().gsvdec_layer_forward(self._h, name.encode(), _ptr(xx), B, L, _ptr(y),
                                              MEM_HOST, None))
        return y

    def layer_forward_device(self, name: str, x, y, stream=None):
        """Device-pointer variant (torch CUDA tensors, fp32, reference layout)."""
        import torch
        B, _, L = x.shape
        st = stream if stream is not None else torch.cuda.current_stream(x.device).cuda_stream
        _check(library().gsvdec_layer_forward(self._h, name.encode(), ctypes.c_void_p(x.data_ptr()),
                                              B, L, ctypes.c_void_p(y.data_ptr()), MEM_DEVICE,
                                              ctypes.c_void_p(st)))
        return y

    def _layer_out(self, name: str, L: int):
        # Output width / length by the load rules (src/models/sovits_decoder.rs:146-194, 551-576).
        if name == "dec.conv_pre":
            return 512, L
        if name.startswith("dec.ups."):
            i = int(name.split(".")[2])
            rates, kernels, chans = (10, 8, 2, 2, 2), (16, 16, 8, 2, 2), (256, 128, 64, 32, 16)
            s, k = rates[i], kernels[i]
            return chans[i], (L - 1) * s + k - 2 * ((k - s) // 2)
        r = int(name.split(".")[2])
        return (256, 128, 64, 32, 16)[r // 3], L

    def tap_shapes(self, B: int, T0: int):
        chans = [512, 256, 128, 64, 32, 16]
        rates = [10, 8, 2, 2, 2]
        shapes = [(B, chans[0], T0)]
        L = T0
        for i in range(self.info["n_upsamples"]):
            L *= rates[i] if i < 5 else 2
            shapes += [(B, chans[i + 1] if i + 1 < len(chans) else -1, L)] * 2
        shapes.append((B, 1, L))
        return shapes

    # -- profiling ----------------------------------------------------------
    def set_stage_timing(self, level) -> None:
        """0 off, 1 stage events, 2 stage + per-launch events."""
        _check(library().gsvdec_set_stage_timing(self._h, int(level)))

    def launch_stats(self) -> list:
        """Per-launch profile of the last forward (needs set_stage_timing(2))."""
        n = ctypes.c_int()
        _check(library().gsvdec_get_launch_stats(self._h, None, 0, ctypes.byref(n)))
        arr = (_LaunchStat * max(1, n.value))()
        _check(library().gsvdec_get_launch_stats(self._h, arr, n.value, ctypes.byref(n)))
        return [{"name": a.name.decode(), "kind": a.kind, "n_convs": a.n_convs, "flops": a.flops,
                 "bytes": a.bytes, "conv_flops": list(a.conv_flops)[:max(1, a.n_convs)],
                 "conv_bytes": list(a.conv_bytes)[:max(1, a.n_convs)], "ms": a.ms}
                for a in arr[:n.value]]

    def stage_times(self) -> dict:
        ms = (ctypes.c_float * 5)()
        _check(library().gsvdec_get_stage_times(self._h, ms))
        return dict(zip(("pre", "upsample", "resblocks", "post", "total"), list(ms)))

    def launch_count(self) -> int:
        n = ctypes.c_int()
        _check(library().gsvdec_launch_count(self._h, 0, 0, ctypes.byref(n)))
        return n.value


# -- several devices ------------------------------------------------------------

def set_alloc_fail_after(n: int) -> None:
    """Allocation-failure hook: the next ``n`` device allocations of the library
    succeed and later ones fail with GSV_E_OOM; ``n < 0`` turns it off."""
    _check(library().gsvdec_set_alloc_fail_after(int(n)))


def plan_multi(lengths, n_workers: int, T0: Optional[int] = None):
    """The utterance plan of gsvdec_forward_multi: (worker, bucket) per utterance
    (-1 for empty utterances)."""
    ln = np.ascontiguousarray(np.asarray(lengths, np.int32))
    B = ln.size
    T = int(ln.max()) if T0 is None else int(T0)
    worker = np.empty(B, np.int32)
    bucket = np.empty(B, np.int32)
    _check(library().gsvdec_plan_multi(_ptr(ln), B, max(T, 1), n_workers, _ptr(worker), _ptr(bucket)))
    return worker, bucket


def _handles(decoders):
    arr = (ctypes.c_void_p * len(decoders))()
    for i, d in enumerate(decoders):
        arr[i] = d._h
    return arr


def forward_multi(decoders: Sequence["Decoder"], x, g=None, lengths: Optional[Sequence[int]] = None,
                  out=None) -> np.ndarray:
    """Decoder::forward over several handles (one per device) on host arrays:
    utterances split over the handles, or one utterance (B = 1) split in time
    with a recomputed halo; the flattened waveform, as forward returns it."""
    z = _host_f32(x)
    if z.ndim != 3:
        raise ValueError("x must be [B, C, T]")
    B, _, T0 = z.shape
    gg = _host_f32(g)
    ln = None if lengths is None else np.ascontiguousarray(np.asarray(lengths, np.int32))
    if ln is not None and ln.shape != (B,):
        raise ValueError("lengths must hold one value per utterance")
    hop = decoders[0].hop
    if out is None:
        out = np.empty(B * hop * T0, np.float32)
    elif out.dtype != np.float32 or out.size != B * hop * T0 or not out.flags.c_contiguous:
        raise ValueError("out must be a contiguous float32 array of B*hop*T0 samples")
    _check(library().gsvdec_forward_multi(_handles(decoders), len(decoders), _ptr(z), _ptr(gg), _ptr(ln), B, T0,
                                          _ptr(out), MEM_HOST, None))
    return out


def forward_multi_device(decoders: Sequence["Decoder"], z, g=None, lengths=None, out=None, stream=None):
    """forward_multi on CUDA tensors of decoders[0]'s device (stream-async in
    that device's stream order)."""
    import torch
    B, _, T0 = z.shape
    assert z.is_cuda and z.dtype == torch.float32 and z.is_contiguous()
    hop = decoders[0].hop
    if out is None:
        out = torch.empty(B * hop * T0, device=z.device, dtype=torch.float32)
    st = stream if stream is not None else torch.cuda.current_stream(z.device).cuda_stream
    p = lambda t: None if t is None else ctypes.c_void_p(t.data_ptr())  # noqa: E731
    _check(library().gsvdec_forward_multi(_handles(decoders), len(decoders), p(z), p(g), p(lengths), B, T0,
                                          p(out), MEM_DEVICE, ctypes.c_void_p(st)))
    return out
