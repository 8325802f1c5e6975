"""The C ABI without a GPU: the library loads, exports every declared symbol,
and rejects bad weights / arguments with the documented status codes before
touching a device."""
from __future__ import annotations

import ctypes
import re

import numpy as np
import pytest

from conftest import ROOT


def header_functions():
    text = (ROOT / "include" / "gsvdec.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(gsvdec_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol(gsv):
    lib = gsv.library()
    declared = header_functions()
    assert declared, "no functions parsed from include/gsvdec.h"
    for name in declared:
        assert hasattr(lib, name), f"{name} declared in gsvdec.h but not exported"
    assert sorted(gsv.EXPORTS) == declared


def test_missing_key_is_reported(gsv):
    sd = gsv.synth.make_state_dict(0)
    del sd["dec.ups.2.weight_g"]
    with pytest.raises(gsv.GsvDecError) as e:
        gsv.Decoder.load(sd, mode="fp32")
    assert e.value.status == "GSV_E_MISSING_KEY"
    assert "dec.ups.2.weight_g" in str(e.value)


def test_resblock_kernel_rule_is_enforced(gsv):
    # k = [3,7,11][rb % 3] (src/models/sovits_decoder.rs:180-181).
    sd = gsv.synth.make_state_dict(0)
    v = sd["dec.resblocks.4.convs1.0.weight_v"]
    sd["dec.resblocks.4.convs1.0.weight_v"] = np.concatenate([v, v[..., :2]], axis=2)
    with pytest.raises(gsv.GsvDecError) as e:
        gsv.Decoder.load(sd, mode="bf16")
    assert e.value.status == "GSV_E_SHAPE"


def test_shape_mismatch_is_reported(gsv):
    sd = gsv.synth.make_state_dict(0)
    sd["dec.conv_post.weight"] = np.zeros((1, 32, 7), np.float32)
    with pytest.raises(gsv.GsvDecError) as e:
        gsv.Decoder.load(sd, mode="fp32")
    assert e.value.status == "GSV_E_SHAPE"


def test_bad_dtype_and_mode(gsv):
    lib = gsv.library()
    a = np.zeros((512, 192, 7), np.float32)
    t = (gsv._Tensor * 1)()
    t[0].name = b"dec.conv_pre.weight"
    t[0].dtype = 9
    t[0].ndim = 3
    for d in range(3):
        t[0].shape[d] = a.shape[d]
    t[0].data = a.ctypes.data
    h = ctypes.c_void_p()
    assert lib.gsvdec_create(t, 1, 0, 0, ctypes.byref(h)) == -4
    assert lib.gsvdec_create(t, 1, 7, 0, ctypes.byref(h)) == -1
    assert lib.gsvdec_create(t, 1, 3, 0, ctypes.byref(h)) == -1  # modes are FP32 0, BF16 1, FP32_TC 2
    assert "mode" in lib.gsvdec_last_error().decode()
    assert lib.gsvdec_create(t, 1, 2, 0, ctypes.byref(h)) == -4  # FP32_TC accepted: the bad dtype is next
    assert lib.gsvdec_create(None, 0, 0, 0, ctypes.byref(h)) == -1
    assert lib.gsvdec_forward(None, None, None, None, 1, 1, None, 0, None) == -1
    assert "NULL" in lib.gsvdec_last_error().decode()


def test_half_precision_weights_are_accepted_by_the_loader(gsv):
    # F16 / BF16 tensors are upcast like src/utils/weights.rs:140-151; without a
    # GPU the call gets past loading and fails on the device check.
    import torch
    sd = {k: torch.from_numpy(v).to(torch.bfloat16) for k, v in gsv.synth.make_state_dict(0).items()}
    sd["dec.conv_pre.weight"] = sd["dec.conv_pre.weight"].to(torch.float16)
    if torch.cuda.is_available():
        pytest.skip("a GPU is present; covered by the GPU tests")
    with pytest.raises(gsv.GsvDecError) as e:
        gsv.Decoder.load(sd, mode="fp32")
    assert e.value.status in ("GSV_E_CUDA", "GSV_E_INVALID_ARG", "GSV_E_UNSUPPORTED")
    assert "device" in str(e.value).lower() or "cuda" in str(e.value).lower()


def test_safetensors_file_loader(gsv, tmp_path):
    from safetensors.numpy import save_file
    bad = tmp_path / "bad.safetensors"
    bad.write_bytes(b"\x10\x00\x00\x00\x00\x00\x00\x00{not json}")
    with pytest.raises(gsv.GsvDecError, match="Failed to parse safetensors"):
        gsv.Decoder.load_file(bad, mode="fp32")
    with pytest.raises(gsv.GsvDecError, match="Failed to open"):
        gsv.Decoder.load_file(tmp_path / "missing.safetensors")
    sd = gsv.synth.make_state_dict(0)
    sd["enc_p.dummy"] = np.zeros(3, np.int64)  # non-decoder keys are ignored
    good = tmp_path / "good.safetensors"
    save_file(sd, str(good))
    nodec = tmp_path / "nodec.safetensors"
    save_file({"enc_p.x": np.zeros(2, np.float32)}, str(nodec))
    with pytest.raises(gsv.GsvDecError) as e:
        gsv.Decoder.load_file(nodec)
    assert e.value.status == "GSV_E_MISSING_KEY"
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present; covered by the GPU tests")
    with pytest.raises(gsv.GsvDecError) as e:
        gsv.Decoder.load_file(good, mode="fp32")
    assert "parse" not in str(e.value)  # parsed fine; failed at the device
