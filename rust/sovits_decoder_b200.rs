//! B200 SoVITS Generator behind the crate's `Decoder` interface, over the C ABI
//! of libgsvdec (include/gsvdec.h).
//!
//! Drop-in for `Decoder` (src/models/sovits_decoder.rs:212-221): `load` keeps
//! `Decoder::load(&StateDict, &Device, DType)` (:231) and `forward` keeps
//! `Decoder::forward(&self, &Tensor, Option<&Tensor>) -> Result<Vec<f32>>`
//! (:386).  The two call sites to switch are `SoVITSModel`'s field
//! (src/models/sovits.rs:39), its load (`:199`) and its decode
//! (`self.decoder.forward(&z_masked, Some(&ge))`, `:400`).  Weights stay the
//! `dec.*` safetensors tensors; errors map onto `crate::Error`
//! (src/lib.rs:76-97) as the weight loader does.
//!
//! Not compiled here: this repository's build image has no Rust toolchain.
//! Place as src/models/sovits_decoder_b200.rs with rust/build.rs as the
//! crate's build.rs.

use crate::utils::StateDict;
use crate::{Error, Result};
use candle_core::{DType, Device, Tensor};
use std::ffi::{c_char, c_int, c_void, CStr, CString};
use std::path::Path;

#[repr(C)]
struct GsvTensor {
    name: *const c_char,
    dtype: c_int,
    ndim: c_int,
    shape: [i64; 4],
    data: *const c_void,
}

#[repr(C)]
struct GsvDec {
    _private: [u8; 0],
}

#[repr(C)]
#[derive(Default)]
struct GsvInfo {
    mode: c_int,
    device: c_int,
    in_channels: c_int,
    gin_channels: c_int,
    n_upsamples: c_int,
    n_resblocks: c_int,
    hop: c_int,
    receptive_halo: c_int,
    weight_bytes: i64,
}

const GSV_DTYPE_F32: c_int = 0;
const GSV_DTYPE_F16: c_int = 1;
const GSV_DTYPE_BF16: c_int = 2;
const GSV_MODE_FP32: c_int = 0;
const GSV_MODE_BF16: c_int = 1;
/// The decoder at fp32 accuracy on the tensor cores (three bf16 pieces per
/// value); for `DecoderB200::load_mode`.
pub const GSV_MODE_FP32_TC: c_int = 2;
const GSV_MEM_HOST: c_int = 0;
const GSV_MEM_DEVICE: c_int = 1;

#[link(name = "gsvdec")]
extern "C" {
    fn gsvdec_create(t: *const GsvTensor, n: c_int, mode: c_int, device: c_int, out: *mut *mut GsvDec) -> c_int;
    fn gsvdec_create_from_file(path: *const c_char, mode: c_int, device: c_int, out: *mut *mut GsvDec) -> c_int;
    fn gsvdec_destroy(h: *mut GsvDec) -> c_int;
    fn gsvdec_get_info(h: *const GsvDec, info: *mut GsvInfo) -> c_int;
    fn gsvdec_forward(h: *mut GsvDec, z: *const f32, g: *const f32, lengths: *const i32, b: c_int, t0: c_int,
                      wav: *mut f32, mem_kind: c_int, stream: *mut c_void) -> c_int;
    fn gsvdec_flow_decode(h: *mut GsvDec, z_p: *const f32, g: *const f32, lengths: *const i32, b: c_int,
                          t0: c_int, wav: *mut f32, mem_kind: c_int, stream: *mut c_void) -> c_int;
    fn gsvdec_forward_multi(hs: *const *mut GsvDec, n: c_int, z: *const f32, g: *const f32, lengths: *const i32,
                            b: c_int, t0: c_int, wav: *mut f32, mem_kind: c_int, stream: *mut c_void) -> c_int;
    fn gsvdec_sync_status(h: *mut GsvDec, stream: *mut c_void) -> c_int;
    fn gsvdec_last_error() -> *const c_char;
}

/// Status -> crate::Error: load-time codes (-2 missing key, -3 shape, -4
/// dtype) are ModelLoadError, as src/utils/weights.rs reports them; the rest
/// (bad argument, CUDA, OOM, unsupported device, device wait timeout) are
/// InferenceError.
fn check(rc: c_int) -> Result<()> {
    if rc == 0 {
        return Ok(());
    }
    let msg = unsafe { CStr::from_ptr(gsvdec_last_error()) }.to_string_lossy().into_owned();
    Err(if (-4..=-2).contains(&rc) { Error::ModelLoadError(msg) } else { Error::InferenceError(msg) })
}

fn ordinal(device: &Device) -> Result<c_int> {
    match device {
        Device::Cuda(d) => Ok(d.ordinal() as c_int),
        _ => Err(Error::InferenceError("DecoderB200 needs a CUDA (B200) device; there is no CPU fallback".into())),
    }
}

fn mode_of(dtype: DType) -> c_int {
    // F32 keeps the reference's arithmetic (src/config/mod.rs:52-58); any
    // half type selects bf16 operands with fp32 accumulation on tcgen05.
    if dtype == DType::F32 { GSV_MODE_FP32 } else { GSV_MODE_BF16 }
}

pub struct DecoderB200 {
    h: *mut GsvDec,
    hop: usize,
}

// One handle owns one device's weights and workspace.  forward is not
// re-entrant per handle; the crate's callers already serialise it behind the
// pipeline mutex (src/server/pipeline_registry.rs:204-205).
unsafe impl Send for DecoderB200 {}

impl std::fmt::Debug for DecoderB200 {
    fn fmt(&self, f: &mut std::fmt::Formatter<'_>) -> std::fmt::Result {
        f.debug_struct("DecoderB200").field("hop", &self.hop).finish()
    }
}

impl DecoderB200 {
    fn wrap(h: *mut GsvDec) -> Result<Self> {
        let mut info = GsvInfo::default();
        check(unsafe { gsvdec_get_info(h, &mut info) })?;
        Ok(Self { h, hop: info.hop as usize })
    }

    /// Decoder::load (src/models/sovits_decoder.rs:231-293): the dec.* tensors
    /// (F32 / F16 / BF16, src/utils/weights.rs:140-151) handed over by pointer;
    /// the library folds weight norm, packs and uploads them.
    pub fn load(sd: &StateDict, device: &Device, dtype: DType) -> Result<Self> {
        Self::load_mode(sd, device, mode_of(dtype))
    }

    /// `load` with an explicit arithmetic mode (GSV_MODE_FP32_TC: F32 results at
    /// tensor-core speed).
    pub fn load_mode(sd: &StateDict, device: &Device, mode: c_int) -> Result<Self> {
        let dev = ordinal(device)?;
        let mut names = Vec::new();
        let mut bytes: Vec<Vec<u8>> = Vec::new();
        let mut ts = Vec::new();
        for k in sd.keys().filter(|k| k.starts_with("dec.") || k.starts_with("flow.") || k.starts_with("enc_p.")) {
            let t = sd.get(k)?.to_device(&Device::Cpu)?;
            let (code, t) = match t.dtype() {
                DType::F16 => (GSV_DTYPE_F16, t),
                DType::BF16 => (GSV_DTYPE_BF16, t),
                _ => (GSV_DTYPE_F32, t.to_dtype(DType::F32)?),
            };
            let dims = t.dims().to_vec();
            if dims.is_empty() || dims.len() > 4 {
                return Err(Error::ModelLoadError(format!("{k}: rank {} not supported", dims.len())));
            }
            let raw: Vec<u8> = match code {
                GSV_DTYPE_F32 => t.flatten_all()?.to_vec1::<f32>()?.iter().flat_map(|v| v.to_le_bytes()).collect(),
                GSV_DTYPE_F16 => t.flatten_all()?.to_vec1::<half::f16>()?.iter().flat_map(|v| v.to_le_bytes()).collect(),
                _ => t.flatten_all()?.to_vec1::<half::bf16>()?.iter().flat_map(|v| v.to_le_bytes()).collect(),
            };
            let mut shape = [0i64; 4];
            for (i, d) in dims.iter().enumerate() {
                shape[i] = *d as i64;
            }
            let name = CString::new(k.as_str()).map_err(|e| Error::ModelLoadError(e.to_string()))?;
            ts.push(GsvTensor { name: name.as_ptr(), dtype: code, ndim: dims.len() as c_int, shape,
                                data: raw.as_ptr() as *const c_void });
            names.push(name);
            bytes.push(raw);
        }
        let mut h = std::ptr::null_mut();
        check(unsafe { gsvdec_create(ts.as_ptr(), ts.len() as c_int, mode, dev, &mut h) })?;
        Self::wrap(h)
    }

    /// The same from a safetensors checkpoint (src/bin/gpt-sovits-convert.rs
    /// layout), read by the library's mmap loader.
    pub fn load_file(path: &Path, device: &Device, dtype: DType) -> Result<Self> {
        let p = CString::new(path.to_string_lossy().as_bytes()).map_err(|e| Error::ModelLoadError(e.to_string()))?;
        let mut h = std::ptr::null_mut();
        check(unsafe { gsvdec_create_from_file(p.as_ptr(), mode_of(dtype), ordinal(device)?, &mut h) })?;
        Self::wrap(h)
    }

    fn host_f32(t: &Tensor) -> Result<Vec<f32>> {
        Ok(t.to_device(&Device::Cpu)?.to_dtype(DType::F32)?.flatten_all()?.to_vec1::<f32>()?)
    }

    /// Decoder::forward (src/models/sovits_decoder.rs:386-458): z [B, 192, T0],
    /// g [B, gin, 1] or None -> the flattened B * hop * T0 waveform.
    pub fn forward(&self, x: &Tensor, g: Option<&Tensor>) -> Result<Vec<f32>> {
        let (b, _, t0) = x.dims3()?;
        let z = Self::host_f32(x)?;
        let gv = match g { Some(g) => Some(Self::host_f32(g)?), None => None };
        let mut wav = vec![0f32; b * t0 * self.hop];
        check(unsafe {
            gsvdec_forward(self.h, z.as_ptr(), gv.as_ref().map_or(std::ptr::null(), |v| v.as_ptr()),
                           std::ptr::null(), b as c_int, t0 as c_int, wav.as_mut_ptr(), GSV_MEM_HOST,
                           std::ptr::null_mut())
        })?;
        Ok(wav)
    }

    /// A right-padded batch with per-utterance frame counts: utterance i is
    /// decoded exactly as if alone; samples past hop * lengths[i] are 0.
    pub fn forward_lengths(&self, x: &Tensor, g: Option<&Tensor>, lengths: &[i32]) -> Result<Vec<f32>> {
        let (b, _, t0) = x.dims3()?;
        if lengths.len() != b {
            return Err(Error::InferenceError("one length per utterance".into()));
        }
        let z = Self::host_f32(x)?;
        let gv = match g { Some(g) => Some(Self::host_f32(g)?), None => None };
        let mut wav = vec![0f32; b * t0 * self.hop];
        check(unsafe {
            gsvdec_forward(self.h, z.as_ptr(), gv.as_ref().map_or(std::ptr::null(), |v| v.as_ptr()),
                           lengths.as_ptr(), b as c_int, t0 as c_int, wav.as_mut_ptr(), GSV_MEM_HOST,
                           std::ptr::null_mut())
        })?;
        Ok(wav)
    }

    /// Flow inverse + y_mask + decoder (src/models/sovits.rs:389-400) in one
    /// call, when the handle was loaded with the flow.flows.* tensors.
    pub fn flow_decode(&self, z_p: &Tensor, g: Option<&Tensor>, lengths: Option<&[i32]>) -> Result<Vec<f32>> {
        let (b, _, t0) = z_p.dims3()?;
        let z = Self::host_f32(z_p)?;
        let gv = match g { Some(g) => Some(Self::host_f32(g)?), None => None };
        let mut wav = vec![0f32; b * t0 * self.hop];
        check(unsafe {
            gsvdec_flow_decode(self.h, z.as_ptr(), gv.as_ref().map_or(std::ptr::null(), |v| v.as_ptr()),
                               lengths.map_or(std::ptr::null(), |l| l.as_ptr()), b as c_int, t0 as c_int,
                               wav.as_mut_ptr(), GSV_MEM_HOST, std::ptr::null_mut())
        })?;
        Ok(wav)
    }

    /// Stream-async forward on device memory (e.g. Candle CUDA buffers):
    /// z, g, wav are device pointers on this handle's device, `stream` a
    /// cudaStream_t of it.  Use `sync_status` to learn of a device-side
    /// give-up.
    ///
    /// # Safety
    /// The pointers must address live device buffers of the stated sizes.
    pub unsafe fn forward_device(&self, z: *const f32, g: *const f32, b: usize, t0: usize, wav: *mut f32,
                                 stream: *mut c_void) -> Result<()> {
        check(gsvdec_forward(self.h, z, g, std::ptr::null(), b as c_int, t0 as c_int, wav, GSV_MEM_DEVICE, stream))
    }

    /// Waits for `stream` and reports a device wait that gave up in an earlier
    /// stream-async call on this handle.
    pub fn sync_status(&self, stream: *mut c_void) -> Result<()> {
        check(unsafe { gsvdec_sync_status(self.h, stream) })
    }
}

impl Drop for DecoderB200 {
    fn drop(&mut self) {
        unsafe {
            gsvdec_destroy(self.h);
        }
    }
}

/// One decoder per GPU of the box, decoding one batch (or one long utterance)
/// across all of them through gsvdec_forward_multi.
pub struct DecoderB200Multi {
    decs: Vec<DecoderB200>,
}

impl DecoderB200Multi {
    pub fn load_file(path: &Path, devices: &[Device], dtype: DType) -> Result<Self> {
        let decs = devices.iter().map(|d| DecoderB200::load_file(path, d, dtype)).collect::<Result<Vec<_>>>()?;
        if decs.is_empty() {
            return Err(Error::InferenceError("no devices".into()));
        }
        Ok(Self { decs })
    }

    /// Same result as DecoderB200::forward_lengths on one device: utterances
    /// split over the devices (B > 1), or one utterance split in time with a
    /// recomputed halo (B == 1).
    pub fn forward(&self, x: &Tensor, g: Option<&Tensor>, lengths: Option<&[i32]>) -> Result<Vec<f32>> {
        let (b, _, t0) = x.dims3()?;
        let z = DecoderB200::host_f32(x)?;
        let gv = match g { Some(g) => Some(DecoderB200::host_f32(g)?), None => None };
        let hs: Vec<*mut GsvDec> = self.decs.iter().map(|d| d.h).collect();
        let mut wav = vec![0f32; b * t0 * self.decs[0].hop];
        check(unsafe {
            gsvdec_forward_multi(hs.as_ptr(), hs.len() as c_int, z.as_ptr(),
                                 gv.as_ref().map_or(std::ptr::null(), |v| v.as_ptr()),
                                 lengths.map_or(std::ptr::null(), |l| l.as_ptr()), b as c_int, t0 as c_int,
                                 wav.as_mut_ptr(), GSV_MEM_HOST, std::ptr::null_mut())
        })?;
        Ok(wav)
    }
}
