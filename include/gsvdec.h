/*
 * gsvdec.h -- C ABI of libgsvdec, the B200 (sm_100a) SoVITS v2 Generator
 * (HiFi-GAN style vocoder) of gpt-sovits-rs.
 *
 * The library replaces the reference crate's decoder call path:
 *   Decoder::load(&StateDict, &Device, DType)   src/models/sovits_decoder.rs:231
 *   Decoder::forward(&self, &Tensor, Option<&Tensor>) -> Result<Vec<f32>>
 *                                                src/models/sovits_decoder.rs:386
 * called by SoVITSModel::synthesize_with_speed_and_sv (src/models/sovits.rs:400).
 * Weights are consumed as the unchanged safetensors `dec.*` tensors
 * (src/models/sovits_decoder.rs:231-293, src/utils/weights.rs:116-162).
 *
 * Conventions: every call returns GSV_OK (0) or a negative GSV_E_* code and
 * leaves a thread-local message for gsvdec_last_error().  No torch or CUDA
 * types appear in the signatures: a stream is passed as `void*`
 * (a cudaStream_t, NULL = the legacy default stream).  One handle owns one
 * device's packed weights and workspace; calls on one handle must not
 * overlap (the reference serialises forward behind a mutex,
 * src/server/pipeline_registry.rs:204-205); distinct handles are independent.
 */
#ifndef GSVDEC_H
#define GSVDEC_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes.  The reference reports these cases as crate::Error values
 * (src/lib.rs:76-97): ModelLoadError for missing keys / bad shapes,
 * InferenceError for runtime failures. */
#define GSV_OK 0
#define GSV_E_INVALID_ARG (-1)  /* null pointer, bad size, bad enum */
#define GSV_E_MISSING_KEY (-2)  /* a required dec.* tensor is absent */
#define GSV_E_SHAPE (-3)        /* tensor shapes disagree with the Generator layout */
#define GSV_E_DTYPE (-4)        /* tensor dtype not in {F32, F16, BF16} */
#define GSV_E_CUDA (-5)         /* CUDA runtime / driver error */
#define GSV_E_OOM (-6)          /* device allocation failed */
#define GSV_E_UNSUPPORTED (-7)  /* device is not sm_100 / feature not built */
#define GSV_E_TIMEOUT (-8)      /* a bounded device wait gave up */

/* Element types of a weight tensor: the safetensors dtypes the reference
 * loader accepts for float weights (src/utils/weights.rs:140-151). */
#define GSV_DTYPE_F32 0
#define GSV_DTYPE_F16 1
#define GSV_DTYPE_BF16 2

/* Arithmetic modes.  FP32: fp32 CUDA-core convolutions (the reference's own
 * F32 arithmetic, src/config/mod.rs:52-58).  BF16: bf16 operands and
 * activations, fp32 accumulation on tcgen05 tensor cores.  FP32_TC: the
 * decoder forward at fp32 accuracy on tcgen05 tensor cores -- every
 * activation and weight held as the exact sum of three bf16 pieces, each
 * product formed from the six piece products that reach 2^-24 of it, fp32
 * accumulation; the flow, EncP chains and single-layer calls of such a handle
 * run as in FP32 mode. */
#define GSV_MODE_FP32 0
#define GSV_MODE_BF16 1
#define GSV_MODE_FP32_TC 2

/* Where the z / g / lengths / wav pointers of a forward call live. */
#define GSV_MEM_HOST 0    /* host memory; the call copies in and out and syncs the stream */
#define GSV_MEM_DEVICE 1  /* device memory on the handle's device; the call is stream-async */
/* Host memory, stream-async and overlapped (gsvdec_forward / _chunk only):
 * the call queues the copy of z / g / lengths in, the decode and the copy of
 * wav out on three internal streams of the handle and returns; wav is
 * complete in `stream` order.  Consecutive calls alternate two staging
 * slots, so one call's copies run while the calls next to it decode.  The
 * host buffers must stay untouched (and wav unread) until `stream` has
 * passed the call; pinned buffers are needed for the copies to overlap.
 * The decode is ordered after earlier calls on this handle, not after other
 * work queued on `stream`.  Errors of the device waits as for stream-async
 * calls (gsvdec_sync_status). */
#define GSV_MEM_HOST_ASYNC 2

typedef struct gsvdec_tensor {
  const char* name;   /* safetensors key, e.g. "dec.ups.0.weight_v" */
  int dtype;          /* GSV_DTYPE_* */
  int ndim;           /* 1..4 */
  int64_t shape[4];
  const void* data;   /* host pointer, contiguous row-major */
} gsvdec_tensor;

typedef struct gsvdec gsvdec_t;

typedef struct gsvdec_info {
  int mode;             /* GSV_MODE_* */
  int device;
  int in_channels;      /* conv_pre input width (192 for v2) */
  int gin_channels;     /* cond input width, 0 when dec.cond is absent */
  int n_upsamples;      /* 5 for v2 */
  int n_resblocks;      /* 15 for v2 */
  int hop;              /* product of the upsample strides: samples per frame (640) */
  int receptive_halo;   /* input frames each side that influence one output frame */
  int64_t weight_bytes; /* packed device weight bytes */
} gsvdec_info;

/* Decoder::load (src/models/sovits_decoder.rs:231-293): folds weight norm
 * (src/utils/weights.rs:589-614), packs the weights for `mode` and uploads
 * them to `device`.  The tensors are only read during the call. */
int gsvdec_create(const gsvdec_tensor* tensors, int n_tensors, int mode, int device,
                  gsvdec_t** out);

/* Same as gsvdec_create, reading the tensors from a safetensors file
 * (the format written by src/bin/gpt-sovits-convert.rs:282-309 and read by
 * src/utils/weights.rs:116-162).  Only the tensors the handle uses are read:
 * dec.*, flow.flows.* and the enc_p.* FFN / LayerNorm / proj tensors. */
int gsvdec_create_from_file(const char* safetensors_path, int mode, int device, gsvdec_t** out);

int gsvdec_destroy(gsvdec_t* h);

int gsvdec_get_info(const gsvdec_t* h, gsvdec_info* info);

/* Decoder::forward (src/models/sovits_decoder.rs:386-458).
 *   z       [B, in_channels, T0] fp32 (the flow output times y_mask)
 *   g       [B, gin_channels, 1] fp32, or NULL (no cond add, :393-399)
 *   lengths [B] valid frame counts, or NULL (all T0, the reference's
 *           behaviour).  With lengths, utterance b is decoded exactly as if it
 *           were alone with length lengths[b]; its samples past
 *           hop*lengths[b] are written as 0.
 *   wav     [B, hop*T0] fp32, utterances concatenated (the flattened Vec<f32>
 *           of :458).
 * mem_kind says where z/g/lengths/wav live (GSV_MEM_*). */
int gsvdec_forward(gsvdec_t* h, const float* z, const float* g, const int32_t* lengths, int B,
                   int T0, float* wav, int mem_kind, void* stream);

/* One time chunk of a single long utterance (z [1, in_channels, T0]):
 * decodes frames [frame_begin, frame_end) using `halo` extra input frames on
 * each side (clamped to the utterance) and writes the hop*(frame_end -
 * frame_begin) samples of that span to wav.  With halo >= receptive_halo the
 * samples equal those of the whole-utterance forward.  No reference
 * counterpart: the reference decodes an utterance whole
 * (src/models/sovits_decoder.rs:386). */
int gsvdec_forward_chunk(gsvdec_t* h, const float* z, const float* g, int T0, int frame_begin,
                         int frame_end, int halo, float* wav, int mem_kind, void* stream);

/* Per-layer taps of Decoder::forward_debug (src/models/sovits_decoder.rs:
 * 473-526), in the reference's [B, C, T] layout, fp32, host memory:
 *   taps[0]          conv_pre (+cond)            [B, 512, T0]
 *   taps[1 + 2i]     after upsample i            [B, C_i, L_i]
 *   taps[2 + 2i]     resblock average, stage i   [B, C_i, L_i]
 *   taps[1 + 2 n_up] conv_post before tanh       [B, 1, L]
 * n_taps must be 2 + 2 n_upsamples; any entry may be NULL. */
int gsvdec_forward_taps(gsvdec_t* h, const float* z, const float* g, int B, int T0,
                        float* wav, float* const* taps, int n_taps);

/* Flow inverse of the SoVITS v2 model, present when gsvdec_create received
 * flow.flows.* tensors (ResidualCouplingBlock::load, src/models/sovits_flow.rs:
 * 346-368; the layer list of ResidualCouplingLayer::load :186-223 and WN::load
 * :19-109).  *n_couplings = 0 when the handle has no flow. */
int gsvdec_flow_info(const gsvdec_t* h, int* n_couplings, int* channels);

/* z = flow^-1(z_p) * y_mask: ResidualCouplingBlock::forward(x, x_mask, g,
 * reverse = true) (src/models/sovits_flow.rs:385-405) followed by
 * z.broadcast_mul(&y_mask) (src/models/sovits.rs:391-394).  z_p and z are
 * [B, C, T0] fp32 (C = 192), g [B, gin, 1] or NULL (no conditioning),
 * lengths [B] valid frames or NULL (all T0: y_mask of ones).  Host or device
 * pointers per mem_kind.  Only mean-only coupling layers (post with C/2
 * outputs, as in v2) are supported (GSV_E_UNSUPPORTED otherwise). */
int gsvdec_flow_inverse(gsvdec_t* h, const float* z_p, const float* g, const int32_t* lengths,
                        int B, int T0, float* z, int mem_kind, void* stream);

/* The flow inverse and then the decoder on its output with the same g and
 * lengths -- the sequence at src/models/sovits.rs:389-400 -- in one call:
 * z_p [B, C, T0] -> wav [B, hop * T0]. */
int gsvdec_flow_decode(gsvdec_t* h, const float* z_p, const float* g, const int32_t* lengths,
                       int B, int T0, float* wav, int mem_kind, void* stream);

/* ---- EncP fused elementwise chains (optional) ----------------------------
 * Present when the tensors include enc_p.* encoder layers: per layer i of a
 * stack, "<stack>.ffn_layers.<i>.conv_{1,2}.{weight,bias}" and
 * "<stack>.norm_layers_{1,2}.<i>.{gamma,beta}" (EncoderLayer::load,
 * src/models/sovits_encp.rs:54-96; FeedForward::load :348-369), and
 * "enc_p.proj.{weight,bias}" (:752-771).  Stacks: */
#define GSV_ENCP_SSL 0  /* enc_p.encoder_ssl  */
#define GSV_ENCP_TEXT 1 /* enc_p.encoder_text */
#define GSV_ENCP_2 2    /* enc_p.encoder2     */

/* Layers per stack (n_layers[3], 0 when absent), hidden channels, FFN filter
 * channels and projection outputs (2 * out_channels; 0 without enc_p.proj). */
int gsvdec_encp_info(const gsvdec_t* h, int n_layers[3], int* channels, int* filter_channels,
                     int* proj_channels);

/* out = norm_layers_<norm>[layer](x + y) (norm = 1 or 2): the post-norm
 * residual of EncoderLayer::forward (src/models/sovits_encp.rs:102, :107)
 * with LayerNorm::forward over the channel axis (src/utils/weights.rs:461-502:
 * mean, biased variance, (v - mean) / sqrt(var + 1e-5) * gamma + beta).
 * x, y, out [B, C, T] fp32; y may be NULL (LayerNorm of x alone); with
 * lengths, frames t >= lengths[b] are multiplied by 0 (the x_mask product,
 * :109). */
int gsvdec_encp_add_norm(gsvdec_t* h, int stack, int layer, int norm, const float* x, const float* y,
                         const int32_t* lengths, int B, int T, float* out, int mem_kind, void* stream);

/* The FFN half of EncoderLayer::forward (src/models/sovits_encp.rs:104-109):
 * out = norm_layers_2[layer](x + conv_2(relu(conv_1(x)))) * x_mask, convs
 * with pad (k-1)/2 (FeedForward::forward :371-375, load_conv1d :378-410).
 * ReLU runs in conv_1's epilogue, the residual in conv_2's, LayerNorm + mask
 * + relayout in one pass.  x, out [B, C, T] fp32; lengths [B] or NULL. */
int gsvdec_encp_ffn(gsvdec_t* h, int stack, int layer, const float* x, const int32_t* lengths, int B,
                    int T, float* out, int mem_kind, void* stream);

/* EncoderLayer::forward after the attention (src/models/sovits_encp.rs:98-110):
 * out = norm_layers_2(h + FFN(h)) * x_mask with h = norm_layers_1(x + attn),
 * attn [B, C, T] the self-attention output (NULL: h = norm_layers_1(x)).
 * norm1 is written straight into the FFN's time-major GEMM operand, so the
 * layer is four launches: norm1, conv_1 + ReLU, conv_2 + residual, norm2 +
 * mask + relayout. */
int gsvdec_encp_layer(gsvdec_t* h, int stack, int layer, const float* x, const float* attn,
                      const int32_t* lengths, int B, int T, float* out, int mem_kind, void* stream);

/* Output length of the speed change (src/models/sovits_encp.rs:857-867):
 * T when |speed - 1| <= FLT_EPSILON, else max(1, trunc(T / speed) + 1).
 * GSV_E_INVALID_ARG for a non-finite or non-positive speed. */
int gsvdec_encp_speed_len(int T, float speed, int* T_out);

/* linear_interpolate_last_dim (src/models/sovits_encp.rs:10-40): y [B, C, T]
 * -> out [B, C, T_out] fp32, half-pixel sampling, bit-identical to the
 * reference's f32 evaluation.  T_out == T copies. */
int gsvdec_encp_interpolate(gsvdec_t* h, const float* y, int B, int C, int T, int T_out, float* out,
                            int mem_kind, void* stream);

/* EncP output projection and prior sample: stats = proj(y) * y_mask;
 * m = stats[:, :Co]; logs = clamp(stats[:, Co:], -5, 2)
 * (src/models/sovits_encp.rs:871-879); z_p = m + noise * exp(logs) *
 * noise_scale (src/models/sovits.rs:378-385, the noise drawn by the caller).
 * y [B, C, T]; noise, m, logs, z_p [B, Co, T] fp32; lengths [B] or NULL.
 * m, logs and z_p may each be NULL (not written); z_p needs noise. */
int gsvdec_encp_project(gsvdec_t* h, const float* y, const int32_t* lengths, int B, int T,
                        const float* noise, float noise_scale, float* m, float* logs, float* z_p,
                        int mem_kind, void* stream);

/* One conv layer of the Generator, named by its dec.* prefix ("dec.conv_pre",
 * "dec.ups.3", "dec.resblocks.7.convs1.2", "dec.conv_post", ...; see
 * gsvdec_layer_names), on x [B, Cin, L] -> y [B, Cout, Lout] in the
 * reference's layout (fp32; host or device per mem_kind), through the same
 * kernel and packed weights the forward uses: the bias is added, no
 * activation is applied (conv_post: the value before tanh).  In BF16 mode x
 * is rounded to bf16 first, as activations are inside the forward.  This is
 * the per-layer tap of the reference's Conv1d/Conv1dWeightNorm::forward
 * (src/utils/weights.rs:533-550, 646-658) and ConvTranspose upsample
 * (src/models/sovits_decoder.rs:551-576), for per-layer parity and sweeps. */
int gsvdec_layer_forward(gsvdec_t* h, const char* layer, const float* x, int B, int L, float* y,
                         int mem_kind, void* stream);

/* Newline-separated layer names of the handle, in forward order (conv_pre,
 * then per stage the upsample and its resblock convs, then conv_post).
 * Writes at most cap bytes including the terminating NUL; *needed gets the
 * full size. */
int gsvdec_layer_names(const gsvdec_t* h, char* buf, size_t cap, size_t* needed);

/* Stage timers, the counterpart of the reference's "profile decoder
 * pre/upsample/resblocks/post" line (src/models/sovits_decoder.rs:459-468):
 * with enable = 1 the following forwards record CUDA events between stages,
 * with enable = 2 also one event after every kernel launch (see
 * gsvdec_get_launch_stats); 0 switches it off.  No host sync is added inside
 * the launch sequence; the times are read back when the forward returns.
 * ms[0] pre, ms[1] upsample (sum), ms[2] resblocks (sum), ms[3] post,
 * ms[4] total. */
int gsvdec_set_stage_timing(gsvdec_t* h, int enable);
int gsvdec_get_stage_times(gsvdec_t* h, float ms[5]);

/* Number of kernels the most recent forward on this handle launched
 * (B and T0 are accepted for future shape queries and ignored today). */
int gsvdec_launch_count(gsvdec_t* h, int B, int T0, int* count);

/* Per-launch profile, recorded when stage timing is enabled with level 2
 * (gsvdec_set_stage_timing(h, 2)): one CUDA-event interval per kernel launch
 * on the forward's stream.  Forwards accumulate without any host sync until
 * this call, which waits for them and returns each launch's duration
 * averaged over the accumulated forwards (those with the same launch
 * sequence as the most recent one), then starts a new accumulation.  flops and bytes are
 * the ALGORITHMIC work of the reference layers the launch computes
 * (F = 2 Cin Cout k L_in B per conv, ConvTranspose counted on input
 * samples; bytes = e B (Cin L_in + Cout L_out) + e Cin Cout k per conv plus
 * e B Cout L_out per residual read, e = activation element size), so that
 * the layer roofline max(F / peak, bytes / bandwidth) can be formed.
 * No reference counterpart beyond its stage timer line. */
typedef struct gsvdec_launch_stat {
  char name[48];   /* e.g. "conv_pre", "ups2", "rb3.step1.conv1", "rb3.final" */
  int kind;        /* 0 tap-GEMM conv, 1 relayout / cond / lengths, 2 conv_post */
  int n_convs;     /* reference conv layers inside this launch */
  double flops;    /* sums over the launch's convs */
  double bytes;
  double conv_flops[6]; /* per conv (first n_convs entries; layer rooflines are per conv) */
  double conv_bytes[6];
  float ms;
} gsvdec_launch_stat;
int gsvdec_get_launch_stats(gsvdec_t* h, gsvdec_launch_stat* out, int max, int* n);

/* Allocation-free forward.  No counterpart in the reference crate.
 *
 * For callers that cannot allocate device memory when they decode -- a
 * real-time audio callback, or a server whose device memory is owned by its
 * own pool allocator, where a cudaMalloc would block, fragment the pool or
 * fail.  Same result as gsvdec_forward with GSV_MEM_DEVICE pointers
 * (z, g, lengths and wav are device pointers on the handle's device; the
 * call is stream-async), but the per-call scratch between layers lives in a
 * static device array of gsvdec_noalloc_scratch_bytes() bytes (32 MiB) that
 * every GPU loading this library holds until process exit; this call never
 * calls cudaMalloc / cudaFree.  Requests whose buffers do not fit (about
 * 130 frames of B*T0 in BF16 mode, 65 in FP32 mode, 45 in FP32_TC mode) are rejected with
 * GSV_E_INVALID_ARG and a message giving the bytes needed.
 * The first call on a device looks up the array's device address (once per
 * device, with that device made current); make that first call before any
 * stream capture.  Every call on a device shares the one array and leaves its
 * contents behind; nothing in it needs clearing, since each layer overwrites
 * all of its output, but calls that overlap on the GPU (two streams, two
 * handles on one device, two threads) race on the array and must be
 * serialised by the caller. */
int gsvdec_forward_noalloc(gsvdec_t* h, const float* z, const float* g, const int32_t* lengths,
                           int B, int T0, float* wav, void* stream);
int64_t gsvdec_noalloc_scratch_bytes(void);

/* ---- Several devices ------------------------------------------------------
 * Decoder::forward over several GPUs in one call: handles[i] is a handle
 * created on device i of the job (the same checkpoint and mode on each; two
 * handles on one device are allowed and run as two workers).  z, g, lengths
 * and wav are as in gsvdec_forward; with GSV_MEM_DEVICE they live on
 * handles[0]'s device and `stream` is a stream of that device.
 *   B > 1 (or one handle): utterances are split over the handles
 *     (longest-processing-time balance of the frame counts), each handle
 *     decoding its share in up to 8 length-bucketed masked batches
 *     (gsvdec_plan_multi shows the plan);
 *   B == 1: the utterance is split into contiguous frame ranges, one per
 *     handle, each decoded with 16 input frames recomputed on both sides.
 * Either way every utterance's samples equal those of gsvdec_forward on it
 * alone (with its own length), and samples past hop*lengths[b] are 0.
 * Each handle works on its own stream from its own host thread; inputs reach
 * a device, and waveform pieces reach handles[0]'s device (or the host), by
 * copy-engine copies -- no kernel reads another device's memory.
 * GSV_MEM_HOST: the call returns when wav is complete.  GSV_MEM_DEVICE: the
 * work starts after the work already queued on `stream` and wav is complete
 * in `stream` order when the call returns (the call itself waits for
 * `stream` only when lengths are given, to plan with them on the host).  A
 * device wait that gives up in a stream-async call is reported by
 * gsvdec_sync_status or the next call on the handle concerned.
 * Calls on one handle must not overlap, as for every other call.  No
 * reference counterpart: the reference decodes on one device
 * (src/config/mod.rs:68-80; SoVITSModel::synthesize_with_speed_and_sv,
 * src/models/sovits.rs:400, calls Decoder::forward once per utterance). */
int gsvdec_forward_multi(gsvdec_t* const* handles, int n_handles, const float* z, const float* g,
                         const int32_t* lengths, int B, int T0, float* wav, int mem_kind, void* stream);

/* The utterance plan gsvdec_forward_multi uses for B > 1 on n_workers
 * handles: worker[b] and bucket[b] (index of utterance b's batch on its
 * worker, batches by increasing length) for every utterance, -1 for an
 * empty one (lengths[b] == 0).  lengths may be NULL (all T0).  Host only. */
int gsvdec_plan_multi(const int32_t* lengths, int B, int T0, int n_workers, int32_t* worker,
                      int32_t* bucket);

/* ---- Status of stream-async calls and failure hooks -----------------------
 * Calls with GSV_MEM_DEVICE pointers (and gsvdec_forward_noalloc) return once
 * their kernels are queued.  A bounded device wait that gives up inside them
 * (after about 2 s without progress) stops its kernel and sets the handle's
 * error word.  It is reported as GSV_E_TIMEOUT by the first of:
 *   - gsvdec_sync_status(h, stream), which waits for `stream` and then
 *     reads and clears the word;
 *   - the next host-memory call on the handle (it syncs its stream);
 *   - the entry of any later call on the handle, once the kernel has ended:
 *     that call then returns GSV_E_TIMEOUT without doing anything else (the
 *     word is cleared, so the call after it proceeds).
 * No reference counterpart beyond its Result propagation (src/lib.rs:76-97). */
int gsvdec_sync_status(gsvdec_t* h, void* stream);

/* Self-test of the give-up path: queues on `stream` one kernel that runs the
 * library's bounded device wait on a barrier nothing completes, limited to
 * limit_ns (1e3..1e10).  The wait runs out and reports through the handle's
 * error word like any decode kernel: gsvdec_sync_status then returns
 * GSV_E_TIMEOUT and the handle keeps working.  Nothing else is in flight in
 * that kernel when it gives up.  No reference counterpart. */
int gsvdec_selftest_wait(gsvdec_t* h, int64_t limit_ns, void* stream);

/* Allocation-failure hook (process-wide, for tests of the callers' error
 * paths): with n >= 0 the next n device allocations of the library succeed
 * and every one after them fails with GSV_E_OOM, until the hook is reset
 * with n < 0 (the default).  A call that fails this way leaves its handle
 * usable.  No reference counterpart. */
int gsvdec_set_alloc_fail_after(int n);

/* Device bytes the handle holds for per-call workspaces (decoder, single
 * layer, flow, EncP), i.e. everything but its packed weights. */
int gsvdec_workspace_bytes(const gsvdec_t* h, int64_t* bytes);

/* Thread-local message describing the last error on this thread. */
const char* gsvdec_last_error(void);

#ifdef __cplusplus
}
#endif
#endif /* GSVDEC_H */
