// gsv_kernels.h -- launchers of the device kernels (host-callable).
#pragma once
#include <cuda_runtime.h>

#include "gsv_internal.h"

namespace gsv {

// Element type of activations / packed weights in one arithmetic mode.  X3:
// an fp32 value held as the exact sum of three bf16 pieces, stored as three
// channel planes per row ([B][L][3][C], piece 0 the bf16 rounding of the
// value, piece 1 that of the remainder, piece 2 the rest); the decoder
// activations of GSV_MODE_FP32_TC.
enum class Dt { F32 = 0, BF16 = 1, X3 = 2 };

// fp32 CUDA-core tap GEMM (weights packed [tap][Cin][N] fp32).
cudaError_t launch_tapconv_f32(const TapConvGroup& g, cudaStream_t st);
// bf16 tcgen05 tap GEMM (weights packed [tap][N][Cin] bf16).
cudaError_t launch_tapconv_tc(const TapConvGroup& g, cudaStream_t st);
// True when the tcgen05 kernel supports this op's geometry.
bool tapconv_tc_supported(const TapConv& op);

// One fused ResBlock1 step (conv1 -> lrelu -> conv2 -> +x) per op, bf16
// tcgen05, for C in {16, 32} (rbstep_tc.cu).  Weights packed like the tap
// GEMM ([tap][C][C] bf16), identity [C][C] bf16.
struct RbStepOp {
  const void* x;      // [B][L][C] raw input
  const void* w1;     // conv1 (dilation d)
  const void* w2;     // conv2 (dilation 1)
  const float* b1;
  const float* b2;
  void* out_raw;      // [B][L][C]
  void* out_act;      // [B][L][C] lrelu(out), or null
  int k, d;
};
struct RbStepGroup {
  RbStepOp op[kMaxGroup];
  int n;
  int C, B, L;
  const int* len;     // [B] valid rows, or null
  float slope;        // LeakyReLU slope inside the step (0.1)
  const void* identity;
  int* err;
};
bool rbstep_supported(int C, int k, int d);
cudaError_t launch_rbstep(const RbStepGroup& g, cudaStream_t st);

// One CTA whose bounded hand-off wait runs out after limit_ns and sets *err
// (selftest.cu; gsvdec_selftest_wait).
cudaError_t launch_wait_selftest(int* err, unsigned long long limit_ns, cudaStream_t st);

// z [B][Cin][Tsrc] fp32 (NCL, the reference layout) -> zt [B][T][Cin] (time-major)
// reading frames [t_off, t_off + T); frames t >= len[b] are written as 0.
cudaError_t launch_transpose_in(const float* z, int B, int Cin, int Tsrc, int t_off, int T,
                                const int* len, void* zt, Dt dt, cudaStream_t st);
// bias_bc[b][c] = sum_i wc[c][i] g[b][i] + bc[c]   (the cond 1x1 conv)
cudaError_t launch_cond(const float* g, const float* wc, const float* bc, int B, int gin, int C,
                        float* bias_bc, cudaStream_t st);
// Per-stage valid lengths: lens[s*B + b] for s in [0, nstage], stage 0 = frames.
cudaError_t launch_lengths(const int* len_in, int B, int T0, const int* mul, const int* add,
                           int nstage, int* lens, cudaStream_t st);
// wav [B][hop * T0]: samples past hop * len[b] of each utterance set to 0
// (len device-resident, clamped to [0, T0]).
cudaError_t launch_zero_tails(float* wav, const int* len, int B, int T0, int hop, cudaStream_t st);
// conv_post weights [K][16] by value (K <= 16), for the kernel-parameter path.
struct PostWeights {
  float w[16 * 16];
};
// conv_post (Cout 1, K taps, pad) + optional bias + tanh over x [B][L][C]:
// wav[b][t] = tanh(sum_{j,c} w[j][c] x[b][t + j - pad][c] + bias); rows t >= len[b]
// give 0.  With pre_tanh != null the pre-tanh value is stored there too.  `w` is
// the device copy; `wh` (or null) the same weights by value for the fast path.
cudaError_t launch_post(const void* x, Dt dt, int B, int L, int C, const float* w, const PostWeights* wh,
                        int K, int pad, float bias, const int* len, float* wav, float* pre_tanh,
                        cudaStream_t st);
// Time-major [B][L][C] (mode dtype) -> [B][C][L] fp32, the reference's layout
// (taps, flow output).  With perm (device, C ints) output channel c reads
// input channel perm[c].
cudaError_t launch_to_ncl(const void* x, Dt dt, int B, int L, int C, float* y, cudaStream_t st,
                          const int* perm = nullptr);
// WN gated activation (src/models/sovits_flow.rs:171-184):
// out[b][t][c] = tanh(xin[b][t][c] + g[c]) * sigmoid(xin[b][t][H + c] + g[H + c]),
// g = cond[b][off ..] (or 0 without cond); rows t >= len[b] give 0.
// xin [B][L][2H], out [B][L][H] in the mode dtype; H % 8 == 0.
cudaError_t launch_gate(const void* xin, const float* cond, int cond_ld, int cond_off, int B, int L,
                        int H, const int* len, void* out, Dt dt, cudaStream_t st);

// EncP elementwise chains (encp_kernels.cu).
// out = LayerNorm_C(x + y) * mask over [B][C][T] fp32 (y or len may be null):
// mean and biased variance over channels, (v - mean) / sqrt(var + eps) *
// gamma + beta; frames t >= len[b] are multiplied by 0.
cudaError_t launch_add_layernorm_ncl(const float* x, const float* y, const float* gamma, const float* beta,
                                     int B, int C, int T, float eps, const int* len, float* out,
                                     cudaStream_t st);
// The same, written time-major [B][T][C] in the mode dtype (a GEMM operand).
cudaError_t launch_add_layernorm_ncl_tm(const float* x, const float* y, const float* gamma, const float* beta,
                                        int B, int C, int T, float eps, const int* len, void* out, Dt dt,
                                        cudaStream_t st);
// The same LayerNorm (+ mask) of a time-major [B][T][C] tensor in the mode
// dtype, written as [B][C][T] fp32.
cudaError_t launch_layernorm_tm_ncl(const void* v, Dt dt, int B, int T, int C, const float* gamma,
                                    const float* beta, float eps, const int* len, float* out, cudaStream_t st);
// Half-pixel linear interpolation of each of `rows` rows from T to Tout
// samples, bit-identical to the reference's f32 evaluation.
cudaError_t launch_interpolate(const float* x, long long rows, int T, int Tout, float* out, cudaStream_t st);
// stats [B][T][2 Co] time-major (mode dtype) -> m = stats[:Co] * mask,
// logs = clamp(stats[Co:] * mask, -5, 2), zp = m + noise * exp(logs) *
// noise_scale, all [B][Co][T] fp32; any output may be null (zp needs noise).
cudaError_t launch_prior_sample(const void* stats, Dt dt, int B, int T, int Co, const int* len,
                                const float* noise, float noise_scale, float* m, float* logs, float* zp,
                                cudaStream_t st);

}  // namespace gsv
