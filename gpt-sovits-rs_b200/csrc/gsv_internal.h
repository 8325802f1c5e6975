// gsv_internal.h -- descriptors shared by the host planner and the kernels.
//
// Every convolution of the Generator is expressed as one "tap GEMM":
//
//   acc[b, q, n] = sum_seg sum_j sum_c  X_seg[b, q + off_seg(j), c] * W_seg[j, n, c]
//
// over activations stored time-major ([B][L][C], channels innermost, so a
// tap shift is a whole-row shift).  Rows outside [0, Lin) read as zero, which
// is the zero padding of Conv1d (src/utils/weights.rs:78-113).
//
// * Conv1d(k, dil, pad):  off(j) = j*dil - pad, N = Cout, output row = q.
// * ConvTranspose1d(k, s, pad) (src/models/sovits_decoder.rs:551-576) is
//   written polyphase: output t = q*s + phi - pad takes the taps
//   kk = phi + m*s, reading x[q - m].  With columns n = phi*Cout + cout the
//   GEMM output [Q][s*Cout] is the [Lout][Cout] output shifted by pad rows,
//   so no zero-stuffed input is ever formed: off(m) = -m, N = s*Cout,
//   crop = pad*Cout elements.
//
// The epilogue maps element (q, n) to the flat output index
// e = q*N + n - crop (dropped unless 0 <= e < Lout*Cout), t = e / Cout,
// c = e % Cout, and computes
//   v = (acc + bias[c] + bias_bc[b, c] + sum_r res_r[b, t, c]) / div
// zeroing rows t >= len[b]; it stores v (out_raw) and/or leaky_relu(v, slope)
// (out_act).  That folds the bias add, the broadcast cond add
// (src/models/sovits_decoder.rs:393-399), the ResBlock residual add (:204),
// the three-branch average (:418-442) and the LeakyReLU that starts the next
// layer (:200, :202, :408, :449) into the producing kernel.
#pragma once
#include <cstdint>

namespace gsv {

constexpr int kMaxSeg = 6;  // up to 3 convs + 3 identity (residual) segments
constexpr int kMaxRes = 3;
constexpr int kMaxGroup = 3;

struct TapSeg {
  const void* x;  // [B][Lin][Cin], mode dtype
  const void* w;  // packed weights of this segment (layout depends on the kernel family)
  int Lin;        // input rows per utterance
  int Cin;
  int ntaps;
  int off0;       // row offset of tap 0
  int offstep;    // row offset step between taps
  // Three-piece operands (bf16 tcgen05 only): when pc > 0, x holds [B][Lin][3 pc]
  // (three bf16 pieces X0, X1, X2 of each fp32 value, channel planes of width
  // pc) and the segment's Cin channels are a K list of pc-wide blocks over
  // those planes: Cin = 5 pc reads planes [X2 X1 X0 X1 X0] (against weight
  // pieces [W0 W1 W2 W0 W1]: the five small products), Cin = pc reads X0
  // (against W0: the large one), Cin = 3 pc reads [X2 X1 X0] (against
  // identities: a residual).
  int pc;
};

struct TapConv {
  TapSeg seg[kMaxSeg];
  int nseg;
  int B, Q, N, Cout, Lout, crop;
  const float* bias;     // [Cout] (sum over segments), never null
  const float* bias_bc;  // [B][Cout] per-utterance bias (cond), or null
  const void* res[kMaxRes];
  int nres;
  float div;             // divisor applied after the sums (1 = none)
  void* out_raw;         // [B][Lout][Cout] or null
  void* out_act;         // [B][Lout][Cout] or null
  float slope;           // LeakyReLU slope of out_act
  const int* len;        // [B] valid output rows, or null
  int row_tiles;         // tiles per utterance along q (set by the launcher)
  int bias_bc_ld;        // row stride of bias_bc (0: Cout)
  // Three-piece outputs (bf16 tcgen05 only): out_raw / out_act (and the
  // residuals read) hold [B][Lout][3 Cout], each value as its three bf16 pieces.
  int split;
  // Gated-activation epilogue (bf16 tcgen05 only): the N = 2H GEMM columns are
  // interleaved in 16-column (a, b) pairs and the op writes
  // out_raw[b][q][H] = tanh(a + bias + bias_bc) * sigmoid(b + bias + bias_bc).
  int gate;
};

struct TapConvGroup {
  TapConv op[kMaxGroup];
  int n;
  int* err;  // device error word set by a kernel whose bounded wait gave up (or null)
  // FP32 CUDA-core kernel only: scratch for partial sums when a small launch
  // is split over its input-channel chunks (null: never split).
  float* partial;
  long long partial_cap;  // floats available at `partial`
};

// Ceil-div helper usable on host and device.
__host__ __device__ inline int cdiv(int a, int b) { return (a + b - 1) / b; }

}  // namespace gsv
