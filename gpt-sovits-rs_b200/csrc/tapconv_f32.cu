// tapconv_f32.cu -- fp32 CUDA-core tap GEMM (the FP32 mode of every conv).
//
// Implements Conv1d (src/utils/weights.rs:78-113) and polyphase
// ConvTranspose1d (src/models/sovits_decoder.rs:88-98, 551-576) in the
// reference's own F32 arithmetic (src/config/mod.rs:52-58), each output an
// fp32 dot product accumulated in the fixed order (segment, Cin chunk, tap,
// channel).  One CTA computes a TQ x TN tile of the GEMM for one utterance:
// the haloed input window [TQ + span rows x 16 channels] is staged once per
// channel chunk in shared memory and reused by every tap (a tap is a row
// shift inside the window), each thread accumulating a 4x4 register tile.
#include <cuda_runtime.h>

#include "gsv_epilogue.cuh"
#include "gsv_kernels.h"
#include "gsv_pdl.cuh"

namespace gsv {

namespace {

constexpr int kThreads = 256;
constexpr int kCK = 16;       // input channels per shared-memory chunk
constexpr int kMaxSpan = 64;  // largest (ntaps - 1) * |offstep| supported

template <int TN>
struct Cfg {
  static constexpr int TX = TN / 4;        // threads along n
  static constexpr int TY = kThreads / TX; // threads along q
  static constexpr int TQ = TY * 4;        // rows per tile
  static constexpr int W = TQ + kMaxSpan + 1;
};

template <int TN>
__global__ void __launch_bounds__(kThreads) tapconv_f32_kernel(const __grid_constant__ TapConvGroup grp) {
  pdl_wait();
  using C = Cfg<TN>;
  const TapConv& op = grp.op[blockIdx.z];
  const int b = blockIdx.x / op.row_tiles;
  if (b >= op.B) return;
  const int q0 = (blockIdx.x % op.row_tiles) * C::TQ;
  const int n0 = blockIdx.y * TN;
  if (n0 >= op.N) return;

  __shared__ float xs[kCK][C::W];
  __shared__ __align__(16) float ws[kCK][TN];

  const int tid = threadIdx.x;
  const int tx = tid % C::TX, ty = tid / C::TX;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;

  const bool masked = op.len != nullptr && first_out_row(op, q0) >= op.len[b];
  if (!masked) {
    for (int s = 0; s < op.nseg; ++s) {
      const TapSeg& sg = op.seg[s];
      const float* x = static_cast<const float*>(sg.x) + (size_t)b * sg.Lin * sg.Cin;
      const float* w = static_cast<const float*>(sg.w);
      const int last = sg.off0 + (sg.ntaps - 1) * sg.offstep;
      const int minoff = sg.offstep >= 0 ? sg.off0 : last;
      const int rows = C::TQ + (sg.ntaps - 1) * abs(sg.offstep);
      for (int c0 = 0; c0 < sg.Cin; c0 += kCK) {
        __syncthreads();
        for (int idx = tid; idx < rows * kCK; idx += kThreads) {
          const int r = idx / kCK, c = idx % kCK;
          const int gr = q0 + minoff + r;
          float v = 0.0f;
          if (gr >= 0 && gr < sg.Lin && c0 + c < sg.Cin) v = x[(size_t)gr * sg.Cin + c0 + c];
          xs[c][r] = v;
        }
        for (int j = 0; j < sg.ntaps; ++j) {
          __syncthreads();
          for (int idx = tid; idx < kCK * TN; idx += kThreads) {
            const int c = idx / TN, n = idx % TN;
            float v = 0.0f;
            if (c0 + c < sg.Cin && n0 + n < op.N)
              v = w[((size_t)j * sg.Cin + c0 + c) * op.N + n0 + n];
            ws[c][n] = v;
          }
          __syncthreads();
          const int d = sg.off0 + j * sg.offstep - minoff + ty * 4;
#pragma unroll
          for (int c = 0; c < kCK; ++c) {
            const float4 wv = *reinterpret_cast<const float4*>(&ws[c][tx * 4]);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float xv = xs[c][d + i];
              acc[i][0] = fmaf(xv, wv.x, acc[i][0]);
              acc[i][1] = fmaf(xv, wv.y, acc[i][1]);
              acc[i][2] = fmaf(xv, wv.z, acc[i][2]);
              acc[i][3] = fmaf(xv, wv.w, acc[i][3]);
            }
          }
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int q = q0 + ty * 4 + i;
    if (q >= op.Q) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx * 4 + j;
      if (n < op.N) epi_element<float>(op, b, q, n, acc[i][j]);
    }
  }
}

template <int TN>
cudaError_t launch_tn(TapConvGroup g, cudaStream_t st) {
  int gx = 0, gy = 0;
  for (int i = 0; i < g.n; ++i) {
    TapConv& op = g.op[i];
    for (int s = 0; s < op.nseg; ++s)
      if ((op.seg[s].ntaps - 1) * abs(op.seg[s].offstep) > kMaxSpan) return cudaErrorInvalidValue;
    op.row_tiles = cdiv(op.Q, Cfg<TN>::TQ);
    gx = max(gx, op.B * op.row_tiles);
    gy = max(gy, cdiv(op.N, TN));
  }
  if (gx == 0 || gy == 0) return cudaSuccess;
  {
    const cudaError_t e_ = launch_k(tapconv_f32_kernel<TN>, dim3(gx, gy, g.n), kThreads, 0, st, g);
    if (e_ != cudaSuccess) return e_;
  }
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_tapconv_f32(const TapConvGroup& g, cudaStream_t st) {
  for (int i = 0; i < g.n; ++i)
    if (g.op[i].gate || (g.op[i].bias_bc_ld && g.op[i].bias_bc_ld != g.op[i].Cout)) return cudaErrorNotSupported;
  int nmax = 0;
  for (int i = 0; i < g.n; ++i) nmax = max(nmax, g.op[i].N);
  if (nmax <= 16) return launch_tn<16>(g, st);
  if (nmax <= 32) return launch_tn<32>(g, st);
  return launch_tn<64>(g, st);
}

}  // namespace gsv
