// tapconv_f32.cu -- fp32 CUDA-core tap GEMM (the FP32 mode of every conv).
//
// Implements Conv1d (src/utils/weights.rs:78-113) and polyphase
// ConvTranspose1d (src/models/sovits_decoder.rs:88-98, 551-576) in the
// reference's own F32 arithmetic (src/config/mod.rs:52-58), each output an
// fp32 dot product accumulated in the fixed order (segment, Cin chunk, tap,
// channel).  One CTA computes a TQ x TN tile of the GEMM for one utterance:
// the haloed input window [TQ + span rows x 16 channels] and the chunk's
// weights for every tap are staged once per channel chunk in shared memory;
// every tap reads the window as a row shift, each thread accumulating an
// RQ x RN register tile.
#include <cuda_runtime.h>

#include <algorithm>

#include "gsv_epilogue.cuh"
#include "gsv_kernels.h"
#include "gsv_pdl.cuh"

namespace gsv {

namespace {

constexpr int kThreads = 256;
constexpr int kCK = 16;       // input channels per shared-memory chunk
constexpr int kMaxSpan = 64;  // largest (ntaps - 1) * |offstep| supported
constexpr int kMaxSplit = 8;  // largest split of one launch's K loop
constexpr int kF32SmsHint = 148, kF32CtasPerSm = 3;  // a wave of this kernel on a B200

// A CTA computes TQ x TN outputs; each thread an RQ x RN register tile (RQ
// consecutive rows, RN consecutive columns).  Four columns per thread keep the
// epilogue's per-element stores and residual loads 16-byte apart across a
// warp (eight measured slower); eight rows per thread at 32/64 columns give
// each thread more independent FMAs per weight load (fp32 forward 279 -> 271 ms
// on B200 against four rows with per-tap weight staging).
template <int TN>
struct Cfg {
  static constexpr int RN = 4;
  static constexpr int RQ = TN >= 32 ? 8 : 4;
  static constexpr int TX = TN / RN;        // threads along n
  static constexpr int TY = kThreads / TX;  // threads along q
  static constexpr int TQ = TY * RQ;        // rows per tile
  static constexpr int W = TQ + kMaxSpan + 1;
};

// Dynamic shared memory: the window [kCK][W] and every tap's weights of one
// channel chunk [ntaps][kCK][TN].
template <int TN>
size_t f32_smem(int max_taps) {
  return sizeof(float) * ((size_t)kCK * Cfg<TN>::W + (size_t)max_taps * kCK * TN);
}

// Input-channel chunks of an op over all its segments (the K loop of one tile).
__host__ __device__ inline int k_chunks(const TapConv& op) {
  int nc = 0;
  for (int s = 0; s < op.nseg; ++s) nc += cdiv(op.seg[s].Cin, kCK);
  return nc;
}

// blockIdx.z = op * nsplit + split.  With nsplit > 1 a CTA accumulates only
// the chunks [split * nc / nsplit, (split + 1) * nc / nsplit) of its tile and
// stores the raw partial sums to grp.partial ([split][op][B][Q][N], `elems`
// floats per (split, op)); f32_split_reduce adds the splits in order and runs
// the epilogue.
template <int TN>
__global__ void __launch_bounds__(kThreads) tapconv_f32_kernel(const __grid_constant__ TapConvGroup grp, int nsplit,
                                                               long long elems) {
  pdl_wait();
  using C = Cfg<TN>;
  constexpr int RQ = C::RQ, RN = C::RN;
  const int oi = blockIdx.z / nsplit, split = blockIdx.z - oi * nsplit;
  const TapConv& op = grp.op[oi];
  const int b = blockIdx.x / op.row_tiles;
  if (b >= op.B) return;
  const int q0 = (blockIdx.x % op.row_tiles) * C::TQ;
  const int n0 = blockIdx.y * TN;
  if (n0 >= op.N) return;
  extern __shared__ __align__(16) float f32_smem_raw[];
  float* xs = f32_smem_raw;               // [kCK][W]
  float* ws = f32_smem_raw + kCK * C::W;  // [tap][kCK][TN]
  const int tid = threadIdx.x;
  const int tx = tid % C::TX, ty = tid / C::TX;
  float acc[RQ][RN];
#pragma unroll
  for (int i = 0; i < RQ; ++i)
#pragma unroll
    for (int j = 0; j < RN; ++j) acc[i][j] = 0.0f;
  const bool masked = op.len != nullptr && first_out_row(op, q0) >= op.len[b];
  const int nc = k_chunks(op);
  const int c_lo = (int)((long long)split * nc / nsplit), c_hi = (int)((long long)(split + 1) * nc / nsplit);
  int ci = 0;  // running chunk index over (segment, chunk)
  if (!masked) {
    for (int s = 0; s < op.nseg; ++s) {
      const TapSeg& sg = op.seg[s];
      const float* x = static_cast<const float*>(sg.x) + (size_t)b * sg.Lin * sg.Cin;
      const float* w = static_cast<const float*>(sg.w);
      const int last = sg.off0 + (sg.ntaps - 1) * sg.offstep;
      const int minoff = sg.offstep >= 0 ? sg.off0 : last;
      const int rows = C::TQ + (sg.ntaps - 1) * abs(sg.offstep);
      for (int c0 = 0; c0 < sg.Cin; c0 += kCK, ++ci) {
        if (ci < c_lo || ci >= c_hi) continue;  // uniform over the CTA
        __syncthreads();
        for (int idx = tid; idx < rows * kCK; idx += kThreads) {
          const int r = idx / kCK, c = idx % kCK;
          const int gr = q0 + minoff + r;
          float v = 0.0f;
          if (gr >= 0 && gr < sg.Lin && c0 + c < sg.Cin) v = x[(size_t)gr * sg.Cin + c0 + c];
          xs[c * C::W + r] = v;
        }
        for (int idx = tid; idx < sg.ntaps * kCK * TN; idx += kThreads) {
          const int j = idx / (kCK * TN), c = (idx / TN) % kCK, n = idx % TN;
          float v = 0.0f;
          if (c0 + c < sg.Cin && n0 + n < op.N) v = w[((size_t)j * sg.Cin + c0 + c) * op.N + n0 + n];
          ws[idx] = v;
        }
        __syncthreads();
        // Per output: taps in order, channels in order within a tap.
        for (int j = 0; j < sg.ntaps; ++j) {
          const float* xr = xs + (sg.off0 + j * sg.offstep - minoff + ty * RQ);
          const float* wr = ws + (size_t)j * kCK * TN + tx * RN;
#pragma unroll
          for (int c = 0; c < kCK; ++c) {
            float wv[RN];
#pragma unroll
            for (int k = 0; k < RN; k += 4) {
              const float4 t = *reinterpret_cast<const float4*>(wr + c * TN + k);
              wv[k] = t.x;
              wv[k + 1] = t.y;
              wv[k + 2] = t.z;
              wv[k + 3] = t.w;
            }
#pragma unroll
            for (int i = 0; i < RQ; ++i) {
              const float xv = xr[c * C::W + i];
#pragma unroll
              for (int k = 0; k < RN; ++k) acc[i][k] = fmaf(xv, wv[k], acc[i][k]);
            }
          }
        }
      }
    }
  }
  if (nsplit > 1) {
    float* part = grp.partial + ((long long)split * grp.n + oi) * elems + (long long)b * op.Q * op.N;
#pragma unroll
    for (int i = 0; i < RQ; ++i) {
      const int q = q0 + ty * RQ + i;
      if (q >= op.Q) continue;
#pragma unroll
      for (int j = 0; j < RN; ++j) {
        const int n = n0 + tx * RN + j;
        if (n < op.N) part[(long long)q * op.N + n] = acc[i][j];
      }
    }
    return;
  }
#pragma unroll
  for (int i = 0; i < RQ; ++i) {
    const int q = q0 + ty * RQ + i;
    if (q >= op.Q) continue;
#pragma unroll
    for (int j = 0; j < RN; ++j) {
      const int n = n0 + tx * RN + j;
      if (n < op.N) epi_element<float>(op, b, q, n, acc[i][j]);
    }
  }
}

// Sum of the splits of GEMM element (op, b, q, n), in split order, then the
// fused epilogue.
__global__ void __launch_bounds__(256) f32_split_reduce(const __grid_constant__ TapConvGroup grp, int nsplit,
                                                        long long elems) {
  pdl_wait();
  const long long total = (long long)grp.n * elems;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int oi = (int)(i / elems);
    const long long r = i - (long long)oi * elems;
    const TapConv& op = grp.op[oi];
    const long long qn = (long long)op.Q * op.N;
    if (r >= (long long)op.B * qn) continue;
    const int b = (int)(r / qn);
    const int q = (int)((r - b * qn) / op.N);
    const int n = (int)(r - b * qn - (long long)q * op.N);
    float v = 0.0f;
    for (int sp = 0; sp < nsplit; ++sp) v += grp.partial[((long long)sp * grp.n + oi) * elems + r];
    epi_element<float>(op, b, q, n, v);
  }
}

template <int TN>
cudaError_t launch_tn(TapConvGroup g, cudaStream_t st) {
  int gx = 0, gy = 0, max_taps = 1;
  for (int i = 0; i < g.n; ++i) {
    TapConv& op = g.op[i];
    for (int s = 0; s < op.nseg; ++s) {
      if ((op.seg[s].ntaps - 1) * abs(op.seg[s].offstep) > kMaxSpan) return cudaErrorInvalidValue;
      max_taps = max(max_taps, op.seg[s].ntaps);
    }
    op.row_tiles = cdiv(op.Q, Cfg<TN>::TQ);
    gx = max(gx, op.B * op.row_tiles);
    gy = max(gy, cdiv(op.N, TN));
  }
  if (gx == 0 || gy == 0) return cudaSuccess;
  const size_t smem = f32_smem<TN>(max_taps);
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  if (smem > 48 * 1024) {
    const cudaError_t e = cudaFuncSetAttribute(tapconv_f32_kernel<TN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               (int)smem);
    if (e != cudaSuccess) return e;
  }
  // Small launches (short utterances, early stages) fill less than two waves
  // of CTAs and run long tiles on a partly idle GPU: split their K loop over
  // the input-channel chunks (partial sums, then an ordered reduction).
  int nsplit = 1;
  long long elems = 0;
  int min_nc = 1 << 30;
  for (int i = 0; i < g.n; ++i) {
    elems = std::max(elems, (long long)g.op[i].B * g.op[i].Q * g.op[i].N);
    min_nc = std::min(min_nc, k_chunks(g.op[i]));
  }
  const long long ctas = (long long)gx * gy * g.n, target = 2LL * kF32SmsHint * kF32CtasPerSm;
  if (g.partial && ctas < target && min_nc >= 2) {
    nsplit = (int)std::min<long long>({(target + ctas - 1) / ctas, (long long)kMaxSplit, (long long)min_nc});
    while (nsplit > 1 && (long long)nsplit * g.n * elems > g.partial_cap) --nsplit;
  }
  const cudaError_t e_ = launch_k(tapconv_f32_kernel<TN>, dim3(gx, gy, g.n * nsplit), kThreads, smem, st, g, nsplit,
                                  elems);
  if (e_ != cudaSuccess) return e_;
  if (nsplit > 1) {
    const long long total = (long long)g.n * elems;
    const int blocks = (int)std::min<long long>((total + 255) / 256, 148LL * 8);
    const cudaError_t e2 = launch_k(f32_split_reduce, blocks, 256, 0, st, g, nsplit, elems);
    if (e2 != cudaSuccess) return e2;
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
