// misc_kernels.cu -- the small memory-bound kernels around the conv stack:
// input relayout, the speaker-cond 1x1 conv, per-stage lengths, conv_post +
// tanh, and the time-major -> reference-layout copy used by the debug taps.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "gsv_epilogue.cuh"
#include "gsv_kernels.h"
#include "gsv_pdl.cuh"

namespace gsv {

namespace {

// 32x32 tiled transpose of z [B][Cin][Tsrc] (frames t_off..t_off+T) into
// [B][T][Cin]; frames past len[b] become 0 (the masked utterance end).
template <typename T>
__global__ void transpose_in_kernel(const float* __restrict__ z, int Cin, int Tsrc, int t_off,
                                    int Tn, const int* __restrict__ len, T* __restrict__ out) {
  pdl_wait();
  __shared__ float tile[32][33];
  const int b = blockIdx.z;
  const int t0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
  const int lim = len ? len[b] : Tn;
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int c = c0 + i, t = t0 + threadIdx.x;
    float v = 0.0f;
    if (c < Cin && t < Tn && t < lim) v = z[((size_t)b * Cin + c) * Tsrc + t_off + t];
    tile[i][threadIdx.x] = v;
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int t = t0 + i, c = c0 + threadIdx.x;
    if (t < Tn && c < Cin) st_act<T>(out, ((size_t)b * Tn + t) * Cin + c, tile[threadIdx.x][i]);
  }
}

// Three bf16 pieces of v at p[0], p[C], p[2C] (their sum is v exactly).
__device__ __forceinline__ void st_x3(__nv_bfloat16* p, int C, float v) {
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    const __nv_bfloat16 h = __float2bfloat16_rn(v);
    p[(size_t)k * C] = h;
    v = v - __bfloat162float(h);
  }
}

// The same relayout into three-piece rows [B][T][3 Cin] (GSV_MODE_FP32_TC).
__global__ void transpose_in_x3_kernel(const float* __restrict__ z, int Cin, int Tsrc, int t_off, int Tn,
                                       const int* __restrict__ len, __nv_bfloat16* __restrict__ out) {
  pdl_wait();
  __shared__ float tile[32][33];
  const int b = blockIdx.z;
  const int t0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
  const int lim = len ? len[b] : Tn;
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int c = c0 + i, t = t0 + threadIdx.x;
    float v = 0.0f;
    if (c < Cin && t < Tn && t < lim) v = z[((size_t)b * Cin + c) * Tsrc + t_off + t];
    tile[i][threadIdx.x] = v;
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int t = t0 + i, c = c0 + threadIdx.x;
    if (t < Tn && c < Cin) st_x3(out + ((size_t)b * Tn + t) * 3 * Cin + c, Cin, tile[threadIdx.x][i]);
  }
}

// One warp per output channel: bias_bc[b][c] = bc[c] + sum_i wc[c][i] g[b][i].
__global__ void cond_kernel(const float* __restrict__ g, const float* __restrict__ wc,
                            const float* __restrict__ bc, int B, int gin, int C,
                            float* __restrict__ out) {
  pdl_wait();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (warp >= B * C) return;
  const int b = warp / C, c = warp % C;
  float s = 0.0f;
  for (int i = lane; i < gin; i += 32) s = fmaf(wc[(size_t)c * gin + i], g[(size_t)b * gin + i], s);
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) out[(size_t)b * C + c] = s + (bc ? bc[c] : 0.0f);
}

// wav [B][row]: samples [hop * len[b], row) of utterance b set to 0 (the
// tails past each utterance's own length in a multi-device decode).
__global__ void zero_tails_kernel(float* __restrict__ wav, const int* __restrict__ len, long long row,
                                  int hop, int T0) {
  pdl_wait();
  const int b = blockIdx.y;
  int l = len[b];
  l = l < 0 ? 0 : (l > T0 ? T0 : l);
  float* w = wav + (size_t)b * row;
  for (long long i = (long long)l * hop + blockIdx.x * (long long)blockDim.x + threadIdx.x; i < row;
       i += (long long)gridDim.x * blockDim.x)
    w[i] = 0.0f;
}

struct StageLen {
  int mul[16];
  int add[16];
};

__global__ void lengths_kernel(const int* __restrict__ len_in, int B, int T0, StageLen sl,
                               int nstage, int* __restrict__ lens) {
  pdl_wait();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  int l = len_in ? len_in[b] : T0;
  l = l < 0 ? 0 : (l > T0 ? T0 : l);
  lens[b] = l;
  for (int s = 0; s < nstage; ++s) {
    l = l > 0 ? l * sl.mul[s] + sl.add[s] : 0;
    lens[(s + 1) * B + b] = l;
  }
}

// conv_post: Cout 1, K taps over C = 16 channels.  Each thread produces 4
// consecutive samples from the K + 3 input rows they span (rows shared with
// neighbouring threads come from L1); weights live in shared memory.
template <int C>
__device__ __forceinline__ void load_row(const float* p, float* v) {
#pragma unroll
  for (int k = 0; k < C / 4; ++k) {
    const float4 f = __ldg(reinterpret_cast<const float4*>(p) + k);
    v[4 * k] = f.x; v[4 * k + 1] = f.y; v[4 * k + 2] = f.z; v[4 * k + 3] = f.w;
  }
}
template <int C>
__device__ __forceinline__ void load_row(const __nv_bfloat16* p, float* v) {
#pragma unroll
  for (int k = 0; k < C / 8; ++k) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(p) + k);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h[i]);
      v[8 * k + 2 * i] = f.x;
      v[8 * k + 2 * i + 1] = f.y;
    }
  }
}

template <typename T, int C>
__global__ void __launch_bounds__(256) post_kernel(const T* __restrict__ x, int L,
                                                   const float* __restrict__ w, int K, int pad,
                                                   float bias, const int* __restrict__ len,
                                                   float* __restrict__ wav, float* __restrict__ pre) {
  pdl_wait();
  constexpr int kPer = 4;
  __shared__ float sw[64 * C];  // [K][C]
  for (int i = threadIdx.x; i < K * C; i += blockDim.x) sw[i] = w[i];
  __syncthreads();
  const int b = blockIdx.y;
  const int t0 = (blockIdx.x * blockDim.x + threadIdx.x) * kPer;
  if (t0 >= L) return;
  const T* xb = x + (size_t)b * L * C;
  float acc[kPer];
#pragma unroll
  for (int o = 0; o < kPer; ++o) acc[o] = bias;
  for (int r = 0; r < K + kPer - 1; ++r) {
    const int row = t0 - pad + r;
    if (row < 0 || row >= L) continue;
    float v[C];
    load_row<C>(xb + (size_t)row * C, v);
#pragma unroll
    for (int o = 0; o < kPer; ++o) {
      const int j = r - o;  // tap of output t0 + o that reads this row
      if (j < 0 || j >= K) continue;
      float s = 0.0f;
#pragma unroll
      for (int c = 0; c < C; ++c) s = fmaf(v[c], sw[j * C + c], s);
      acc[o] += s;
    }
  }
  const int lim = len ? len[b] : L;
#pragma unroll
  for (int o = 0; o < kPer; ++o) {
    const int t = t0 + o;
    if (t >= L) break;
    const bool dead = t >= lim;
    if (pre) pre[(size_t)b * L + t] = dead ? 0.0f : acc[o];
    wav[(size_t)b * L + t] = dead ? 0.0f : tanhf(acc[o]);
  }
}

// conv_post for a kernel size known at compile time: the K x 16 weights are a
// kernel parameter (the FMAs read them from the constant bank), a block stages
// its input rows in shared memory with coalesced 16-byte loads, and thread i
// computes samples t_base + i + 256 o (o < kPostPer), so a warp's row reads
// are contiguous (no bank conflicts) and its stores coalesce.  The staged rows
// take 33 KB of shared memory in either precision.
constexpr int kPostThreads = 256;
template <typename T>
constexpr int post_per() { return sizeof(T) == 2 ? 4 : 2; }

// conv_post with the weights as a kernel parameter, in two passes over a block
// of kPostOut samples: (1) every input row of the block's window is read once
// (16-byte loads, a warp reads 1 KB contiguous) and turned into its K per-tap
// partial dots d_j(r) = sum_c w[j][c] x[r][c], stored as sd[j][r]; (2) sample t
// sums d_j(t + j) over j, reading K consecutive floats per tap across the warp.
// Each row is fetched from HBM once and read from shared memory as 4 K bytes
// instead of K times 32; the sums run in the same order as a direct
// per-sample loop (over c within a tap, then over taps, from the bias).
// NP = 3: three-piece rows [L][3][16] bf16 (GSV_MODE_FP32_TC), each value the
// exact sum of its pieces.
template <typename T, int K, int NP = 1>
__global__ void __launch_bounds__(kPostThreads) post_fast_kernel(const T* __restrict__ x, int L,
                                                                 const __grid_constant__ PostWeights P,
                                                                 int pad, float bias,
                                                                 const int* __restrict__ len,
                                                                 float* __restrict__ wav,
                                                                 float* __restrict__ pre) {
  pdl_wait();
  constexpr int C = 16;
  constexpr int U = C * (int)sizeof(T) / 16;  // 16-byte units per input row
  constexpr int kPostPer = post_per<T>(), kPostOut = kPostThreads * kPostPer;
  constexpr int kRows = kPostOut + K - 1;
  __shared__ float sd[K][kRows];
  const int b = blockIdx.y;
  const int t_base = blockIdx.x * kPostOut;
  const int r0 = t_base - pad;
  const uint4* xb = reinterpret_cast<const uint4*>(x + (size_t)b * L * C * NP);
  for (int i = threadIdx.x; i < kRows; i += kPostThreads) {
    const int row = r0 + i;
    float v[C];
    if (NP == 3 && row >= 0 && row < L) {
#pragma unroll
      for (int c = 0; c < C; ++c) v[c] = 0.0f;
#pragma unroll
      for (int k = 0; k < 3 * U; ++k) {  // plane k / U, channels 8 (k % U) ..
        const uint4 u = __ldg(xb + (size_t)row * 3 * U + k);
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(h[e]);
          v[8 * (k % U) + 2 * e] += f.x;
          v[8 * (k % U) + 2 * e + 1] += f.y;
        }
      }
    } else if (row >= 0 && row < L) {
#pragma unroll
      for (int k = 0; k < U; ++k) {
        const uint4 u = __ldg(xb + (size_t)row * U + k);
        if constexpr (sizeof(T) == 2) {
          const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = __bfloat1622float2(h[e]);
            v[8 * k + 2 * e] = f.x;
            v[8 * k + 2 * e + 1] = f.y;
          }
        } else {
          v[4 * k] = __uint_as_float(u.x);
          v[4 * k + 1] = __uint_as_float(u.y);
          v[4 * k + 2] = __uint_as_float(u.z);
          v[4 * k + 3] = __uint_as_float(u.w);
        }
      }
    } else {
#pragma unroll
      for (int c = 0; c < C; ++c) v[c] = 0.0f;
    }
#pragma unroll
    for (int j = 0; j < K; ++j) {
      float s = 0.0f;
#pragma unroll
      for (int c = 0; c < C; ++c) s = fmaf(v[c], P.w[j * C + c], s);
      sd[j][i] = s;
    }
  }
  __syncthreads();
  const int lim = len ? min(len[b], L) : L;
#pragma unroll
  for (int o = 0; o < kPostPer; ++o) {
    const int tl = threadIdx.x + o * kPostThreads;  // sample within the block
    const int t = t_base + tl;
    if (t >= L) break;
    float acc = bias;
#pragma unroll
    for (int j = 0; j < K; ++j) acc += sd[j][tl + j];
    const bool dead = t >= lim;
    if (pre) pre[(size_t)b * L + t] = dead ? 0.0f : acc;
    wav[(size_t)b * L + t] = dead ? 0.0f : tanhf(acc);
  }
}

template <typename T>
__global__ void to_ncl_kernel(const T* __restrict__ x, int L, int C, float* __restrict__ y,
                              const int* __restrict__ perm) {
  pdl_wait();
  __shared__ float tile[32][33];
  const int b = blockIdx.z;
  const int t0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
  if (perm != nullptr) {
    // Permuted channels: output channel c reads input channel perm[c]
    // (gathered directly; used for the flow's small output).
    for (int i = threadIdx.y; i < 32; i += 8) {
      const int c = c0 + i, t = t0 + threadIdx.x;
      if (c < C && t < L) y[((size_t)b * C + c) * L + t] = ld_act<T>(x, ((size_t)b * L + t) * C + perm[c]);
    }
    return;
  }
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int t = t0 + i, c = c0 + threadIdx.x;
    tile[i][threadIdx.x] = (t < L && c < C) ? ld_act<T>(x, ((size_t)b * L + t) * C + c) : 0.0f;
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int c = c0 + i, t = t0 + threadIdx.x;
    if (c < C && t < L) y[((size_t)b * C + c) * L + t] = tile[threadIdx.x][i];
  }
}

// Three-piece rows [B][L][3 C] -> [B][C][L] fp32 (each value the sum of its pieces).
__global__ void to_ncl_x3_kernel(const __nv_bfloat16* __restrict__ x, int L, int C, float* __restrict__ y) {
  pdl_wait();
  __shared__ float tile[32][33];
  const int b = blockIdx.z;
  const int t0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int t = t0 + i, c = c0 + threadIdx.x;
    float v = 0.0f;
    if (t < L && c < C) {
      const __nv_bfloat16* p = x + ((size_t)b * L + t) * 3 * C + c;
      v = __bfloat162float(p[0]) + __bfloat162float(p[C]) + __bfloat162float(p[2 * C]);
    }
    tile[i][threadIdx.x] = v;
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int c = c0 + i, t = t0 + threadIdx.x;
    if (c < C && t < L) y[((size_t)b * C + c) * L + t] = tile[threadIdx.x][i];
  }
}

// WN gated activation, 8 channels per thread.
template <typename T>
__global__ void gate_kernel(const T* __restrict__ xin, const float* __restrict__ cond, int cond_ld,
                            int cond_off, int B, int L, int H, const int* __restrict__ len,
                            T* __restrict__ out) {
  pdl_wait();
  const int groups = H / 8;
  const long long total = (long long)B * L * groups;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int cg = (int)(i % groups);
    const long long bt = i / groups;
    const int b = (int)(bt / L), t = (int)(bt % L);
    const bool live = len == nullptr || t < len[b];
    const T* row = xin + bt * 2 * H;
    const float* g = cond ? cond + (size_t)b * cond_ld + cond_off : nullptr;
    float o[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int c = cg * 8 + e;
      float a = ld_act<T>(row, c), s = ld_act<T>(row, H + c);
      if (g) {
        a = a + g[c];
        s = s + g[H + c];
      }
      o[e] = live ? tanhf(a) * (1.0f / (1.0f + expf(-s))) : 0.0f;
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) st_act<T>(out, bt * H + cg * 8 + e, o[e]);
  }
}

}  // namespace

cudaError_t launch_transpose_in(const float* z, int B, int Cin, int Tsrc, int t_off, int T,
                                const int* len, void* zt, Dt dt, cudaStream_t st) {
  dim3 grid(cdiv(T, 32), cdiv(Cin, 32), B), block(32, 8);
  if (dt == Dt::X3)
    {
      const cudaError_t e_ = launch_k(transpose_in_x3_kernel, grid, block, 0, st, z, Cin, Tsrc, t_off, T, len,
                                      static_cast<__nv_bfloat16*>(zt));
      if (e_ != cudaSuccess) return e_;
    }
  else if (dt == Dt::F32)
    {
      const cudaError_t e_ = launch_k(transpose_in_kernel<float>, grid, block, 0, st, z, Cin, Tsrc, t_off, T,
                                      len, static_cast<float*>(zt));
      if (e_ != cudaSuccess) return e_;
    }
  else
    {
      const cudaError_t e_ = launch_k(transpose_in_kernel<__nv_bfloat16>, grid, block, 0, st, z, Cin, Tsrc,
                                      t_off, T, len, static_cast<__nv_bfloat16*>(zt));
      if (e_ != cudaSuccess) return e_;
    }
  return cudaGetLastError();
}

cudaError_t launch_cond(const float* g, const float* wc, const float* bc, int B, int gin, int C,
                        float* bias_bc, cudaStream_t st) {
  const int warps = B * C;
  {
    const cudaError_t e_ = launch_k(cond_kernel, cdiv(warps * 32, 256), 256, 0, st, g, wc, bc, B, gin, C,
                                    bias_bc);
    if (e_ != cudaSuccess) return e_;
  }
  return cudaGetLastError();
}

cudaError_t launch_lengths(const int* len_in, int B, int T0, const int* mul, const int* add,
                           int nstage, int* lens, cudaStream_t st) {
  if (nstage > 15) return cudaErrorInvalidValue;
  StageLen sl{};
  for (int s = 0; s < nstage; ++s) { sl.mul[s] = mul[s]; sl.add[s] = add[s]; }
  {
    const cudaError_t e_ = launch_k(lengths_kernel, cdiv(B, 128), 128, 0, st, len_in, B, T0, sl, nstage, lens);
    if (e_ != cudaSuccess) return e_;
  }
  return cudaGetLastError();
}

cudaError_t launch_zero_tails(float* wav, const int* len, int B, int T0, int hop, cudaStream_t st) {
  if (B <= 0) return cudaSuccess;
  if (B > 65535) return cudaErrorInvalidValue;
  const long long row = (long long)T0 * hop;
  const int gx = (int)std::min<long long>(cdiv((int)std::min<long long>(row, 1 << 30), 256), 64);
  {
    const cudaError_t e_ = launch_k(zero_tails_kernel, dim3(std::max(gx, 1), B), 256, 0, st, wav, len, row, hop, T0);
    if (e_ != cudaSuccess) return e_;
  }
  return cudaGetLastError();
}

cudaError_t launch_post(const void* x, Dt dt, int B, int L, int C, const float* w, const PostWeights* wh,
                        int K, int pad, float bias, const int* len, float* wav, float* pre, cudaStream_t st) {
  if (K > 64 || C != 16) return cudaErrorInvalidValue;
  if (dt == Dt::X3) {  // three-piece rows: the kernel-parameter path only
    if (wh == nullptr || K != 7) return cudaErrorNotSupported;
    {
      const cudaError_t e_ = launch_k(post_fast_kernel<__nv_bfloat16, 7, 3>,
                                      dim3(cdiv(L, kPostThreads * post_per<__nv_bfloat16>()), B), kPostThreads,
                                      0, st, static_cast<const __nv_bfloat16*>(x), L, *wh, pad, bias, len, wav, pre);
      if (e_ != cudaSuccess) return e_;
    }
    return cudaGetLastError();
  }
  if (wh != nullptr && K == 7) {
    if (dt == Dt::F32)
      {
        const cudaError_t e_ = launch_k(post_fast_kernel<float, 7>,
                                        dim3(cdiv(L, kPostThreads * post_per<float>()), B), kPostThreads, 0, st,
                                        static_cast<const float*>(x), L, *wh, pad, bias, len, wav, pre);
        if (e_ != cudaSuccess) return e_;
      }
    else
      {
        const cudaError_t e_ = launch_k(post_fast_kernel<__nv_bfloat16, 7>,
                                        dim3(cdiv(L, kPostThreads * post_per<__nv_bfloat16>()), B),
                                        kPostThreads, 0, st, static_cast<const __nv_bfloat16*>(x), L, *wh, pad,
                                        bias, len, wav, pre);
        if (e_ != cudaSuccess) return e_;
      }
    return cudaGetLastError();
  }
  dim3 grid(cdiv(L, 256 * 4), B);
  if (dt == Dt::F32)
    {
      const cudaError_t e_ = launch_k(post_kernel<float, 16>, grid, 256, 0, st, static_cast<const float*>(x), L,
                                      w, K, pad, bias, len, wav, pre);
      if (e_ != cudaSuccess) return e_;
    }
  else
    {
      const cudaError_t e_ = launch_k(post_kernel<__nv_bfloat16, 16>, grid, 256, 0, st,
                                      static_cast<const __nv_bfloat16*>(x), L, w, K, pad, bias, len, wav, pre);
      if (e_ != cudaSuccess) return e_;
    }
  return cudaGetLastError();
}

cudaError_t launch_to_ncl(const void* x, Dt dt, int B, int L, int C, float* y, cudaStream_t st,
                          const int* perm) {
  dim3 grid(cdiv(L, 32), cdiv(C, 32), B), block(32, 8);
  if (dt == Dt::X3)
    {
      if (perm != nullptr) return cudaErrorInvalidValue;
      const cudaError_t e_ = launch_k(to_ncl_x3_kernel, grid, block, 0, st, static_cast<const __nv_bfloat16*>(x),
                                      L, C, y);
      if (e_ != cudaSuccess) return e_;
    }
  else if (dt == Dt::F32)
    {
      const cudaError_t e_ = launch_k(to_ncl_kernel<float>, grid, block, 0, st, static_cast<const float*>(x), L,
                                      C, y, perm);
      if (e_ != cudaSuccess) return e_;
    }
  else
    {
      const cudaError_t e_ = launch_k(to_ncl_kernel<__nv_bfloat16>, grid, block, 0, st,
                                      static_cast<const __nv_bfloat16*>(x), L, C, y, perm);
      if (e_ != cudaSuccess) return e_;
    }
  return cudaGetLastError();
}

cudaError_t launch_gate(const void* xin, const float* cond, int cond_ld, int cond_off, int B, int L,
                        int H, const int* len, void* out, Dt dt, cudaStream_t st) {
  if (H % 8 || B <= 0 || L <= 0) return cudaErrorInvalidValue;
  const long long total = (long long)B * L * (H / 8);
  const int grid = (int)std::min<long long>((total + 255) / 256, 148LL * 16);
  if (dt == Dt::F32)
    {
      const cudaError_t e_ = launch_k(gate_kernel<float>, grid, 256, 0, st, static_cast<const float*>(xin),
                                      cond, cond_ld, cond_off, B, L, H, len, static_cast<float*>(out));
      if (e_ != cudaSuccess) return e_;
    }
  else
    {
      const cudaError_t e_ = launch_k(gate_kernel<__nv_bfloat16>, grid, 256, 0, st,
                                      static_cast<const __nv_bfloat16*>(xin), cond, cond_ld, cond_off, B, L, H,
                                      len, static_cast<__nv_bfloat16*>(out));
      if (e_ != cudaSuccess) return e_;
    }
  return cudaGetLastError();
}

}  // namespace gsv
