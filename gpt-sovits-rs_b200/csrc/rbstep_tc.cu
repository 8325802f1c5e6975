// rbstep_tc.cu -- one whole ResBlock1 step, fused, on tcgen05 (narrow stages).
//
//   x_out = x + conv2_k,1( lrelu( conv1_k,d( lrelu(x) ) ) )   (+ biases)
//
// (src/models/sovits_decoder.rs:196-208) for the 16- and 32-channel stages,
// where the unfused step moves 6 activation tensors through HBM per branch and
// is memory-bound.  Here the conv1 output never leaves the SM: per tile of
// P = 128 - (k - 1) output rows of one utterance
//   warp 0     TMA-loads the raw window x[q0 - h2 - h1, + 128 + 2 h1) (h2 =
//              (k-1)/2, h1 = d (k-1)/2; rows outside the utterance read 0);
//   warps 2-5  write lrelu(window) to a second buffer (same swizzle), then
//              later turn the conv1 accumulator into t = lrelu(conv1 + b1) for
//              rows q0 - h2 .. q0 - h2 + 127 (rows outside [0, len) are 0: the
//              zero padding conv2 sees) as bf16 in shared memory, and finally
//              store x + conv2 + b2 for the P output rows;
//   warp 1     issues conv1 (k taps over row-shifted views of the lrelu window),
//              then conv2 (k taps over row-shifted views of t) plus the residual
//              as an identity-weight MMA over the raw window, into two TMEM
//              accumulators.
// Weights (conv1, conv2, identity) stay resident in shared memory; every CTA
// works on one branch.  The epilogue warps run one tile ahead on the window
// transform so the MMA warp always has work.  All waits are bounded.
#include "gsv_epilogue.cuh"
#include "gsv_kernels.h"
#include "gsv_pdl.cuh"
#include "tc_common.cuh"

namespace gsv {

namespace {

constexpr int kRbThreads = 192;

struct RbOpDev {
  const __nv_bfloat16* x;
  const float* b1;
  const float* b2;
  __nv_bfloat16* out_raw;
  __nv_bfloat16* out_act;
  int k, d, P, tiles, row_tiles, pad_;
};

struct alignas(64) RbParams {
  CUtensorMap mapX[kMaxGroup];
  CUtensorMap mapW1[kMaxGroup];
  CUtensorMap mapW2[kMaxGroup];
  CUtensorMap mapI;
  RbOpDev op[kMaxGroup];
  int nops, B, L;
  const int* len;
  float slope;
  int cta_base[kMaxGroup + 1];
  int a_stage;  // bytes per window buffer (multiple of 1024)
  int t_bytes;  // bytes of the t buffer (multiple of 1024)
  int* err;
  int len_smem;  // lengths copied to shared memory (B ints) rather than read per tile
};

static_assert(sizeof(RbParams) <= 4096, "kernel parameter space");

template <int C>
struct RbShape {
  static constexpr int kRow = C * 2;                          // bytes per row
  static constexpr uint32_t kW = C * C * 2;                   // bytes per weight tile
  static constexpr uint32_t kWPitch = (kW + 1023) / 1024 * 1024;
  static constexpr uint32_t kSwMask = C == 16 ? 1 : (C == 32 ? 3 : 7);
  static constexpr uint32_t kTmemCols = 2 * C <= 32 ? 32 : (2 * C <= 64 ? 64 : 128);
};

// Byte address of 16-byte chunk h of row r in a K-major swizzled buffer whose
// base is 1024-byte aligned: the swizzle XORs address bits [4, ..) with bits
// [7, ..) of the absolute shared address.
template <int C>
__device__ __forceinline__ uint32_t swz(uint32_t base, int r, int h) {
  const uint32_t a = base + (uint32_t)r * RbShape<C>::kRow + (uint32_t)h * 16;
  return a ^ (((a >> 7) & RbShape<C>::kSwMask) << 4);
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

// WS: raw windows in flight (hides the HBM latency of the next loads); 2 where
// that lets one more CTA share the SM.
template <int C, int WS>
__global__ void __launch_bounds__(kRbThreads, 1) rbstep_kernel(const __grid_constant__ RbParams P) {
  constexpr int kRbWindowStages = WS;
  using S = RbShape<C>;
  // ---- which branch this CTA serves
  int oi = 0;
  while (oi + 1 < P.nops && (int)blockIdx.x >= P.cta_base[oi + 1]) ++oi;
  const RbOpDev op = P.op[oi];
  const int lc = blockIdx.x - P.cta_base[oi];
  const int ncta = P.cta_base[oi + 1] - P.cta_base[oi];
  const int k = op.k, d = op.d, Pr = op.P;
  const int h2 = (k - 1) / 2, h1 = d * (k - 1) / 2;
  const int win_rows = kM + 2 * h1;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sW1 = smem;
  uint8_t* sW2 = sW1 + k * S::kWPitch;
  uint8_t* sI = sW2 + k * S::kWPitch;
  uint8_t* sX = sI + S::kWPitch;                       // kRbWindowStages windows
  uint8_t* sAX = sX + kRbWindowStages * P.a_stage;     // lrelu(window)
  uint8_t* sT = sAX + P.a_stage;                       // t = lrelu(conv1 + b1)
  uint64_t* bars = reinterpret_cast<uint64_t*>(sT + P.t_bytes);
  const uint32_t w_full = smem_u32(bars);
  const uint32_t x_full = w_full + 8;
  const uint32_t x_empty = x_full + 8 * kRbWindowStages;
  const uint32_t ax_full = x_empty + 8 * kRbWindowStages;
  const uint32_t acc1_full = ax_full + 8;
  const uint32_t acc1_empty = acc1_full + 8;
  const uint32_t t_full = acc1_empty + 8;
  const uint32_t acc2_full = t_full + 8;
  const uint32_t acc2_empty = acc2_full + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 8 + 2 * kRbWindowStages);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* sb = reinterpret_cast<float*>(tmem_slot + 4);  // b1[C], b2[C]
  int* slen = reinterpret_cast<int*>(sb + 2 * C);        // valid rows per utterance

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  for (int c = threadIdx.x; c < 2 * C; c += kRbThreads) sb[c] = c < C ? op.b1[c] : op.b2[c - C];
  if (threadIdx.x == 0) {
    mbar_init(w_full, 1);
    for (int s = 0; s < kRbWindowStages; ++s) {
      mbar_init(x_full + 8 * s, 1);
      mbar_init(x_empty + 8 * s, 1);
    }
    mbar_init(ax_full, 4);
    mbar_init(acc1_full, 1);
    mbar_init(acc1_empty, 4);
    mbar_init(t_full, 4);
    mbar_init(acc2_full, 1);
    mbar_init(acc2_empty, 4);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) tmem_alloc(smem_u32(tmem_slot), S::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // Everything above touched only this CTA's resources, the kernel parameters
  // and the static biases; the input window and lengths come from earlier kernels.
  pdl_wait();
  if (P.len_smem) {
    for (int b = threadIdx.x; b < P.B; b += kRbThreads) slen[b] = P.len ? P.len[b] : P.L;
    __syncthreads();
  }
  const uint32_t tmem = *tmem_slot;
  int* err = P.err;
  const int ntiles = op.tiles;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&P.mapX[oi])) : "memory");
      mbar_expect_tx(w_full, (uint32_t)(2 * k + 1) * S::kW);
      for (int j = 0; j < k; ++j) {
        tma_load_2d(smem_u32(sW1 + j * S::kWPitch), &P.mapW1[oi], w_full, 0, j * C);
        tma_load_2d(smem_u32(sW2 + j * S::kWPitch), &P.mapW2[oi], w_full, 0, j * C);
      }
      tma_load_2d(smem_u32(sI), &P.mapI, w_full, 0, 0);
      uint32_t i = 0;
      for (int t = lc; t < ntiles; t += ncta, ++i) {
        const int b = t / op.row_tiles, q0 = (t - b * op.row_tiles) * Pr;
        const uint32_t s = i % kRbWindowStages;
        if (!mbar_wait(x_empty + 8 * s, ((i / kRbWindowStages) & 1u) ^ 1u, abort)) {
          raise_err(err, abort, 11);
          break;
        }
        mbar_expect_tx(x_full + 8 * s, (uint32_t)win_rows * S::kRow);
        tma_load_3d(smem_u32(sX + s * P.a_stage), &P.mapX[oi], x_full + 8 * s, 0, q0 - h2 - h1, b);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16<C>();
      const uint32_t acc1 = tmem, acc2 = tmem + C;
      bool ok = mbar_wait(w_full, 0, abort);
      if (!ok) raise_err(err, abort, 12);
      // Descriptors built once and advanced by constant adds (address >> 4 in
      // the descriptor's start field): the single issuing thread sets the pace
      // of these short MMAs, so no per-MMA address arithmetic.
      const uint64_t w1d = sdesc<C>(smem_u32(sW1)), w2d = sdesc<C>(smem_u32(sW2)), wid = sdesc<C>(smem_u32(sI));
      const uint64_t axd = sdesc<C>(smem_u32(sAX)), tbd = sdesc<C>(smem_u32(sT));
      constexpr uint64_t kRowD = S::kRow >> 4, kWD = S::kWPitch >> 4, kK = 2;
      const uint64_t ax_step = (uint64_t)d * kRowD;
      uint32_t i = 0;
      for (int t = lc; t < ntiles && ok; t += ncta, ++i) {
        const uint32_t par = i & 1u;
        if (!mbar_wait_fast(ax_full, par, abort) ||
            !mbar_wait_fast(acc1_empty, par ^ 1u, abort)) {
          raise_err(err, abort, 13);
          break;
        }
        tc_fence_after();
        {
          // conv1: k taps over row-shifted views (dilation d) of lrelu(window)
          uint64_t ad = axd, bd = w1d;
          mma_bf16_first(acc1, ad, bd, idesc);
#pragma unroll
          for (int kk = 1; kk < C / 16; ++kk) mma_bf16_acc(acc1, ad + kk * kK, bd + kk * kK, idesc);
#pragma unroll 2
          for (int j = 1; j < k; ++j) {
            ad += ax_step;
            bd += kWD;
#pragma unroll
            for (int kk = 0; kk < C / 16; ++kk) mma_bf16_acc(acc1, ad + kk * kK, bd + kk * kK, idesc);
          }
        }
        mma_commit(acc1_full);
        if (!mbar_wait_fast(t_full, par, abort) ||
            !mbar_wait_fast(acc2_empty, par ^ 1u, abort)) {
          raise_err(err, abort, 14);
          break;
        }
        tc_fence_after();
        {
          // conv2: k taps over row-shifted views of t, then the residual as an
          // identity MMA over the raw window
          uint64_t ad = tbd, bd = w2d;
          mma_bf16_first(acc2, ad, bd, idesc);
#pragma unroll
          for (int kk = 1; kk < C / 16; ++kk) mma_bf16_acc(acc2, ad + kk * kK, bd + kk * kK, idesc);
#pragma unroll 2
          for (int j = 1; j < k; ++j) {
            ad += kRowD;
            bd += kWD;
#pragma unroll
            for (int kk = 0; kk < C / 16; ++kk) mma_bf16_acc(acc2, ad + kk * kK, bd + kk * kK, idesc);
          }
        }
        const uint32_t s = i % kRbWindowStages;
        const uint64_t xd = sdesc<C>(smem_u32(sX + s * P.a_stage) + (uint32_t)(h2 + h1) * S::kRow);
#pragma unroll
        for (int kk = 0; kk < C / 16; ++kk) mma_bf16_acc(acc2, xd + kk * kK, wid + kk * kK, idesc);
        mma_commit(x_empty + 8 * s);
        mma_commit(acc2_full);
      }
    }
  } else {
    // ------------------------------------------------ transform + epilogues
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // TMEM lane = tile row
    const int tid = threadIdx.x - 64;
    const uint32_t lane_addr = tmem + ((uint32_t)(quarter * 32) << 16);
    const uint32_t ax = smem_u32(sAX), tb = smem_u32(sT);
    const float slope = P.slope;
    const __nv_bfloat162 slope2 = __float2bfloat162_rn(slope);
    const bool v8 = ((reinterpret_cast<uintptr_t>(op.out_raw) | reinterpret_cast<uintptr_t>(op.out_act)) & 31) == 0;
    const int L = P.L;
    bool ok = true;
    // a(i): lrelu of window i into the conv1 operand buffer (same swizzle).
    auto transform = [&](uint32_t i) -> bool {
      const uint32_t s = i % kRbWindowStages;
      if (!mbar_wait_fast(x_full + 8 * s, (i / kRbWindowStages) & 1u, abort)) return false;
      const uint32_t src = smem_u32(sX + s * P.a_stage);
      const int n16 = win_rows * S::kRow / 16;
      for (int c = tid; c < n16; c += 128)
        st_shared_v4(ax + c * 16, lrelu_bf16x8(ld_shared_v4(src + c * 16), slope2));
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(ax_full);
      return true;
    };
    uint32_t i = 0;
    if (lc < ntiles) ok = transform(0);
    for (int t = lc; t < ntiles && ok; t += ncta, ++i) {
      const int b = t / op.row_tiles, q0 = (t - b * op.row_tiles) * Pr;
      const int lim = min(L, P.len_smem ? slen[b] : (P.len ? __ldg(P.len + b) : L));
      const uint32_t par = i & 1u;
      // b(i): t = lrelu(conv1 + b1) into shared memory, zero outside the utterance.
      if (!mbar_wait_fast(acc1_full, par, abort)) {
        ok = false;
        break;
      }
      tc_fence_after();
      {
        const int g1 = q0 - h2 + r;
        const bool live = g1 >= 0 && g1 < lim;
#pragma unroll
        for (int c0 = 0; c0 < C; c0 += 16) {
          float v[16];
          tmem_ld16(lane_addr + (uint32_t)c0, v);
#pragma unroll
          for (int e = 0; e < 16; ++e) v[e] = v[e] + sb[c0 + e];
          uint4 u0 = lrelu_bf16x8(pack_bf16x8(v), slope2), u1 = lrelu_bf16x8(pack_bf16x8(v + 8), slope2);
          if (!live) u0 = u1 = make_uint4(0, 0, 0, 0);
          st_shared_v4(swz<C>(tb, r, c0 / 8), u0);
          st_shared_v4(swz<C>(tb, r, c0 / 8 + 1), u1);
        }
      }
      tc_fence_before();
      fence_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(acc1_empty);
        mbar_arrive(t_full);
      }
      // a(i+1): the next window's transform (conv1(i) has finished with the buffer).
      if (t + ncta < ntiles && !transform(i + 1)) {
        ok = false;
        break;
      }
      // c(i): x + conv2 + b2 for the P output rows.
      if (!mbar_wait_fast(acc2_full, par, abort)) {
        ok = false;
        break;
      }
      tc_fence_after();
      {
        const int g = q0 + r;
        const bool store = r < Pr && g < L;
        const bool dead = g >= lim;
        const size_t base = ((size_t)b * L + (store ? g : 0)) * C;
#pragma unroll
        for (int c0 = 0; c0 < C; c0 += 16) {
          float v[16];
          tmem_ld16(lane_addr + (uint32_t)(C + c0), v);
#pragma unroll
          for (int e = 0; e < 16; ++e) v[e] = dead ? 0.0f : v[e] + sb[C + c0 + e];
          const uint4 x0 = pack_bf16x8(v), x1 = pack_bf16x8(v + 8);
          if (store) {
            // A 16-channel run is 32 bytes at a 32-byte offset: one 256-bit
            // store where the output bases are 32-byte aligned.
            if (op.out_raw) {
              if (v8) {
                st_global_v8(op.out_raw + base + c0, x0, x1);
              } else {
                *reinterpret_cast<uint4*>(op.out_raw + base + c0) = x0;
                *reinterpret_cast<uint4*>(op.out_raw + base + c0 + 8) = x1;
              }
            }
            if (op.out_act) {
              const uint4 a0 = lrelu_bf16x8(x0, slope2), a1 = lrelu_bf16x8(x1, slope2);
              if (v8) {
                st_global_v8(op.out_act + base + c0, a0, a1);
              } else {
                *reinterpret_cast<uint4*>(op.out_act + base + c0) = a0;
                *reinterpret_cast<uint4*>(op.out_act + base + c0 + 8) = a1;
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc2_empty);
    }
    if (!ok && lane == 0) raise_err(err, abort, 15);
  }
  // This CTA's work is done: the next kernel's CTAs may be scheduled.
  pdl_trigger();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, S::kTmemCols);
  }
}

template <int C>
size_t rb_smem(const RbParams& P, int ws) {
  using S = RbShape<C>;
  int kmax = 0;
  for (int i = 0; i < P.nops; ++i) kmax = std::max(kmax, P.op[i].k);
  return 1024 + (size_t)(2 * kmax + 1) * S::kWPitch + (size_t)(ws + 1) * P.a_stage + P.t_bytes +
         8 * (8 + 2 * ws) + 16 + 2 * C * sizeof(float) + (P.len_smem ? sizeof(int) * (size_t)P.B : 0);
}

// CTAs of rbstep_kernel<C, WS> per SM for these parameters, bounded by
// shared memory (1 KB reserved per CTA), registers, threads and TMEM; 0 when
// the kernel cannot be set up.
template <int C, int WS>
int rb_per_sm(const RbParams& P) {
  using S = RbShape<C>;
  const size_t smem = rb_smem<C>(P, WS);
  if (smem > 227 * 1024) return 0;
  int nregs = 0;
  if (kernel_setup(rbstep_kernel<C, WS>, smem, &nregs) != cudaSuccess) return 0;
  const int regs_cta = ((nregs * 32 + 255) / 256 * 256) * (kRbThreads / 32);
  return std::max(1, std::min({smem_per_sm() / (int)(smem + 1024), 65536 / std::max(regs_cta, 1),
                               2048 / kRbThreads, (int)(512 / S::kTmemCols)}));
}

template <int C, int WS>
cudaError_t launch_c(RbParams& P, cudaStream_t st) {
  const size_t smem = rb_smem<C>(P, WS);
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  auto kern = rbstep_kernel<C, WS>;
  int nregs = 0;
  cudaError_t e = kernel_setup(kern, smem, &nregs);
  if (e != cudaSuccess) return e;
  const int smem_sm = smem_per_sm();
  const int per_sm = rb_per_sm<C, WS>(P);
  if (per_sm < 1) return cudaErrorInvalidValue;
  // Split the persistent CTAs over the branches in proportion to their tiles.
  long long total = 0;
  for (int i = 0; i < P.nops; ++i) total += P.op[i].tiles;
  const int ctas = sm_count() * per_sm;
  P.cta_base[0] = 0;
  for (int i = 0; i < P.nops; ++i) {
    int n = (int)std::max<long long>(1, (long long)ctas * P.op[i].tiles / std::max<long long>(total, 1));
    n = std::min(n, P.op[i].tiles);
    P.cta_base[i + 1] = P.cta_base[i] + n;
  }
  {
    const size_t smem_launch = pad_smem_to_occupancy(smem, per_sm, smem_sm);
    e = kernel_setup(kern, smem_launch, &nregs);
    if (e != cudaSuccess) return e;
    const cudaError_t e_ = launch_k(kern, P.cta_base[P.nops], kRbThreads, smem_launch, st, P);
    if (e_ != cudaSuccess) return e_;
  }
  return cudaGetLastError();
}

}  // namespace

bool rbstep_supported(int C, int k, int d) {
  return (C == 16 || C == 32) && k >= 1 && k <= 15 && d >= 1 && d * (k - 1) <= 256 - kM;
}

cudaError_t launch_rbstep(const RbStepGroup& g, cudaStream_t st) {
  if (!encode_fn()) return cudaErrorNotSupported;
  if (g.n < 1 || g.n > kMaxGroup || !rbstep_supported(g.C, 1, 1)) return cudaErrorInvalidValue;
  RbParams P;
  memset(&P, 0, sizeof P);
  P.nops = g.n;
  P.B = g.B;
  P.L = g.L;
  P.len = g.len;
  P.slope = g.slope;
  P.err = g.err;
  P.len_smem = g.B <= 1024;
  int max_win = kM;
  for (int i = 0; i < g.n; ++i) {
    const RbStepOp& o = g.op[i];
    if (!rbstep_supported(g.C, o.k, o.d) || (o.k - 1) % 2) return cudaErrorInvalidValue;
    RbOpDev& d = P.op[i];
    d.x = static_cast<const __nv_bfloat16*>(o.x);
    d.b1 = o.b1;
    d.b2 = o.b2;
    d.out_raw = static_cast<__nv_bfloat16*>(o.out_raw);
    d.out_act = static_cast<__nv_bfloat16*>(o.out_act);
    d.k = o.k;
    d.d = o.d;
    d.P = kM - (o.k - 1);
    d.row_tiles = cdiv(g.L, d.P);
    d.tiles = g.B * d.row_tiles;
    const int rows = kM + o.d * (o.k - 1);
    max_win = std::max(max_win, rows);
    if (!encode_act(&P.mapX[i], o.x, g.B, g.L, g.C, g.C, rows)) return cudaErrorInvalidValue;
    if (!encode_w(&P.mapW1[i], o.w1, o.k * g.C, g.C, g.C, g.C)) return cudaErrorInvalidValue;
    if (!encode_w(&P.mapW2[i], o.w2, o.k * g.C, g.C, g.C, g.C)) return cudaErrorInvalidValue;
  }
  if (!encode_w(&P.mapI, g.identity, g.C, g.C, g.C, g.C)) return cudaErrorInvalidValue;
  P.a_stage = (max_win * g.C * 2 + 1023) / 1024 * 1024;
  P.t_bytes = ((kM + 16) * g.C * 2 + 1023) / 1024 * 1024;
  if (g.B <= 0 || g.L <= 0) return cudaSuccess;
  // Each branch is its own launch, with shared memory sized for its own kernel
  // width (the k = 11 branch's weights would otherwise set every CTA's size),
  // and two window stages where that fits one more CTA per SM.
  for (int i = 0; i < g.n; ++i) {
    RbParams Q = P;
    Q.nops = 1;
    Q.op[0] = P.op[i];
    Q.mapX[0] = P.mapX[i];
    Q.mapW1[0] = P.mapW1[i];
    Q.mapW2[0] = P.mapW2[i];
    Q.a_stage = ((kM + Q.op[0].d * (Q.op[0].k - 1)) * g.C * 2 + 1023) / 1024 * 1024;
    // The 2-deep ring only where it buys a CTA per SM once registers, threads
    // and TMEM are counted too (shared memory alone would pick it for every
    // 16-channel branch, whose registers allow no extra CTA).
    cudaError_t e;
    if (g.C == 16) {
      const bool two = rb_per_sm<16, 2>(Q) > rb_per_sm<16, 3>(Q);
      e = two ? launch_c<16, 2>(Q, st) : launch_c<16, 3>(Q, st);
    } else {
      const bool two = rb_per_sm<32, 2>(Q) > rb_per_sm<32, 3>(Q);
      e = two ? launch_c<32, 2>(Q, st) : launch_c<32, 3>(Q, st);
    }
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace gsv
