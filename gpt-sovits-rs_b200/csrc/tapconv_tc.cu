// tapconv_tc.cu -- bf16 tap GEMM on the 5th-generation tensor cores (tcgen05).
//
// One CTA computes a 128-row x NT-column tile of a tap GEMM (gsv_internal.h)
// for one utterance:
//   warp 0      TMA producer: for every (segment, tap, channel chunk) it loads
//               the tap-shifted activation tile [128 rows x CK channels] from
//               the time-major activation (a 3-D tensor map over (C, L, B),
//               whose out-of-range rows read as zero = the conv zero padding)
//               and the weight tile [NT x CK] into a STAGES-deep ring;
//   warp 1      allocates TMEM and issues tcgen05.mma (M=128, N=NT, K=16,
//               bf16 x bf16 -> fp32 in TMEM), committing each stage back to
//               the producer and the finished accumulator to the epilogue;
//   warps 2-5   epilogue: tcgen05.ld of the accumulator rows, then the fused
//               bias / cond / residual / branch-average / LeakyReLU of
//               gsv_epilogue.cuh, stored as bf16 in 16-byte vectors.
// Operands are K-major with the swizzle that matches the chunk width
// (64 ch -> 128B, 32 ch -> 64B, 16 ch -> 32B).  Every mbarrier wait is
// bounded; a wait that gives up sets the group's error word and the CTA
// drains and frees its TMEM instead of hanging.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>

#include "gsv_epilogue.cuh"
#include "gsv_kernels.h"

namespace gsv {

namespace {

constexpr int kM = 128;
constexpr int kThreads = 192;
constexpr uint32_t kWaitLimit = 1u << 25;

struct alignas(64) TcParams {
  CUtensorMap mapA[kMaxSeg];  // activation maps, one per flattened segment
  CUtensorMap mapB[kMaxSeg];  // weight maps
  TapConvGroup grp;
  int seg_base[kMaxGroup];    // first flattened segment of each op
};

// ---------------------------------------------------------------- PTX helpers
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: false after kWaitLimit polls (each poll itself may suspend).
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  for (uint32_t i = 0; i < kWaitLimit; ++i)
    if (mbar_try(bar, parity)) return true;
  return false;
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void mma_bf16(uint32_t tmem, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// K-major shared-memory matrix descriptor (tcgen05): start address, LBO = 16 B
// (unused by swizzled K-major), SBO = 8 rows, version 1, swizzle = row width.
template <int CK>
__device__ __forceinline__ uint64_t sdesc(uint32_t addr) {
  constexpr uint64_t layout = CK == 64 ? 2 : (CK == 32 ? 4 : 6);  // SW128 / SW64 / SW32
  constexpr uint64_t sbo = (8 * CK * 2) >> 4;
  return (uint64_t)((addr >> 4) & 0x3FFF) | (1ull << 16) | (sbo << 32) | (1ull << 46) |
         (layout << 61);
}

// Instruction descriptor: D fp32, A/B bf16, both K-major, M = 128, N = NT.
template <int NT>
__host__ __device__ constexpr uint32_t idesc_bf16() {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(NT >> 3) << 17) |
         ((uint32_t)(kM >> 4) << 24);
}

__device__ __forceinline__ void raise_err(int* err, int code) {
  if (err) atomicExch(err, code);
}

// Epilogue of 16 consecutive GEMM columns [n, n + 16) of row q: their flat
// output indices are consecutive (see gsv_internal.h), so the residuals and
// outputs move as two 16-byte vectors when the run is fully in range.
__device__ __forceinline__ void epi_run16(const TapConv& op, int b, int q, int n, const float* acc) {
  const long long total = (long long)op.Lout * op.Cout;
  const long long e0 = (long long)q * op.N + n - op.crop;
  if (e0 < 0 || e0 + 16 > total) {
#pragma unroll 1
    for (int i = 0; i < 16; ++i) epi_element<__nv_bfloat16>(op, b, q, n + i, acc[i]);
    return;
  }
  const size_t base = (size_t)b * (size_t)total + (size_t)e0;
  int t = (int)(e0 / op.Cout);
  int c = (int)(e0 - (long long)t * op.Cout);
  const int lim = op.len ? op.len[b] : 0x7fffffff;
#pragma unroll
  for (int g = 0; g < 2; ++g) {
    float v[8];
    uint32_t dead = 0;  // masked rows (t >= len[b]) stay exactly zero
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float x = acc[g * 8 + i] + op.bias[c];
      if (op.bias_bc != nullptr) x += op.bias_bc[(size_t)b * op.Cout + c];
      v[i] = x;
      if (t >= lim) dead |= 1u << i;
      if (++c == op.Cout) { c = 0; ++t; }
    }
    for (int r = 0; r < op.nres; ++r) {
      const uint4 raw = *reinterpret_cast<const uint4*>(
          static_cast<const __nv_bfloat16*>(op.res[r]) + base + g * 8);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(h[i]);
        v[2 * i] = f.x + v[2 * i];
        v[2 * i + 1] = f.y + v[2 * i + 1];
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (dead >> i & 1u) v[i] = 0.0f;
    if (op.div != 1.0f) {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = v[i] / op.div;
    }
    if (op.out_raw != nullptr) {
      uint4 o;
      __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
      for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
      *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(op.out_raw) + base + g * 8) = o;
    }
    if (op.out_act != nullptr) {
      uint4 o;
      __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
      for (int i = 0; i < 4; ++i)
        h[i] = __floats2bfloat162_rn(lrelu(v[2 * i], op.slope), lrelu(v[2 * i + 1], op.slope));
      *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(op.out_act) + base + g * 8) = o;
    }
  }
}

template <int CK, int NT, int STAGES>
struct TcCfg {
  static constexpr uint32_t kABytes = kM * CK * 2;
  static constexpr uint32_t kBBytes = NT * CK * 2;
  static constexpr uint32_t kBPitch = (kBBytes + 1023) / 1024 * 1024;
  static constexpr uint32_t kStage = kABytes + kBPitch;
  static constexpr uint32_t kTmemCols = NT <= 32 ? 32 : (NT <= 64 ? 64 : (NT <= 128 ? 128 : 256));
  static constexpr size_t kSmem = 1024 + (size_t)STAGES * kStage + 256;
};

template <int CK, int NT, int STAGES>
__global__ void __launch_bounds__(kThreads, 1) tapconv_tc_kernel(const __grid_constant__ TcParams P) {
  using C = TcCfg<CK, NT, STAGES>;
  const TapConv& op = P.grp.op[blockIdx.z];
  const int b = blockIdx.x / op.row_tiles;
  if (b >= op.B) return;
  const int q0 = (blockIdx.x % op.row_tiles) * kM;
  const int n0 = blockIdx.y * NT;
  if (n0 >= op.N) return;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * C::kStage);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 1);
  const uint32_t full0 = smem_u32(bars);
  const uint32_t empty0 = smem_u32(bars + STAGES);
  const uint32_t accum = smem_u32(bars + 2 * STAGES);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const bool masked = op.len != nullptr && first_out_row(op, q0) >= op.len[b];
  int iters = 0;
  if (!masked)
    for (int s = 0; s < op.nseg; ++s) iters += op.seg[s].ntaps * (op.seg[s].Cin / CK);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    mbar_init(accum, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) tmem_alloc(smem_u32(tmem_slot), C::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0 && iters > 0) {
      int it = 0;
      bool ok = true;
      for (int s = 0; s < op.nseg && ok; ++s) {
        const TapSeg& sg = op.seg[s];
        const CUtensorMap* ma = &P.mapA[P.seg_base[blockIdx.z] + s];
        const CUtensorMap* mb = &P.mapB[P.seg_base[blockIdx.z] + s];
        for (int j = 0; j < sg.ntaps && ok; ++j) {
          const int row = q0 + sg.off0 + j * sg.offstep;
          for (int c0 = 0; c0 < sg.Cin; c0 += CK, ++it) {
            const int st = it % STAGES;
            const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
            if (!mbar_wait(empty0 + 8 * st, ph ^ 1u)) {
              raise_err(P.grp.err, 1);
              ok = false;
              break;
            }
            const uint32_t a = smem_u32(smem + st * C::kStage);
            mbar_expect_tx(full0 + 8 * st, C::kABytes + C::kBBytes);
            tma_load_3d(a, ma, full0 + 8 * st, c0, row, b);
            tma_load_2d(a + C::kABytes, mb, full0 + 8 * st, c0, j * op.N + n0);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && iters > 0) {
      constexpr uint32_t idesc = idesc_bf16<NT>();
      for (int it = 0; it < iters; ++it) {
        const int st = it % STAGES;
        const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
        if (!mbar_wait(full0 + 8 * st, ph)) {
          raise_err(P.grp.err, 2);
          break;
        }
        tc_fence_after();
        const uint32_t a = smem_u32(smem + st * C::kStage);
        const uint32_t bb = a + C::kABytes;
#pragma unroll
        for (int kk = 0; kk < CK / 16; ++kk)
          mma_bf16(tmem, sdesc<CK>(a + kk * 32), sdesc<CK>(bb + kk * 32), idesc,
                   (it | kk) != 0 ? 1u : 0u);
        mma_commit(empty0 + 8 * st);
      }
      mma_commit(accum);  // also covers an early exit: arrives once issued MMAs finish
    }
  } else {
    const int quarter = warp & 3;  // TMEM lanes this warp may access
    const int row = quarter * 32 + lane;
    const int q = q0 + row;
    bool have = iters > 0;
    if (have) {
      const bool ok = mbar_wait(accum, 0);
      if (!ok) raise_err(P.grp.err, 3);
      have = __all_sync(0xffffffffu, ok);
      tc_fence_after();
    }
#pragma unroll 1
    for (int c0 = 0; c0 < NT; c0 += 16) {
      float v[16];
      if (have) {
        tmem_ld16(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)c0, v);
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = 0.0f;
      }
      if (q < op.Q && (have || iters == 0)) epi_run16(op, b, q, n0 + c0, v);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

// ------------------------------------------------------------------- host side
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

CUtensorMapSwizzle swizzle_for(int ck) {
  return ck == 64 ? CU_TENSOR_MAP_SWIZZLE_128B
                  : (ck == 32 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B);
}

// Activation [B][Lin][Cin] bf16 as a 3-D map (Cin, Lin, B); box CK x 128 x 1.
bool encode_act(CUtensorMap* m, const void* x, int B, int Lin, int Cin, int ck) {
  cuuint64_t dims[3] = {(cuuint64_t)Cin, (cuuint64_t)Lin, (cuuint64_t)B};
  cuuint64_t strides[2] = {(cuuint64_t)Cin * 2, (cuuint64_t)Lin * Cin * 2};
  cuuint32_t box[3] = {(cuuint32_t)ck, (cuuint32_t)kM, 1};
  cuuint32_t es[3] = {1, 1, 1};
  return encode_fn()(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(x), dims, strides, box,
                     es, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle_for(ck),
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

// Weights [ntaps * N][Cin] bf16 as a 2-D map; box CK x NT.
bool encode_w(CUtensorMap* m, const void* w, int rows, int Cin, int ck, int nt) {
  cuuint64_t dims[2] = {(cuuint64_t)Cin, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)Cin * 2};
  cuuint32_t box[2] = {(cuuint32_t)ck, (cuuint32_t)nt};
  cuuint32_t es[2] = {1, 1};
  return encode_fn()(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(w), dims, strides, box,
                     es, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle_for(ck),
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

int ck_for(int cin) { return cin % 64 == 0 ? 64 : (cin == 32 ? 32 : (cin == 16 ? 16 : 0)); }
int nt_for(int n) {
  if (n <= 256) return (n % 16 == 0 && n >= 16) ? n : 0;
  return n % 256 == 0 ? 256 : (n % 128 == 0 ? 128 : 0);
}

template <int CK, int NT, int STAGES>
cudaError_t launch_cfg(TcParams& P, cudaStream_t st) {
  using C = TcCfg<CK, NT, STAGES>;
  static_assert(C::kSmem <= 227 * 1024, "shared memory budget");
  cudaError_t e = cudaFuncSetAttribute(tapconv_tc_kernel<CK, NT, STAGES>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::kSmem);
  if (e != cudaSuccess) return e;
  int gx = 0, gy = 0;
  for (int i = 0; i < P.grp.n; ++i) {
    TapConv& op = P.grp.op[i];
    op.row_tiles = cdiv(op.Q, kM);
    gx = max(gx, op.B * op.row_tiles);
    gy = max(gy, op.N / NT);
  }
  if (gx == 0 || gy == 0) return cudaSuccess;
  tapconv_tc_kernel<CK, NT, STAGES><<<dim3(gx, gy, P.grp.n), kThreads, C::kSmem, st>>>(P);
  return cudaGetLastError();
}

}  // namespace

bool tapconv_tc_supported(const TapConv& op) {
  if (op.nseg < 1 || op.nseg > kMaxSeg) return false;
  const int cin = op.seg[0].Cin;
  for (int s = 0; s < op.nseg; ++s)
    if (op.seg[s].Cin != cin || op.seg[s].ntaps < 1) return false;
  const int ck = ck_for(cin), nt = nt_for(op.N);
  if (!ck || !nt || op.N % nt) return false;
  if (op.Cout % 16) return false;  // 16-element epilogue runs stay row-aligned in bytes
  // Instantiated (CK, NT) pairs.
  return (ck == 64 && (nt == 256 || nt == 128 || nt == 64)) || (ck == 32 && nt == 32) ||
         (ck == 16 && nt == 16);
}

cudaError_t launch_tapconv_tc(const TapConvGroup& g, cudaStream_t st) {
  if (!encode_fn()) return cudaErrorNotSupported;
  TcParams P;
  memset(&P, 0, sizeof P);
  P.grp = g;
  int nseg = 0;
  const int ck = ck_for(g.op[0].seg[0].Cin), nt = nt_for(g.op[0].N);
  for (int i = 0; i < g.n; ++i) {
    const TapConv& op = g.op[i];
    if (!tapconv_tc_supported(op) || ck_for(op.seg[0].Cin) != ck || nt_for(op.N) != nt)
      return cudaErrorInvalidValue;
    P.seg_base[i] = nseg;
    for (int s = 0; s < op.nseg; ++s, ++nseg) {
      if (nseg >= kMaxSeg) return cudaErrorInvalidValue;
      const TapSeg& sg = op.seg[s];
      if (!encode_act(&P.mapA[nseg], sg.x, op.B, sg.Lin, sg.Cin, ck)) return cudaErrorInvalidValue;
      if (!encode_w(&P.mapB[nseg], sg.w, sg.ntaps * op.N, sg.Cin, ck, nt)) return cudaErrorInvalidValue;
    }
  }
  if (ck == 64 && nt == 256) return launch_cfg<64, 256, 4>(P, st);
  if (ck == 64 && nt == 128) return launch_cfg<64, 128, 4>(P, st);
  if (ck == 64 && nt == 64) return launch_cfg<64, 64, 4>(P, st);
  if (ck == 32 && nt == 32) return launch_cfg<32, 32, 4>(P, st);
  if (ck == 16 && nt == 16) return launch_cfg<16, 16, 4>(P, st);
  return cudaErrorInvalidValue;
}

}  // namespace gsv
