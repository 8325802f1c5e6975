// tc_common.cuh -- PTX helpers, descriptors and tensor-map encoding shared by
// the tcgen05 kernels (tapconv_tc.cu, rbstep_tc.cu).  Everything lives in an
// anonymous namespace: each translation unit gets its own copy.
#pragma once
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <mutex>

namespace gsv {
namespace {

constexpr int kM = 128;  // MMA rows per tile (TMEM lanes)
// Bounded waits: each poll may suspend the warp for up to kSuspendNs until the
// barrier phase completes (so idle roles stop consuming issue slots); after
// kWaitPolls polls (about 1.3 s) the wait gives up and reports an error.
constexpr uint32_t kSuspendNs = 20000;
constexpr uint32_t kWaitPolls = 1u << 16;
constexpr uint32_t kHandoffNs = 1000;  // suspension bound on accumulator hand-offs
constexpr uint64_t kFastWaitNs = 2000000000ull;  // bound of a hand-off wait (2 s)

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

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Bounded wait: false after about kWaitPolls * kSuspendNs, or as soon as
// another role of the CTA has given up.  `hint_ns` bounds each poll's
// suspension: short on the accumulator hand-offs (latency-critical), long on
// the producer's ring waits.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort,
                                          uint32_t hint_ns = kSuspendNs) {
  const uint32_t polls = hint_ns >= kSuspendNs ? kWaitPolls : kWaitPolls * (kSuspendNs / (hint_ns | 1));
  for (uint32_t i = 0; i < polls; ++i) {
    if (mbar_try(bar, parity, hint_ns)) return true;
    if (*abort) return false;
  }
  return false;
}

__device__ __forceinline__ bool mbar_try_nohint(uint32_t bar, uint32_t parity) {
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

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Wait for the latency-critical hand-offs between the roles of a CTA:
// try_wait without a suspend-time hint sleeps until the phase completes
// (wake-up measured at about 120 cycles, and a sleeping warp takes no issue
// slots).  Bounded by kFastWaitNs of wall time; abandoned as soon as another
// role gave up.
__device__ __forceinline__ bool mbar_wait_fast(uint32_t bar, uint32_t parity, volatile int* abort,
                                               uint64_t limit_ns = kFastWaitNs) {
  if (mbar_try_nohint(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 1; i != 0; ++i) {
    if (mbar_try_nohint(bar, parity)) return true;
    if ((i & 15u) == 0 && (*abort || global_ns() - t0 > limit_ns)) return false;
  }
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

// Generic-proxy shared-memory writes become visible to the async proxy
// (TMA, tcgen05.mma) that reads them next.
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
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

// The same MMA with the accumulate flag fixed: D = A.B (starts an
// accumulator) and D += A.B.  No predicate to compute per MMA.
__device__ __forceinline__ void mma_bf16_first(uint32_t tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc) {
  asm volatile("tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, 0;" ::"r"(tmem), "l"(adesc), "l"(bdesc),
               "r"(idesc));
}
__device__ __forceinline__ void mma_bf16_acc(uint32_t tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc) {
  asm volatile("tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, 1;" ::"r"(tmem), "l"(adesc), "l"(bdesc),
               "r"(idesc));
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
// (unused by swizzled K-major), SBO = 8 rows, version 1, base offset 0,
// swizzle = row width.  Valid for any row-aligned start (absolute-address swizzle).
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

// The error word may live in mapped host memory (the handle's), so it is set
// with a plain system-visible store: any non-zero code marks the call failed.
__device__ __forceinline__ void raise_err(int* err, volatile int* abort, int code) {
  *abort = 1;
  if (err) {
    *reinterpret_cast<volatile int*>(err) = code;
    __threadfence_system();
  }
}

__device__ __forceinline__ void store8(__nv_bfloat16* p, const float* v) {
  uint4 o;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = o;
}

// One 256-bit global store of two 16-byte halves (p 32-byte aligned; sm_100).
__device__ __forceinline__ void st_global_v8(void* p, uint4 lo, uint4 hi) {
  asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "r"(lo.x), "r"(lo.y),
               "r"(lo.z), "r"(lo.w), "r"(hi.x), "r"(hi.y), "r"(hi.z), "r"(hi.w)
               : "memory");
}

// One 256-bit read-only global load into two 16-byte halves (p 32-byte aligned).
__device__ __forceinline__ void ld_global_nc_v8(const void* p, uint4& lo, uint4& hi) {
  asm volatile("ld.global.nc.v8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(lo.x), "=r"(lo.y), "=r"(lo.z), "=r"(lo.w), "=r"(hi.x), "=r"(hi.y), "=r"(hi.z), "=r"(hi.w)
               : "l"(p));
}

// 8 floats -> 8 packed bf16 (round to nearest even).
__device__ __forceinline__ uint4 pack_bf16x8(const float* v) {
  uint4 o;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  return o;
}

// LeakyReLU of 8 packed bf16 values in bf16 arithmetic, max(x, x * slope)
// (slope in [0, 1]): two instructions per pair instead of unpack, fp32
// multiply, max and repack.  For x < 0 it rounds x * bf16(slope) once, which
// can differ from rounding fp32(x) * slope by one bf16 ulp.
__device__ __forceinline__ uint4 lrelu_bf16x8(uint4 u, __nv_bfloat162 s2) {
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __hmax2(h[i], __hmul2(h[i], s2));
  return u;
}

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

// Activation [B][Lin][Cin] bf16 as a 3-D map (Cin, Lin, B); box CK x rows x 1.
bool encode_act(CUtensorMap* m, const void* x, int B, int Lin, int Cin, int ck, int rows) {
  cuuint64_t dims[3] = {(cuuint64_t)Cin, (cuuint64_t)Lin, (cuuint64_t)B};
  cuuint64_t strides[2] = {(cuuint64_t)Cin * 2, (cuuint64_t)Lin * Cin * 2};
  cuuint32_t box[3] = {(cuuint32_t)ck, (cuuint32_t)rows, 1};
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
// Column tile of an N-column GEMM: the widest of 256 / 128 / 64 that divides N
// (N = 192 or 384 tile by 64 / 128), else N itself for the 16/32-column convs.
int nt_for(int n) {
  if (n % 256 == 0) return 256;
  if (n % 128 == 0) return 128;
  if (n % 64 == 0) return 64;
  return (n == 32 || n == 16) ? n : 0;
}

int window_rows(const TapSeg& s) { return kM + (s.ntaps - 1) * abs(s.offstep); }

struct DevInfo {
  int sms = 0;
};

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (!cached[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

int smem_per_sm() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 228 * 1024;
  if (!cached[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
    cached[dev] = n > 0 ? n : 228 * 1024;
  }
  return cached[dev];
}

// Launch setup of a kernel done once per (kernel, device) instead of per
// launch: the shared-memory carveout, the register count, and the dynamic
// shared-memory limit (raised only when a launch needs more).  Short launches
// (the flow's) were bound by these host calls.
// Dynamic shared memory for a launch meant to hold per_sm CTAs per SM: smem,
// padded where needed so that per_sm + 1 CTAs (1 KB reserved each) do not fit
// the SM's shared memory.  A persistent grid of sm_count x per_sm CTAs then
// lands exactly per_sm CTAs on every SM even when its CTAs are placed while
// the previous kernel still holds some SMs (programmatic dependent launch);
// otherwise an early-free SM can take extra CTAs (TMEM or registers permitting
// only later) while another SM gets fewer, and the launch ends late.
size_t pad_smem_to_occupancy(size_t smem, int per_sm, int smem_sm) {
  const size_t floor_excl = (size_t)(smem_sm / (per_sm + 1)) + 16;  // (per_sm + 1) x this > smem_sm
  const size_t pad = floor_excl > 1024 ? floor_excl - 1024 : 0;
  const size_t out = std::max(smem, pad);
  return out <= 227 * 1024 ? out : smem;
}

// Slots per device and kernel signature: every instantiation of a kernel
// template shares one signature, and the tap GEMM has a few dozen.
constexpr int kSetupSlots = 64;

template <typename K>
cudaError_t kernel_setup(K kern, size_t smem, int* regs) {
  struct Entry {
    int regs = 0, smem = 0;
    bool ready = false;
  };
  static std::mutex mu;
  static Entry table[64][kSetupSlots];
  static const void* keys[64][kSetupSlots] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(mu);
  Entry* en = nullptr;
  for (int i = 0; i < kSetupSlots && !en; ++i) {
    if (keys[dev][i] == (const void*)kern) en = &table[dev][i];
    else if (!keys[dev][i]) {
      keys[dev][i] = (const void*)kern;
      en = &table[dev][i];
    }
  }
  Entry scratch;
  if (!en) en = &scratch;  // more instantiations than slots on one device: no caching
  if (!en->ready) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                                         cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return e;
    cudaFuncAttributes fa;
    e = cudaFuncGetAttributes(&fa, kern);
    if (e != cudaSuccess) return e;
    en->regs = fa.numRegs;
    en->ready = true;
  }
  if ((int)smem > en->smem) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    en->smem = (int)smem;
  }
  *regs = en->regs;
  return cudaSuccess;
}

}  // namespace
}  // namespace gsv
