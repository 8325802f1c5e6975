// selftest.cu -- device side of gsvdec_selftest_wait.
//
// Runs the library's bounded hand-off wait (mbar_wait_fast, tc_common.cuh:
// the same function every tcgen05 kernel waits with) on an mbarrier that
// nothing ever completes, limited to `limit_ns`.  The wait gives up and
// reports through the handle's error word exactly as a decode kernel would;
// nothing else is in flight in the CTA (no TMA copy, no MMA, no TMEM), so it
// simply returns.  This lets a caller (and the tests) check on its own GPU
// that a wait which runs out ends the kernel and surfaces as GSV_E_TIMEOUT.
#include "gsv_kernels.h"
#include "tc_common.cuh"

namespace gsv {
namespace {

constexpr int kSelftestCode = 16;  // error code of a give-up in this kernel

__global__ void wait_selftest_kernel(int* err, unsigned long long limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // No thread arrives on `bar`: phase 0 never completes.
    if (!mbar_wait_fast(smem_u32(&bar), 0, &abort_flag, limit_ns)) raise_err(err, &abort_flag, kSelftestCode);
  }
}

}  // namespace

cudaError_t launch_wait_selftest(int* err, unsigned long long limit_ns, cudaStream_t st) {
  wait_selftest_kernel<<<1, 32, 0, st>>>(err, limit_ns);
  return cudaGetLastError();
}

}  // namespace gsv
