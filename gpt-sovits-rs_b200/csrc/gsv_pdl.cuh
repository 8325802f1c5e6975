// gsv_pdl.cuh -- programmatic dependent launch (PDL) for every kernel of the
// library.
//
// One forward is a chain of 35-45 kernels on one stream, each depending on the
// one before.  Launched with the programmatic-stream-serialisation attribute,
// kernel i+1's CTAs may be scheduled before kernel i has finished; they do
// their set-up (shared-memory carve-up, mbarrier init, TMEM allocation:
// nothing another kernel writes) and then block in pdl_wait() until kernel i
// has completed and its writes are visible.  That hides the launch latency and
// the set-up of i+1 behind the end of i.
//
// Rules every kernel here follows:
//  * pdl_wait() is executed by all threads of every CTA, before the first
//    global-memory access to activations, lengths or any buffer another kernel
//    reads or writes, and before any early return.  Because every kernel waits,
//    kernel i+1 completing implies kernel i completed: the stream order stays
//    transitive.
//  * pdl_trigger() (where a kernel issues it at all; a CTA that exits counts
//    as triggered) comes when the CTA's work is done.  Triggered at the start,
//    the next kernel's CTAs sat on the SMs for the whole kernel and every
//    persistent decoder launch ran 2-4 % slower.  A CTA holds its TMEM before
//    it triggers, so a dependent CTA never takes TMEM it still needs.
//  * Without the attribute (or with PDL disabled) both are no-ops.
#pragma once
#include <cuda_runtime.h>

#include <cstdlib>
#include <utility>

namespace gsv {

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// PDL is used only inside a PdlScope: the entry points open one where it
// measured faster.  On B200 (bf16, 16 x 10 s) the flow inverse's 39 short,
// sub-wave launches went from 0.68 to 0.58 ms per call with it; the decoder's
// persistent launches (0.1-0.3 ms each) and the EncP chains measured 1-4 %
// slower, so they launch without it.  GSVDEC_NO_PDL set to a non-empty value
// other than "0" turns it off everywhere (read once per process).
inline bool pdl_allowed() {
  static const bool on = [] {
    const char* v = std::getenv("GSVDEC_NO_PDL");
    return !(v && *v && !(v[0] == '0' && v[1] == 0));
  }();
  return on;
}

inline bool& pdl_scope_flag() {
  static thread_local bool on = false;
  return on;
}

// Launches made by this thread while a PdlScope is alive carry the attribute.
struct PdlScope {
  bool prev;
  explicit PdlScope(bool on) : prev(pdl_scope_flag()) { pdl_scope_flag() = on; }
  ~PdlScope() { pdl_scope_flag() = prev; }
  PdlScope(const PdlScope&) = delete;
  PdlScope& operator=(const PdlScope&) = delete;
};

inline bool pdl_enabled() { return pdl_scope_flag() && pdl_allowed(); }

// kern<<<grid, block, smem, st>>>(args...), with the PDL attribute inside a
// PdlScope.
template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                     Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

}  // namespace gsv
