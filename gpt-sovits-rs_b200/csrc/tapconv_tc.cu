// tapconv_tc.cu -- bf16 tcgen05 tap GEMM (placeholder until the kernel lands).
#include "gsv_kernels.h"

namespace gsv {
bool tapconv_tc_supported(const TapConv&) { return false; }
cudaError_t launch_tapconv_tc(const TapConvGroup&, cudaStream_t) { return cudaErrorNotSupported; }
}  // namespace gsv
