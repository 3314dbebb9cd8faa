// tcgen05 / TMEM working-set attention (placeholder until the tensor-core kernel lands).
#include "hga_common.cuh"
namespace hga {
bool attend_tc_supported(const hga_params& p) { (void)p; return false; }
cudaError_t launch_attend_tc(const hga_params&, int64_t, const void*, int, const void*, const void*, int64_t,
                             const int32_t*, const int32_t*, int, void*, int, cudaStream_t) {
  return cudaErrorNotSupported;
}
}  // namespace hga
