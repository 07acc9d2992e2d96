// Decode-like and wide-group packed forward instantiations for element type __half.
#include "dynconv_fwd_wide.cuh"
#include "dynconv_launch_decode.cuh"

namespace greta {

cudaError_t launch_fwd_decode_f16(const FwdParams& p, int norm, int gv, const LaunchShape& s, cudaStream_t st) {
  return launch_fwd_decode<__half>(p, norm, gv, s, st);
}

cudaError_t launch_fwd_wide_f16(const FwdParams& p, int norm, dim3 grid, dim3 block, int groups, cudaStream_t st) {
  return launch_fwd_wide<__half>(p, norm, grid, block, groups, st);
}

}  // namespace greta
