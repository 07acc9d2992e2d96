// Decode-like and wide-group packed forward instantiations for element type float.
#include "dynconv_fwd_wide.cuh"
#include "dynconv_launch_decode.cuh"

namespace greta {

cudaError_t launch_fwd_decode_f32(const FwdParams& p, int norm, int gv, const LaunchShape& s, cudaStream_t st) {
  return launch_fwd_decode<float>(p, norm, gv, s, st);
}

cudaError_t launch_fwd_wide_f32(const FwdParams& p, int norm, dim3 grid, dim3 block, int groups, cudaStream_t st) {
  return launch_fwd_wide<float>(p, norm, grid, block, groups, st);
}

}  // namespace greta
