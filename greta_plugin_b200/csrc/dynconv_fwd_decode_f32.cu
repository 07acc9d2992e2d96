// Decode-like packed forward instantiations for element type float.
#include "dynconv_launch_decode.cuh"

namespace greta {

cudaError_t launch_fwd_decode_f32(const FwdParams& p, int norm, int gv, const LaunchShape& s, cudaStream_t st) {
  return launch_fwd_decode<float>(p, norm, gv, s, st);
}

}  // namespace greta
