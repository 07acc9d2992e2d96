// Decode-like packed forward instantiations for element type __half.
#include "dynconv_launch_decode.cuh"

namespace greta {

cudaError_t launch_fwd_decode_f16(const FwdParams& p, int norm, int gv, const LaunchShape& s, cudaStream_t st) {
  return launch_fwd_decode<__half>(p, norm, gv, s, st);
}

}  // namespace greta
