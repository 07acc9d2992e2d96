// Kernel instantiations for element type float.
#include "dynconv_launch.cuh"

namespace greta {

cudaError_t launch_fwd_f32(const FwdParams& p, int nv, int norm, int gv, const LaunchShape& s,
                         cudaStream_t st) {
  return launch_fwd<float>(p, nv, norm, gv, s, st);
}

cudaError_t launch_bwd_f32(const BwdParams& p, int nv, int norm, int gv, const LaunchShape& s,
                         cudaStream_t st) {
  return launch_bwd<float>(p, nv, norm, gv, s, st);
}

cudaError_t launch_fwd_rows_f32(const RowsParams& p, int norm, int gv, dim3 grid, dim3 block, size_t smem,
                                cudaStream_t st) {
  return launch_fwd_rows<float>(p, norm, gv, grid, block, smem, st);
}

int device_errors_f32(bool clear) { return read_device_errors(clear); }

}  // namespace greta
