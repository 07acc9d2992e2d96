// Kernel instantiations for element type __half.
#include "dynconv_launch.cuh"

namespace greta {

cudaError_t launch_fwd_f16(const FwdParams& p, int nv, int norm, int gv, const LaunchShape& s,
                         cudaStream_t st) {
  return launch_fwd<__half>(p, nv, norm, gv, s, st);
}

cudaError_t launch_bwd_f16(const BwdParams& p, int nv, int norm, int gv, const LaunchShape& s,
                         cudaStream_t st) {
  return launch_bwd<__half>(p, nv, norm, gv, s, st);
}

cudaError_t launch_fwd_rows_f16(const RowsParams& p, int norm, int gv, dim3 grid, dim3 block, size_t smem,
                                cudaStream_t st) {
  return launch_fwd_rows<__half>(p, norm, gv, grid, block, smem, st);
}

int device_errors_f16(bool clear) { return read_device_errors(clear); }

}  // namespace greta
