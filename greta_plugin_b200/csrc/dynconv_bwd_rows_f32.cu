// Row-streaming backward instantiations for element type float.
#include "dynconv_launch_bwd_rows.cuh"

namespace greta {

cudaError_t launch_bwd_rows_f32(const BwdRowsParams& p, int norm, int gv, dim3 grid, dim3 block, size_t smem,
                              cudaStream_t st) {
  return launch_bwd_rows<float>(p, norm, gv, grid, block, smem, st);
}

int device_errors_bwd_rows_f32(bool clear) { return read_device_errors(clear); }

}  // namespace greta
