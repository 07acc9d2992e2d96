// Compile-time dispatch of the row-streaming backward (dynconv_bwd_tma.cuh)
// from runtime (W, norm, GV) to a kernel instantiation. Included once per
// element type (dynconv_bwd_rows_<dtype>.cu), apart from the other kernels,
// so that all instantiations compile in parallel. W: 4 and 7 exact, else a
// runtime W <= 8.
#pragma once

#include "dynconv_launch.cuh"

namespace greta {

template <typename T, int WT, int NORM, int GV>
cudaError_t bwd_rows_one(const BwdRowsParams& p, dim3 grid, dim3 block, size_t smem, cudaStream_t st) {
  auto k = dynconv_bwd_rows_kernel<T, WT, NORM, GV>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  return launch_pdl(k, grid, block, smem, st, p);
}

template <typename T, int WT, int NORM>
cudaError_t bwd_rows_gv(const BwdRowsParams& p, int gv, dim3 grid, dim3 block, size_t smem, cudaStream_t st) {
  switch (gv) {
    case 8: return bwd_rows_one<T, WT, NORM, 8>(p, grid, block, smem, st);
    case 4: return bwd_rows_one<T, WT, NORM, 4>(p, grid, block, smem, st);
    case 2: return bwd_rows_one<T, WT, NORM, 2>(p, grid, block, smem, st);
    case 1: return bwd_rows_one<T, WT, NORM, 1>(p, grid, block, smem, st);
    default: return cudaErrorInvalidValue;
  }
}

template <typename T, int WT>
cudaError_t bwd_rows_norm(const BwdRowsParams& p, int norm, int gv, dim3 grid, dim3 block, size_t smem,
                          cudaStream_t st) {
  switch (norm) {
    case kNormNone: return bwd_rows_gv<T, WT, kNormNone>(p, gv, grid, block, smem, st);
    case kNormPlain: return bwd_rows_gv<T, WT, kNormPlain>(p, gv, grid, block, smem, st);
    default: return cudaErrorInvalidValue;
  }
}

template <typename T>
cudaError_t launch_bwd_rows(const BwdRowsParams& p, int norm, int gv, dim3 grid, dim3 block, size_t smem,
                            cudaStream_t st) {
  if (p.W == 4) return bwd_rows_norm<T, 4>(p, norm, gv, grid, block, smem, st);
  if (p.W == 7) return bwd_rows_norm<T, 7>(p, norm, gv, grid, block, smem, st);
  if (p.W <= kMaxWBwdRows) return bwd_rows_norm<T, -kMaxWBwdRows>(p, norm, gv, grid, block, smem, st);
  return cudaErrorInvalidValue;
}

}  // namespace greta
