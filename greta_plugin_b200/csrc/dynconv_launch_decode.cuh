// Compile-time dispatch of the decode-like packed forward
// (dynconv_fwd_decode.cuh) from runtime (W, norm, GV) to a kernel
// instantiation. Included once per element type
// (dynconv_fwd_decode_<dtype>.cu), apart from the other kernels, so that all
// instantiations compile in parallel. W: 4 or 7.
#pragma once

#include "dynconv_fwd_decode.cuh"
#include "dynconv_launch.cuh"

namespace greta {

template <typename T, int WT, int NORM, int GV>
cudaError_t decode_one(FwdParams p, const LaunchShape& s, cudaStream_t st) {
  p.nblk = s.nblk;
  if (p.mode == kModeRows) return launch_pdl(dynconv_fwd_decode_kernel<T, WT, NORM, GV, true>, s.grid, s.block, 0, st, p);
  return launch_pdl(dynconv_fwd_decode_kernel<T, WT, NORM, GV, false>, s.grid, s.block, 0, st, p);
}

template <typename T, int WT, int NORM>
cudaError_t decode_gv(const FwdParams& p, int gv, const LaunchShape& s, cudaStream_t st) {
  switch (gv) {
    case 8: return decode_one<T, WT, NORM, 8>(p, s, st);
    case 4: return decode_one<T, WT, NORM, 4>(p, s, st);
    case 2: return decode_one<T, WT, NORM, 2>(p, s, st);
    case 1: return decode_one<T, WT, NORM, 1>(p, s, st);
    default: return cudaErrorInvalidValue;
  }
}

template <typename T, int WT>
cudaError_t decode_norm(const FwdParams& p, int norm, int gv, const LaunchShape& s, cudaStream_t st) {
  switch (norm) {
    case kNormNone: return decode_gv<T, WT, kNormNone>(p, gv, s, st);
    case kNormPlain: return decode_gv<T, WT, kNormPlain>(p, gv, s, st);
    case kNormStable: return decode_gv<T, WT, kNormStable>(p, gv, s, st);
    default: return cudaErrorInvalidValue;
  }
}

template <typename T>
cudaError_t launch_fwd_decode(const FwdParams& p, int norm, int gv, const LaunchShape& s, cudaStream_t st) {
  if (p.W == 4) return decode_norm<T, 4>(p, norm, gv, s, st);
  if (p.W == 7) return decode_norm<T, 7>(p, norm, gv, s, st);
  return cudaErrorInvalidValue;
}

}  // namespace greta
