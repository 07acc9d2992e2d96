// Compile-time dispatch from runtime (NV, W, norm, GV) to a kernel
// instantiation. The W template argument is the exact kernel size when > 0
// (the common W = 4 and W = 7), or -MAXW for a runtime W <= MAXW. Included once per element type (dynconv_<dtype>.cu) so the
// three element types compile in parallel.
#pragma once

#include "dynconv_bwd.cuh"
#include "dynconv_bwd_tma.cuh"
#include "dynconv_fwd.cuh"
#include "dynconv_fwd_tma.cuh"

namespace greta {

struct LaunchShape {
  dim3 grid;
  dim3 block;
  int nblk = 1;     // channel blocks (blockIdx.x = chunk * nblk + channel block)
  size_t smem = 0;  // dynamic shared memory per CTA
};

// Launch with programmatic stream serialization: the kernel may start while
// the kernel ahead of it in the stream finishes, and waits for it
// (pdl_wait) before its first access to global memory. Captured into CUDA
// graphs as a programmatic edge.
template <typename P>
cudaError_t launch_pdl(void (*k)(P), dim3 grid, dim3 block, size_t smem, cudaStream_t st, const P& p) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k, p);
}

// Raise a kernel's dynamic shared-memory limit when a launch needs more than
// the default 48 KB (large W with wide CTAs, or fp32).
template <typename K>
cudaError_t allow_smem(K kernel, size_t smem) {
  if (smem <= 48 * 1024) return cudaSuccess;
  return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
}

template <typename T, int NV, int WT, int NORM, int GV>
cudaError_t fwd_one(FwdParams p, const LaunchShape& s, cudaStream_t st) {
  auto k = dynconv_fwd_kernel<T, NV, WT, NORM, GV>;
  cudaError_t e = allow_smem(k, s.smem);
  if (e != cudaSuccess) return e;
  p.nblk = s.nblk;
  return launch_pdl(k, s.grid, s.block, s.smem, st, p);
}

template <typename T, int NV, int WT, int NORM>
cudaError_t fwd_gv(const FwdParams& p, int gv, const LaunchShape& s, cudaStream_t st) {
  if constexpr (NV == kVec) {
    switch (gv) {
      case 8: return fwd_one<T, NV, WT, NORM, 8>(p, s, st);
      case 4: return fwd_one<T, NV, WT, NORM, 4>(p, s, st);
      case 2: return fwd_one<T, NV, WT, NORM, 2>(p, s, st);
      case 1: return fwd_one<T, NV, WT, NORM, 1>(p, s, st);
      default: return cudaErrorInvalidValue;
    }
  } else {
    if (gv != 1) return cudaErrorInvalidValue;
    return fwd_one<T, NV, WT, NORM, 1>(p, s, st);
  }
}

template <typename T, int NV, int WT>
cudaError_t fwd_norm(const FwdParams& p, int norm, int gv, const LaunchShape& s, cudaStream_t st) {
  switch (norm) {
    case kNormNone: return fwd_gv<T, NV, WT, kNormNone>(p, gv, s, st);
    case kNormPlain: return fwd_gv<T, NV, WT, kNormPlain>(p, gv, s, st);
    case kNormStable: return fwd_gv<T, NV, WT, kNormStable>(p, gv, s, st);
    default: return cudaErrorInvalidValue;
  }
}

template <typename T>
cudaError_t launch_fwd(const FwdParams& p, int nv, int norm, int gv, const LaunchShape& s,
                       cudaStream_t st) {
  if (nv == kVec) {
    if (p.W == 4) return fwd_norm<T, kVec, 4>(p, norm, gv, s, st);
    if (p.W == 7) return fwd_norm<T, kVec, 7>(p, norm, gv, s, st);
    if (p.W <= 8) return fwd_norm<T, kVec, -8>(p, norm, gv, s, st);
    return fwd_norm<T, kVec, -kMaxWGeneric>(p, norm, gv, s, st);
  }
  return fwd_norm<T, 1, -kMaxWGeneric>(p, norm, gv, s, st);
}

template <typename T, int NV, int WT, int NORM, int GV>
cudaError_t bwd_one(BwdParams p, const LaunchShape& s, cudaStream_t st) {
  p.nblk = s.nblk;
  return launch_pdl(dynconv_bwd_kernel<T, NV, WT, NORM, GV>, s.grid, s.block, 0, st, p);
}

template <typename T, int NV, int WT, int NORM>
cudaError_t bwd_gv(const BwdParams& p, int gv, const LaunchShape& s, cudaStream_t st) {
  if constexpr (NV == kVec) {
    switch (gv) {
      case 8: return bwd_one<T, NV, WT, NORM, 8>(p, s, st);
      case 4: return bwd_one<T, NV, WT, NORM, 4>(p, s, st);
      case 2: return bwd_one<T, NV, WT, NORM, 2>(p, s, st);
      case 1: return bwd_one<T, NV, WT, NORM, 1>(p, s, st);
      default: return cudaErrorInvalidValue;
    }
  } else {
    if (gv != 1) return cudaErrorInvalidValue;
    return bwd_one<T, NV, WT, NORM, 1>(p, s, st);
  }
}

template <typename T, int NV, int WT>
cudaError_t bwd_norm(const BwdParams& p, int norm, int gv, const LaunchShape& s, cudaStream_t st) {
  switch (norm) {
    case kNormNone: return bwd_gv<T, NV, WT, kNormNone>(p, gv, s, st);
    case kNormPlain: return bwd_gv<T, NV, WT, kNormPlain>(p, gv, s, st);
    default: return cudaErrorInvalidValue;
  }
}

template <typename T>
cudaError_t launch_bwd(const BwdParams& p, int nv, int norm, int gv, const LaunchShape& s,
                       cudaStream_t st) {
  if (nv == kVec) {
    if (p.W == 4) return bwd_norm<T, kVec, 4>(p, norm, gv, s, st);
    if (p.W == 7) return bwd_norm<T, kVec, 7>(p, norm, gv, s, st);
    if (p.W <= 8) return bwd_norm<T, kVec, -8>(p, norm, gv, s, st);
    return bwd_norm<T, kVec, -kMaxWGeneric>(p, norm, gv, s, st);
  }
  return bwd_norm<T, 1, -kMaxWGeneric>(p, norm, gv, s, st);
}

template <typename T, int WT, int NORM, int GV>
cudaError_t rows_one(const RowsParams& p, dim3 grid, dim3 block, size_t smem, cudaStream_t st) {
  auto k = dynconv_fwd_rows_kernel<T, WT, NORM, GV>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  return launch_pdl(k, grid, block, smem, st, p);
}

template <typename T, int WT, int NORM>
cudaError_t rows_gv(const RowsParams& p, int gv, dim3 grid, dim3 block, size_t smem, cudaStream_t st) {
  switch (gv) {
    case 8: return rows_one<T, WT, NORM, 8>(p, grid, block, smem, st);
    case 4: return rows_one<T, WT, NORM, 4>(p, grid, block, smem, st);
    case 2: return rows_one<T, WT, NORM, 2>(p, grid, block, smem, st);
    case 1: return rows_one<T, WT, NORM, 1>(p, grid, block, smem, st);
    default: return cudaErrorInvalidValue;
  }
}

template <typename T, int WT>
cudaError_t rows_norm(const RowsParams& p, int norm, int gv, dim3 grid, dim3 block, size_t smem, cudaStream_t st) {
  switch (norm) {
    case kNormNone: return rows_gv<T, WT, kNormNone>(p, gv, grid, block, smem, st);
    case kNormPlain: return rows_gv<T, WT, kNormPlain>(p, gv, grid, block, smem, st);
    case kNormStable: return rows_gv<T, WT, kNormStable>(p, gv, grid, block, smem, st);
    default: return cudaErrorInvalidValue;
  }
}

template <typename T>
cudaError_t launch_fwd_rows(const RowsParams& p, int norm, int gv, dim3 grid, dim3 block, size_t smem,
                            cudaStream_t st) {
  if (p.W == 4) return rows_norm<T, 4>(p, norm, gv, grid, block, smem, st);
  if (p.W == 7) return rows_norm<T, 7>(p, norm, gv, grid, block, smem, st);
  if (p.W <= 8) return rows_norm<T, -8>(p, norm, gv, grid, block, smem, st);
  return rows_norm<T, -kMaxWGeneric>(p, norm, gv, grid, block, smem, st);
}

// Entry points defined by the per-dtype translation units.
cudaError_t launch_fwd_f32(const FwdParams&, int, int, int, const LaunchShape&, cudaStream_t);
cudaError_t launch_fwd_f16(const FwdParams&, int, int, int, const LaunchShape&, cudaStream_t);
cudaError_t launch_fwd_bf16(const FwdParams&, int, int, int, const LaunchShape&, cudaStream_t);
cudaError_t launch_bwd_f32(const BwdParams&, int, int, int, const LaunchShape&, cudaStream_t);
cudaError_t launch_bwd_f16(const BwdParams&, int, int, int, const LaunchShape&, cudaStream_t);
cudaError_t launch_bwd_bf16(const BwdParams&, int, int, int, const LaunchShape&, cudaStream_t);
cudaError_t launch_fwd_rows_f32(const RowsParams&, int, int, dim3, dim3, size_t, cudaStream_t);
cudaError_t launch_fwd_rows_f16(const RowsParams&, int, int, dim3, dim3, size_t, cudaStream_t);
cudaError_t launch_fwd_rows_bf16(const RowsParams&, int, int, dim3, dim3, size_t, cudaStream_t);
// decode-like packed forward (dynconv_fwd_decode_<dtype>.cu)
cudaError_t launch_fwd_decode_f32(const FwdParams&, int, int, const LaunchShape&, cudaStream_t);
cudaError_t launch_fwd_decode_f16(const FwdParams&, int, int, const LaunchShape&, cudaStream_t);
cudaError_t launch_fwd_decode_bf16(const FwdParams&, int, int, const LaunchShape&, cudaStream_t);
// packed forward for groups wider than 256 channels (dynconv_fwd_decode_<dtype>.cu)
cudaError_t launch_fwd_wide_f32(const FwdParams&, int, dim3, dim3, int, cudaStream_t);
cudaError_t launch_fwd_wide_f16(const FwdParams&, int, dim3, dim3, int, cudaStream_t);
cudaError_t launch_fwd_wide_bf16(const FwdParams&, int, dim3, dim3, int, cudaStream_t);
int device_errors_f32(bool clear);
int device_errors_f16(bool clear);
int device_errors_bf16(bool clear);
// row-streaming backward (dynconv_bwd_rows_<dtype>.cu)
cudaError_t launch_bwd_rows_f32(const BwdRowsParams&, int, int, dim3, dim3, size_t, cudaStream_t);
cudaError_t launch_bwd_rows_f16(const BwdRowsParams&, int, int, dim3, dim3, size_t, cudaStream_t);
cudaError_t launch_bwd_rows_bf16(const BwdRowsParams&, int, int, dim3, dim3, size_t, cudaStream_t);
int device_errors_bwd_rows_f32(bool clear);
int device_errors_bwd_rows_f16(bool clear);
int device_errors_bwd_rows_bf16(bool clear);

}  // namespace greta
