// Pieces shared by the row-streaming kernels (dynconv_fwd_tma.cuh,
// dynconv_bwd_tma.cuh): limits, the device error word, mbarrier and bulk-copy
// primitives (inline PTX), and the request lookup over sequence offsets held
// in shared memory.
#pragma once

#include "dynconv_common.cuh"

namespace greta {

constexpr int kMaxStages = 8;
constexpr int kMaxSeqsTma = 2048;   // sequence offsets held in shared memory
constexpr int kErrTimeout = 2;      // device error bit: an mbarrier wait gave up

// Most channels per CTA of the row-streaming forward for a filter-width
// template WT (exact W > 0, or -MAXW): each consumer thread keeps W-1 inputs
// of its 8 channels in registers, and a 1-CTA-per-SM launch of 32 + C/8
// threads leaves 96 registers per thread at C = 4096, 168 at 2048 and 255
// at 1024; wider filters (and the runtime-W templates, which keep more
// state) take narrower CTAs so that little or nothing spills.
__host__ __device__ constexpr int fwd_rows_max_channels(int wt) {
  return wt == 4 ? 4096 : (wt == 7 ? 2048 : (wt >= -8 ? 1024 : 512));
}

// Device error word of this translation unit; read and cleared on the host
// through greta_dynconv_device_errors.
static __device__ int g_tma_errors = 0;

// Read (and clear) this translation unit's device error word. Internal
// linkage: every translation unit reads its own word.
static inline int read_device_errors(bool clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_tma_errors, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v != 0) {
    const int z = 0;
    cudaMemcpyToSymbol(g_tma_errors, &z, sizeof(int));
  }
  return v;
}

// ---------------------------------------------------------------------------
// mbarrier and bulk-copy primitives (PTX)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(unsigned bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(unsigned bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(unsigned bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}

// Polls of a pipeline wait: 2^24 (about a second) unless a launch option
// asks for fewer (tests that make a wait run out).
__host__ __device__ constexpr unsigned wait_limit(int log2) {
  return (log2 >= 8 && log2 <= 24) ? (1u << log2) : (1u << 24);
}

// Bounded wait for the phase with the given parity; false once `limit`
// polls have passed.
__device__ __forceinline__ bool mbar_wait(unsigned bar, unsigned parity, unsigned limit) {
  for (unsigned it = 0; it < limit; ++it) {
    unsigned done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    if (done) return true;
    if (it > 64) __nanosleep(64);
  }
  return false;
}

// Bulk prefetch of [src, src + bytes) into L2, in pieces of at most 256 KB;
// bytes a multiple of 16, src 16-byte aligned. Completion is not tracked.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, unsigned bytes) {
  const char* a = static_cast<const char*>(src);
  while (bytes > 0) {
    const unsigned n = bytes < (256u << 10) ? bytes : (256u << 10);
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(a), "r"(n) : "memory");
    a += n;
    bytes -= n;
  }
}

// global -> shared bulk copy; bytes a multiple of 16, both addresses 16-byte aligned
__device__ __forceinline__ void bulk_g2s(unsigned dst, const void* src, unsigned bytes, unsigned bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

// ---------------------------------------------------------------------------
// ranges
// ---------------------------------------------------------------------------
// last s in [0, n) with bnd[s] <= v (bnd non-decreasing, bnd[0] <= v)
__device__ __forceinline__ long long seq_of(const long long* bnd, long long n, long long v) {
  long long lo = 0, hi = n - 1;
  while (lo < hi) {
    const long long mid = (lo + hi + 1) >> 1;
    if (bnd[mid] <= v)
      lo = mid;
    else
      hi = mid - 1;
  }
  return lo;
}

// Make the offsets in shared memory non-decreasing (a decreasing offset is an
// empty request) when some thread saw a decrease; all threads call this after
// the barrier that published the offsets, and it ends with one when it works.
__device__ __forceinline__ void monotone_offsets(long long* bnd, long long nseq, int any_decrease) {
  if (!any_decrease) return;  // uniform: the barrier's reduction
  if (threadIdx.x == 0)
    for (long long i = 1; i <= nseq; ++i)
      if (bnd[i] < bnd[i - 1]) bnd[i] = bnd[i - 1];
  __syncthreads();
}

// Load the sequence offsets into shared memory (clamped to [0, T]) and make
// them non-decreasing: a decreasing offset is an empty request. Ends with a
// CTA barrier.
__device__ __forceinline__ void load_offsets(long long* bnd, const void* starts, int is64, long long nseq,
                                             long long T) {
  int dec = 0;  // this thread saw a decreasing offset
  for (long long i = threadIdx.x; i <= nseq; i += blockDim.x) {
    const long long v = clampll(load_idx(starts, i, is64), 0, T);
    bnd[i] = v;
    if (i > 0 && v < clampll(load_idx(starts, i - 1, is64), 0, T)) dec = 1;
  }
  monotone_offsets(bnd, nseq, __syncthreads_or(dec));
}

}  // namespace greta
