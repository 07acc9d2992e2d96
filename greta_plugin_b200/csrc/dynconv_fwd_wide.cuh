// vLLM packed forward for norm groups wider than one warp's 256 channels
// (G >= 512, a power of two dividing D): greta_vllm/triton_conv.py:28-116,
// whose supports() (:119-121) accepts any such G and tiles channels by
// BD = max(G, 128), one whole group per program.
//
// A CTA owns ONE group (G channels, filter f) for a chunk of up to `chunk`
// tokens of one request; its threads stride over the group's 8-channel
// vectors (any G, up to the whole row). Every channel of a vector shares the token's W filter values
// (G >= 8), which are CTA-uniform loads. The group's RMS statistics are a
// block reduction (warp butterflies, then the warps' partials through shared
// memory, added in warp order by every thread, so all threads hold the same
// totals). The conv is recomputed after the reduction instead of being kept:
// a group of any width then needs no per-token buffer, and the history rows
// the recomputation reads again are L1/L2 hits.
//
// History and the cache slot follow dynconv_fwd_kernel (dynconv_fwd.cuh):
// CTA row r < num_reqs is request r's first chunk (chunk >= W-1 tokens, so
// only it reaches before the request's first token and reads the slot's old
// taps); after its tokens it writes the slot's new taps for its channels --
// the same threads that read them, so no barrier is needed. Slots are
// addressed through their strides (any layout).
#pragma once

#include "dynconv_launch.cuh"

namespace greta {

constexpr int kWideThreads = 256;
constexpr int kWideChunk = 16;  // tokens per CTA row (>= W-1 for W <= 16)

// Sum and max of one value per thread over the CTA; every thread returns the
// same totals. All threads must call it.
__device__ __forceinline__ void block_sum_max(float& s, float& m) {
  __shared__ float sh_s[32], sh_m[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    s += __shfl_xor_sync(0xffffffffu, s, o);
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  }
  if (lane == 0) {
    sh_s[warp] = s;
    sh_m[warp] = m;
  }
  __syncthreads();
  s = 0.f;
  m = 0.f;
  for (int i = 0; i < nw; ++i) {
    s += sh_s[i];
    m = fmaxf(m, sh_m[i]);
  }
  __syncthreads();  // the arrays are reused by the next call
}

// Input vector of channels [d0, d0 + 8) at local position q of the chunk's
// request: a request row for q >= 0, else the slot's old tap H + q (zeros
// without history).
template <typename T>
__device__ __forceinline__ Pack<T, kVec> wide_input(const FwdParams& p, const ChunkInfo& ci, long long q, int d0,
                                                    int H) {
  if (q >= 0) return ld<T, kVec>(reinterpret_cast<const T*>(p.x) + (ci.x_base + q) * p.ldx + d0);
  Pack<T, kVec> v;
  zero(v);
  if (ci.has_state) {
    const T* base = reinterpret_cast<const T*>(p.state) + ci.slot * p.s_slot + (long long)(H + q) * p.s_h;
#pragma unroll
    for (int j = 0; j < kVec; ++j) v.v[j] = base[(long long)(d0 + j) * p.s_d];
  }
  return v;
}

// The conv of one vector at local position t, taps oldest first (the
// arithmetic of the other forward kernels: fp32 sums, one FMA per tap).
template <typename T>
__device__ __forceinline__ void wide_conv(const FwdParams& p, const ChunkInfo& ci, long long t, int d0, int W,
                                          const T (&wk)[kMaxWGeneric], float (&acc)[kVec]) {
#pragma unroll
  for (int c = 0; c < kVec; ++c) acc[c] = 0.f;
  for (int k = 0; k < W; ++k) {
    const Pack<T, kVec> xv = wide_input<T>(p, ci, t + k - (W - 1), d0, W - 1);
#pragma unroll
    for (int c = 0; c < kVec; ++c) acc[c] = fma_io(xv.v[c], wk[k], acc[c]);
  }
}

template <typename T, int NORM>
__global__ void __launch_bounds__(kWideThreads) dynconv_fwd_wide_kernel(const FwdParams p) {
  pdl_wait();
  pdl_trigger();
  const int W = p.W, H = W - 1, D = p.D, G = p.G;
  ChunkInfo ci;
  if (!resolve_fwd_chunk(p, ci, W)) return;
  const long long f = blockIdx.x % p.nblk;  // the group (filter) of this CTA
  const int g0 = (int)(f * G);
  const int nvec = G / kVec;
  const long long DC = D / G;
  const float inv_g = 1.f / (float)G;  // G is a power of two: exact
  const T* __restrict__ wg = reinterpret_cast<const T*>(p.w);
  const T* __restrict__ gg = reinterpret_cast<const T*>(p.g);
  T* __restrict__ yg = reinterpret_cast<T*>(p.y);

  for (long long t = ci.c0; t < ci.c1; ++t) {
    const long long orow = ci.o_base + t;
    T wk[kMaxWGeneric];
#pragma unroll
    for (int k = 0; k < kMaxWGeneric; ++k) wk[k] = k < W ? wg[orow * p.ldw + k * DC + f] : from_f<T>(0.f);
    float scale = 1.f;
    if (NORM != kNormNone) {
      float ss = 0.f, mx = 0.f;
      for (int v = threadIdx.x; v < nvec; v += blockDim.x) {
        float acc[kVec];
        wide_conv<T>(p, ci, t, g0 + v * kVec, W, wk, acc);
#pragma unroll
        for (int c = 0; c < kVec; ++c) {
          ss = fmaf(acc[c], acc[c], ss);
          mx = fmaxf(mx, fabsf(acc[c]));
        }
      }
      block_sum_max(ss, mx);
      if (NORM == kNormPlain) {
        scale = rsqrtf(ss * inv_g + p.eps);
      } else if (mx < 0x1p48f) {
        // overflow-safe form s * sqrt(mean((y/s)^2) + eps/s^2), s = max(max|y|, 1),
        // equals sqrt(mean(y^2) + eps); below 2^48 the sum of fewer than 2^32
        // squares (G <= D < 2^30) stays below 2^128, so it is computed directly
        scale = rsqrtf(ss * inv_g + p.eps);
      } else {
        // the rescaled form (also taken for a NaN)
        const float rs = __frcp_rn(fmaxf(mx, 1.f));
        float s2 = 0.f, unused = 0.f;
        for (int v = threadIdx.x; v < nvec; v += blockDim.x) {
          float acc[kVec];
          wide_conv<T>(p, ci, t, g0 + v * kVec, W, wk, acc);
#pragma unroll
          for (int c = 0; c < kVec; ++c) {
            const float q = acc[c] * rs;
            s2 = fmaf(q, q, s2);
          }
        }
        block_sum_max(s2, unused);
        scale = rs * rsqrtf(s2 * inv_g + p.eps * rs * rs);
      }
    }
    for (int v = threadIdx.x; v < nvec; v += blockDim.x) {
      const int d0 = g0 + v * kVec;
      float acc[kVec];
      wide_conv<T>(p, ci, t, d0, W, wk, acc);
      if (gg != nullptr) {
        const Pack<T, kVec> gv = ld<T, kVec>(gg + orow * p.ldg + d0);
#pragma unroll
        for (int c = 0; c < kVec; ++c) {
          const float gf = to_f(gv.v[c]);
          acc[c] = (acc[c] * scale) * (gf * sigmoidf_(gf));
        }
      } else {
#pragma unroll
        for (int c = 0; c < kVec; ++c) acc[c] *= scale;
      }
      Pack<T, kVec> o;
#pragma unroll
      for (int c = 0; c < kVec; ++c) o.v[c] = from_f<T>(acc[c]);
      st<T, kVec>(yg + orow * D + d0, o);
    }
  }

  // the slot's new taps: tap h = the input at local position len - H + h
  // (a request row, or the old tap len + h for requests shorter than W-1)
  if (ci.hist == kHistState && ci.head && ci.slot >= 0) {
    T* base = reinterpret_cast<T*>(p.state) + ci.slot * p.s_slot;
    for (int v = threadIdx.x; v < nvec; v += blockDim.x) {
      const int d0 = g0 + v * kVec;
      Pack<T, kVec> taps[kMaxWGeneric - 1];
      for (int h = 0; h < H; ++h) taps[h] = wide_input<T>(p, ci, ci.len - H + h, d0, H);
      for (int h = 0; h < H; ++h)
#pragma unroll
        for (int j = 0; j < kVec; ++j) base[(long long)(d0 + j) * p.s_d + (long long)h * p.s_h] = taps[h].v[j];
    }
  }
}

template <typename T>
cudaError_t launch_fwd_wide(FwdParams p, int norm, dim3 grid, dim3 block, int nblk, cudaStream_t st) {
  p.nblk = nblk;
  switch (norm) {
    case kNormNone: return launch_pdl(dynconv_fwd_wide_kernel<T, kNormNone>, grid, block, 0, st, p);
    case kNormPlain: return launch_pdl(dynconv_fwd_wide_kernel<T, kNormPlain>, grid, block, 0, st, p);
    case kNormStable: return launch_pdl(dynconv_fwd_wide_kernel<T, kNormStable>, grid, block, 0, st, p);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace greta
