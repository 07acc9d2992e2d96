// Forward family of the dynamic causal depthwise convolution.
//
// One kernel template serves four callers, selected by FwdParams::mode:
//   SINGLE / PACKED  training forward over cu_seqlens segments, zero history
//                    (greta/dynamic_conv.py:179-261 dynconv_fwd_kernel)
//   CONTEXT          HF batched inference; history = W-1 context rows
//                    (greta/dynamic_conv.py:435-506 dynconv_inference_kernel)
//   ROWS             HF single-token decode; history = conv_state[row], shifted
//                    in place (greta/dynamic_conv.py:513-602 dynconv_decode_kernel)
//   PACKED + state   vLLM packed batch; history = cache slot; the slot's new
//                    contents are written by the same thread that read the old
//                    ones (greta_vllm/triton_conv.py:28-116, both kernels fused)
//
// Per thread: NV channels x a run of L tokens, walked in time order with the
// last W-1 input vectors kept in registers. Loads of U consecutive tokens are
// issued before their arithmetic so every thread keeps several 16-byte loads
// in flight.
#pragma once

#include "dynconv_common.cuh"

namespace greta {

__device__ __forceinline__ bool resolve_fwd_chunk(const FwdParams& p, ChunkInfo& ci, int W) {
  const long long cid = blockIdx.x;
  const int H = W - 1;
  ci.slot = -1;
  ci.has_state = 0;
  ci.hist = kHistZero;
  ci.head = 0;
  if (p.mode == kModeSingle) {
    ci.len = p.T;
    ci.x_base = 0;
    ci.o_base = 0;
    ci.c0 = cid * p.chunk;
    if (ci.c0 >= ci.len) return false;
    ci.c1 = min(ci.c0 + (long long)p.chunk, ci.len);
    ci.head = cid == 0;
    return true;
  }
  if (p.mode == kModeContext) {
    const long long Q = p.T;
    const long long cpb = (Q + p.chunk - 1) / p.chunk;
    if (cpb == 0) return false;
    const long long b = cid / cpb, j = cid % cpb;
    if (b >= p.nseq) return false;
    ci.len = Q;
    ci.x_base = b * (Q + H) + H;
    ci.o_base = b * Q;
    ci.c0 = j * p.chunk;
    ci.c1 = min(ci.c0 + (long long)p.chunk, Q);
    ci.head = j == 0;
    ci.hist = kHistX;
    return true;
  }
  if (p.mode == kModeRows) {
    if (cid >= p.nseq) return false;
    ci.len = 1;
    ci.x_base = cid;
    ci.o_base = cid;
    ci.c0 = 0;
    ci.c1 = 1;
    ci.head = 1;
    ci.hist = kHistState;
    ci.slot = cid;
    ci.has_state = 1;
    return true;
  }
  // PACKED
  SeqHit h;
  if (!block_find_chunk<4>(p.starts, p.starts_i64, p.nseq, p.T, p.chunk, cid, p.slots, p.initial, h))
    return false;
  ci.len = h.b - h.a;
  ci.x_base = h.a;
  ci.o_base = h.a;
  ci.c0 = h.j * p.chunk;
  ci.c1 = min(ci.c0 + (long long)p.chunk, ci.len);
  ci.head = h.j == 0;
  if (p.state != nullptr) {
    ci.hist = kHistState;
    long long slot = h.slot_raw;
    if (slot >= p.num_slots) {
      if (p.err != nullptr && threadIdx.x == 0 && threadIdx.y == 0 && blockIdx.y == 0) atomicOr(p.err, 1);
      slot = -1;
    }
    ci.slot = slot < 0 ? -1 : slot;
    ci.has_state = (h.init != 0 && slot >= 0) ? 1 : 0;
  }
  return true;
}

// Old slot contents of this thread's NV channels in history order:
// sr[i] = tap (H-1-i) = the input at local position -1-i. Zeros when the slot
// is not used.
template <typename T, int NV, int WT, int MAXH>
__device__ __forceinline__ void load_old_state(const FwdParams& p, const ChunkInfo& ci, int d0,
                                               bool active, int H, Pack<T, NV> (&sr)[MAXH]) {
#pragma unroll
  for (int i = 0; i < MAXH; ++i) zero(sr[i]);
  if (!active || !ci.has_state) return;
  const T* base = reinterpret_cast<const T*>(p.state) + ci.slot * p.s_slot;
  if constexpr (NV == kVec && WT > 1) {
    if (p.st_layout == kStDS) {
      // [D, H] per slot: this thread's NV*H elements are contiguous.
      constexpr int HH = WT - 1;
      Pack<T, NV> raw[HH];
#pragma unroll
      for (int q = 0; q < HH; ++q) raw[q] = ld<T, NV>(base + (long long)d0 * HH + q * NV);
#pragma unroll
      for (int h = 0; h < HH; ++h)
#pragma unroll
        for (int j = 0; j < NV; ++j) {
          const int e = j * HH + h;
          sr[HH - 1 - h].v[j] = raw[e / NV].v[e % NV];
        }
      return;
    }
  }
  if constexpr (NV == kVec) {
    if (p.st_layout == kStSD) {
      // channel stride 1: one vector per tap
#pragma unroll
      for (int i = 0; i < MAXH; ++i)
        if (i < H) sr[i] = ld<T, NV>(base + (long long)(H - 1 - i) * p.s_h + d0);
      return;
    }
  }
#pragma unroll
  for (int i = 0; i < MAXH; ++i)
    if (i < H)
#pragma unroll
      for (int j = 0; j < NV; ++j)
        sr[i].v[j] = base[(long long)(d0 + j) * p.s_d + (long long)(H - 1 - i) * p.s_h];
}

// New slot contents: tap h <- input at local position len-H+h when that is
// inside the chunk, else the old tap len+h (zero without history).
// Element copies only, so the state stays bit-exact
// (greta_vllm/triton_conv.py:102-116, greta_vllm/conv.py:61-69).
template <typename T, int NV, int WT, int MAXH>
__device__ __forceinline__ void store_new_state(const FwdParams& p, const ChunkInfo& ci, int d0,
                                                int H, const Pack<T, NV> (&sr)[MAXH]) {
  const T* xg = reinterpret_cast<const T*>(p.x);
  Pack<T, NV> nv[MAXH];
#pragma unroll
  for (int h = 0; h < MAXH; ++h) {
    zero(nv[h]);
    if (h < H) {
      const long long q = ci.len - H + h;
      if (q >= 0)
        nv[h] = ld<T, NV>(xg + (ci.x_base + q) * p.D + d0);
      else
        nv[h] = sel(sr, (int)(H - 1 - ci.len - h));
    }
  }
  T* base = reinterpret_cast<T*>(p.state) + ci.slot * p.s_slot;
  if constexpr (NV == kVec && WT > 1) {
    if (p.st_layout == kStDS) {
      constexpr int HH = WT - 1;
      Pack<T, NV> raw[HH];
#pragma unroll
      for (int h = 0; h < HH; ++h)
#pragma unroll
        for (int j = 0; j < NV; ++j) {
          const int e = j * HH + h;
          raw[e / NV].v[e % NV] = nv[h].v[j];
        }
#pragma unroll
      for (int q = 0; q < HH; ++q) st<T, NV>(base + (long long)d0 * HH + q * NV, raw[q]);
      return;
    }
  }
  if constexpr (NV == kVec) {
    if (p.st_layout == kStSD) {
#pragma unroll
      for (int h = 0; h < MAXH; ++h)
        if (h < H) st<T, NV>(base + (long long)h * p.s_h + d0, nv[h]);
      return;
    }
  }
#pragma unroll
  for (int h = 0; h < MAXH; ++h)
    if (h < H)
#pragma unroll
      for (int j = 0; j < NV; ++j) base[(long long)(d0 + j) * p.s_d + (long long)h * p.s_h] = nv[h].v[j];
}

template <typename T, int NV, int WT, int NORM, int GV>
__global__ void __launch_bounds__(256) dynconv_fwd_kernel(const FwdParams p) {
  constexpr int MAXW = WT > 0 ? WT : -WT;
  constexpr int MAXH = MAXW > 1 ? MAXW - 1 : 1;
  constexpr int GC = NV / GV;
  constexpr int U = 1;
  const int W = WT > 0 ? WT : p.W;
  const int H = W - 1;
  const int D = p.D;
  const int G = p.G;
  const long long DC = D / G;

  ChunkInfo ci;
  if (!resolve_fwd_chunk(p, ci, W)) return;

  const int d0 = (blockIdx.y * blockDim.x + threadIdx.x) * NV;
  const bool active = d0 < D;
  const int lpg = (GV == 1 && G > NV) ? G / NV : 1;
  const long long f0 = d0 / G;
  const long long rs = ci.c0 + (long long)threadIdx.y * p.L;
  const long long re = min(rs + (long long)p.L, ci.c1);

  const T* __restrict__ xg = reinterpret_cast<const T*>(p.x);
  const T* __restrict__ wg = reinterpret_cast<const T*>(p.w);
  const T* __restrict__ gg = reinterpret_cast<const T*>(p.g);
  T* __restrict__ yg = reinterpret_cast<T*>(p.y);
  T* __restrict__ yrg = reinterpret_cast<T*>(p.yr);

  Pack<T, NV> hw[MAXH];  // hw[i] = input at (current position - 1 - i)
  if (ci.hist == kHistState && ci.head && threadIdx.y == 0) {
    Pack<T, NV> sr[MAXH];
    load_old_state<T, NV, WT, MAXH>(p, ci, d0, active, H, sr);
    if (ci.slot >= 0 && active) store_new_state<T, NV, WT, MAXH>(p, ci, d0, H, sr);
#pragma unroll
    for (int i = 0; i < MAXH; ++i) hw[i] = sr[i];
  } else {
#pragma unroll
    for (int i = 0; i < MAXH; ++i) {
      zero(hw[i]);
      if (i < H && active) {
        const long long q = rs - 1 - i;
        if (q >= 0 || ci.hist == kHistX) hw[i] = ld<T, NV>(xg + (ci.x_base + q) * D + d0);
      }
    }
  }

  for (long long t0 = rs; t0 < re; t0 += U) {
    Pack<T, NV> xr[U], gr[U];
    Pack<T, GV> wr[U][MAXW];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      zero(xr[u]);
      zero(gr[u]);
#pragma unroll
      for (int i = 0; i < MAXW; ++i) zero(wr[u][i]);
      const long long t = t0 + u;
      if (t < re && active) {
        xr[u] = ld<T, NV>(xg + (ci.x_base + t) * D + d0);
        const T* wrow = wg + (ci.o_base + t) * W * DC + f0;
#pragma unroll
        for (int i = 0; i < MAXW; ++i)
          if (i < W) wr[u][i] = ld<T, GV>(wrow + (long long)(W - 1 - i) * DC);
        if (gg != nullptr) gr[u] = ld<T, NV>(gg + (ci.o_base + t) * D + d0);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const long long t = t0 + u;
      if (t < re) {  // uniform across the warp
        float acc[NV];
#pragma unroll
        for (int c = 0; c < NV; ++c) acc[c] = 0.f;
        // taps oldest first: i = distance into the past
#pragma unroll
        for (int i = MAXW - 1; i >= 0; --i) {
          if (i < W) {
            if (i == 0) {
#pragma unroll
              for (int c = 0; c < NV; ++c) acc[c] = fmaf(to_f(xr[u].v[c]), to_f(wr[u][0].v[c / GC]), acc[c]);
            } else {
#pragma unroll
              for (int c = 0; c < NV; ++c)
                acc[c] = fmaf(to_f(hw[i > 0 ? i - 1 : 0].v[c]), to_f(wr[u][i].v[c / GC]), acc[c]);
            }
          }
        }
        const long long orow = (ci.o_base + t) * D + d0;
        if (NORM != kNormNone) {
          if (yrg != nullptr && active) {
            Pack<T, NV> o;
#pragma unroll
            for (int c = 0; c < NV; ++c) o.v[c] = from_f<T>(acc[c]);
            st<T, NV>(yrg + orow, o);
          }
          apply_norm<NORM, NV, GV>(acc, G, lpg, p.eps);
        }
        if (gg != nullptr) {
#pragma unroll
          for (int c = 0; c < NV; ++c) {
            const float gf = to_f(gr[u].v[c]);
            acc[c] = acc[c] * (gf * sigmoidf_(gf));
          }
        }
        if (active) {
          Pack<T, NV> o;
#pragma unroll
          for (int c = 0; c < NV; ++c) o.v[c] = from_f<T>(acc[c]);
          st<T, NV>(yg + orow, o);
        }
#pragma unroll
        for (int i = MAXH - 1; i > 0; --i) hw[i] = hw[i - 1];
        hw[0] = xr[u];
      }
    }
  }
}

}  // namespace greta
