// Backward of the packed training convolution: dx, compact dw and dg in one
// pass (greta/dynamic_conv.py:271-428 dynconv_bwd_kernel).
//
//   dn[t]    = dout[t] * silu(g[t])                       (or dout without gate)
//   dy[t]    = rinv * (dn - n * mean_G(n * dn)),  n = yr * rinv   (norm)   else dn
//   dx[t]    = sum_i dy[t+i] * w[t+i, W-1-i]               (within the sequence)
//   dw[t,k,f]= sum_{d in f} dy[t,d] * x[t+k-W+1, d]
//   dg[t]    = dout * hat * sig * (1 + g * (1 - sig)),  hat = n (norm) or conv(x,w)
//
// A thread owns NV channels x a run [rs, re) of tokens and walks t = rs ..
// re+W-2 in time order. x history stays in registers (for dw and the conv
// recompute); dx is formed by scattering dy[t] into W-1 pending register
// accumulators, so a dx row is complete W-1 steps after its token. The last
// W-1 steps are the run's right halo: dy is recomputed there (dout, g, yr, w
// rows of the next run, normally L2 hits) and only dx is stored.
#pragma once

#include "dynconv_common.cuh"

namespace greta {

__device__ __forceinline__ bool resolve_bwd_chunk(const BwdParams& p, ChunkInfo& ci) {
  const long long cid = blockIdx.x / p.nblk;
  ci.slot = -1;
  ci.has_state = 0;
  ci.hist = kHistZero;
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
  SeqHit h;
  if (!block_find_chunk<4>(p.starts, p.starts_i64, p.nseq, p.T, p.chunk, cid, nullptr, nullptr, h))
    return false;
  ci.len = h.b - h.a;
  ci.x_base = h.a;
  ci.o_base = h.a;
  ci.c0 = h.j * p.chunk;
  ci.c1 = min(ci.c0 + (long long)p.chunk, ci.len);
  ci.head = h.j == 0;
  return true;
}

template <typename T, int NV, int WT, int NORM, int GV>
__global__ void __launch_bounds__(256) dynconv_bwd_kernel(const BwdParams p) {
  constexpr int MAXW = WT > 0 ? WT : -WT;
  constexpr int MAXH = MAXW > 1 ? MAXW - 1 : 1;
  constexpr int GC = NV / GV;
  const int W = WT > 0 ? WT : p.W;
  const int H = W - 1;
  const int D = p.D;
  const int G = p.G;
  const long long DC = D / G;
  const float inv_g = 1.f / (float)G;

  pdl_wait();
  pdl_trigger();
  ChunkInfo ci;
  if (!resolve_bwd_chunk(p, ci)) return;

  const int d0 = ((int)(blockIdx.x % p.nblk) * blockDim.x + threadIdx.x) * NV;
  const bool active = d0 < D;
  const int lpg = (GV == 1 && G > NV) ? G / NV : 1;
  const bool dw_writer = active && (GV > 1 || (threadIdx.x & (lpg - 1)) == 0);
  const long long f0 = d0 / G;
  const long long rs = ci.c0 + (long long)threadIdx.y * p.L;
  const long long re = min(rs + (long long)p.L, ci.c1);
  if (rs >= re) return;  // whole warp: same threadIdx.y

  const T* __restrict__ xg = reinterpret_cast<const T*>(p.x);
  const T* __restrict__ wg = reinterpret_cast<const T*>(p.w);
  const T* __restrict__ gg = reinterpret_cast<const T*>(p.g);
  const T* __restrict__ yrg = reinterpret_cast<const T*>(p.yr);
  const T* __restrict__ dog = reinterpret_cast<const T*>(p.dout);
  T* __restrict__ dxg = reinterpret_cast<T*>(p.dx);
  T* __restrict__ dwg = reinterpret_cast<T*>(p.dw);
  T* __restrict__ dgg = reinterpret_cast<T*>(p.dg);

  Pack<T, NV> hw[MAXH];
#pragma unroll
  for (int i = 0; i < MAXH; ++i) {
    zero(hw[i]);
    if (i < H && active) {
      const long long q = rs - 1 - i;
      if (q >= 0) hw[i] = ld<T, NV>(xg + (ci.x_base + q) * p.ldx + d0);
    }
  }
  float pend[MAXH][NV];  // pend[j] = partial dx of token (t - 1 - j)
#pragma unroll
  for (int j = 0; j < MAXH; ++j)
#pragma unroll
    for (int c = 0; c < NV; ++c) pend[j][c] = 0.f;

  const long long tend = re + H;
  for (long long t = rs; t < tend; ++t) {
    const bool own = t < re;
    const bool live = t < ci.len;  // dy is zero past the end of the sequence
    const long long orow = (ci.o_base + t) * D + d0;  // dout and yr (contiguous)
    const long long trow = ci.o_base + t;
    Pack<T, NV> xr, dor, gr, yrr;
    Pack<T, GV> wr[MAXW];  // wr[i] = w[t, W-1-i]
    zero(xr);
    zero(dor);
    zero(gr);
    zero(yrr);
#pragma unroll
    for (int i = 0; i < MAXW; ++i) zero(wr[i]);
    if (live && active) {
      if (own) xr = ld<T, NV>(xg + (ci.x_base + t) * p.ldx + d0);
      dor = ld<T, NV>(dog + orow);
      if (gg != nullptr) gr = ld<T, NV>(gg + trow * p.ldg + d0);
      if (NORM != kNormNone) yrr = ld<T, NV>(yrg + orow);
      const T* wrow = wg + trow * p.ldw + f0;
#pragma unroll
      for (int i = 0; i < MAXW; ++i)
        if (i < W) wr[i] = ld<T, GV>(wrow + (long long)(W - 1 - i) * DC);
    }

    // dy = d(out)/d(pre-norm conv). Gate and norm terms are recomputed from
    // the packed inputs where dg needs them again, to keep registers low.
    float dy[NV], rinv[GV];
#pragma unroll
    for (int c = 0; c < NV; ++c) dy[c] = 0.f;
#pragma unroll
    for (int gi = 0; gi < GV; ++gi) rinv[gi] = 0.f;
    if (live) {  // uniform across the warp
      {
        float dv[NV], gf[NV];
#pragma unroll
        for (int c = 0; c < NV; ++c) {
          dv[c] = to_f(dor.v[c]);
          gf[c] = to_f(gr.v[c]);
        }
        if (gg != nullptr) {
          bwd_gate_dy<NV>(dv, gf, dy);
        } else {
#pragma unroll
          for (int c = 0; c < NV; ++c) dy[c] = dv[c];
        }
      }
      if (NORM == kNormPlain) {
        float yf[NV];
#pragma unroll
        for (int c = 0; c < NV; ++c) yf[c] = to_f(yrr.v[c]);
        bwd_norm<NV, GV>(yf, dy, rinv, inv_g, p.eps, lpg);
      }
    }

    if (own) {
      // dw[t, k, f] for k = W-1-i; x at distance i
      float yc[NV];
#pragma unroll
      for (int c = 0; c < NV; ++c) yc[c] = 0.f;
#pragma unroll
      for (int i = MAXW - 1; i >= 0; --i) {
        if (i < W) {
          const Pack<T, NV>& xs = (i == 0) ? xr : hw[i > 0 ? i - 1 : 0];
          float xf[NV], s[GV];
#pragma unroll
          for (int c = 0; c < NV; ++c) {
            xf[c] = to_f(xs.v[c]);
            if (NORM == kNormNone && gg != nullptr) yc[c] = fma_io(xs.v[c], wr[i].v[c / GC], yc[c]);
          }
          // the thread's part of the group sum, then the butterfly over its lanes
          group_local_dot<NV, GV>(dy, xf, s);
          if (GV == 1) group_xlane_sum(s[0], lpg);
          if (dw_writer) {
            Pack<T, GV> o;
#pragma unroll
            for (int gi = 0; gi < GV; ++gi) o.v[gi] = from_f<T>(s[gi]);
            st<T, GV>(dwg + trow * p.lddw + (long long)(W - 1 - i) * DC + f0, o);
          }
        }
      }
      if (gg != nullptr && active) {
        float dv[NV], gf[NV], hat[NV], dgv[NV];
#pragma unroll
        for (int c = 0; c < NV; ++c) {
          dv[c] = to_f(dor.v[c]);
          gf[c] = to_f(gr.v[c]);
          hat[c] = (NORM == kNormNone) ? yc[c] : to_f(yrr.v[c]);
        }
        if (NORM != kNormNone) scale_pairs<NV, GV>(hat, rinv);  // the normed output yr * rinv
        bwd_gate_dg<NV>(dv, gf, hat, dgv);
        Pack<T, NV> o;
#pragma unroll
        for (int c = 0; c < NV; ++c) o.v[c] = from_f<T>(dgv[c]);
        st<T, NV>(dgg + trow * p.lddg + d0, o);
      }
    }

    // dx: scatter dy[t] into the pending rows t-1 .. t-H, complete row t-H.
    float done[NV];
    if (H == 0) {
#pragma unroll
      for (int c = 0; c < NV; ++c) done[c] = __fmul_rn(dy[c], to_f(wr[0].v[c / GC]));
    } else {
#pragma unroll
      for (int j = 0; j < MAXH; ++j)
        if (j < H)
#pragma unroll
          for (int c = 0; c < NV; ++c)
            pend[j][c] = fmaf(dy[c], to_f(wr[j + 1 < MAXW ? j + 1 : 0].v[c / GC]), pend[j][c]);
#pragma unroll
      for (int c = 0; c < NV; ++c) {
        float v = pend[0][c];
#pragma unroll
        for (int j = 1; j < MAXH; ++j)
          if (j == H - 1) v = pend[j][c];
        done[c] = v;
      }
#pragma unroll
      for (int j = MAXH - 1; j > 0; --j)
#pragma unroll
        for (int c = 0; c < NV; ++c) pend[j][c] = pend[j - 1][c];
#pragma unroll
      for (int c = 0; c < NV; ++c) pend[0][c] = __fmul_rn(dy[c], to_f(wr[0].v[c / GC]));
    }
    const long long tc = t - H;
    if (tc >= rs && tc < re && active) {
      Pack<T, NV> o;
#pragma unroll
      for (int c = 0; c < NV; ++c) o.v[c] = from_f<T>(done[c]);
      st<T, NV>(dxg + (ci.x_base + tc) * p.lddx + d0, o);
    }
    if (own) {
#pragma unroll
      for (int i = MAXH - 1; i > 0; --i) hw[i] = hw[i - 1];
      hw[0] = xr;
    }
  }
}

}  // namespace greta
