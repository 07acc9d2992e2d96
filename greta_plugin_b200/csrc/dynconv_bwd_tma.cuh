// Backward of the packed training convolution over long token streams:
// row streaming through the Tensor Memory Accelerator
// (greta/dynamic_conv.py:271-428 dynconv_bwd_kernel computes the same dx, dw, dg).
//
//   dn[t]     = dout[t] * silu(g[t])                       (or dout without gate)
//   dy[t]     = rinv * (dn - n * mean_G(n * dn)),  n = yr * rinv   (norm) else dn
//   dx[t]     = sum_i dy[t+i] * w[t+i, W-1-i]               (within the sequence)
//   dw[t,k,f] = sum_{d in f} dy[t,d] * x[t+k-W+1, d]
//   dg[t]     = dout * hat * sig * (1 + g * (1 - sig)),  hat = n (norm) or conv(x,w)
//
// Each persistent CTA (one per SM) owns a contiguous token range [u0, u1)
// and a slice of dcta channels (all D when D <= bwd_rows_max_channels; else the
// channels are split over nsplit CTAs that stream the same range). Its
// producer (a warp of its own, or lane 0 of consumer warp 0) streams the
// slice's token rows of x, the filters, dout (and gate, saved pre-norm output)
// into a ring of shared-memory stages with cp.async.bulk; completion is
// counted on each stage's "full" mbarrier and consumers release a stage on its
// "empty" mbarrier. The inline producer refills the stage of tile i - 1 with
// tile i - 1 + S once it has finished tile i, so it seldom waits. Each of the
// dcta/8 consumer threads owns 8 channels for the whole range and walks it in
// time order, keeping the last W-1 inputs (for dw and the conv recompute) and
// W-1 partial dx rows in registers: dy[t] is scattered into the pending rows,
// so the dx row of token t-(W-1) is complete at token t. dw and dg of token t
// are complete at token t and stored at once.
//
// The range is followed by a right halo of up to W-1 tokens of the request of
// its last token, streamed like the others: there only dy is formed, to
// finish the dx rows of the range's last W-1 tokens. At the end of a request
// the pending rows are complete and stored. The first W-1 inputs before the
// range (a range that starts inside a request) are plain loads.
//
// The arithmetic and its order are those of dynconv_bwd_kernel (the
// register-staged backward), so both give bit-identical results. Every
// mbarrier wait is bounded; on a timeout the kernel records kErrTimeout in the
// device error word and returns.
#pragma once

#include "dynconv_tma_common.cuh"

namespace greta {

// Widest filter of the row-streaming backward, and the most channels per CTA
// for a filter-width template WT (exact W > 0, or -MAXW) and GV filter groups
// per thread. W-1 pending dx rows and W-1 inputs of a thread's 8 channels stay
// in registers: ~160 registers per thread at W = 4, ~210 at W = 7 with one
// group per thread, up to 255 for the others. A scheduler (a quarter of the
// SM's register file) holds two warps of 255 registers or three of 168, so:
//   W <= 4          32 + 2048/8 threads (a producer warp + 8 consumer warps)
//   W = 7, GV = 1   2048/8 threads, no producer warp: consumer warp 0 issues
//                   the copies (bwd_rows_inline_producer)
//   otherwise       32 + 1024/8 threads
// A lone warp per scheduler leaves the long dependent chains of the wide
// filters exposed; two hide much of them.
constexpr int kMaxWBwdRows = 8;
__host__ __device__ constexpr bool bwd_rows_inline_producer(int wt, int gv) { return wt == 7 && gv == 1; }
__host__ __device__ constexpr int bwd_rows_max_channels(int wt, int gv) {
  return ((wt < 0 ? -wt : wt) <= 4 || bwd_rows_inline_producer(wt, gv)) ? 2048 : 1024;
}
__host__ __device__ constexpr int bwd_rows_threads(int wt, int gv, int dcta) {
  return (bwd_rows_inline_producer(wt, gv) ? 0 : 32) + dcta / kVec;
}

struct BwdRowsParams {
  const void* x;
  const void* w;
  const void* g;
  const void* yr;
  const void* dout;
  void* dx;
  void* dw;
  void* dg;
  const void* starts;
  int starts_i64;
  int mode;        // kModeSingle, kModePacked
  long long nseq;  // sequences (PACKED)
  long long T;     // tokens
  int D, W, G;
  int dcta;    // channels per CTA (a multiple of 256 dividing D)
  int nsplit;  // D / dcta: CTAs per token range
  int wsplit;  // 1: stage only the CTA's filters (per tap), 0: whole filter rows
  int BT;      // token rows per stage
  int stages;  // ring depth (<= kMaxStages)
  float eps;
  int wait_log2;  // pipeline wait bound: 2^wait_log2 polls (0 = default)
  // shared-memory layout (bytes from the dynamic base)
  int off_bnd, off_stage, stage_bytes, so_w, so_do, so_g, so_yr;
  // row strides (elements): inputs x, gate (D when contiguous) and filters
  // (W * D/G); outputs dx, dg and dw likewise; yr and dout are contiguous
  long long ldx, ldg, ldw, lddx, lddg, lddw;
};

template <typename T, int WT, int NORM, int GV>
__global__ void __launch_bounds__(bwd_rows_threads(WT, GV, bwd_rows_max_channels(WT, GV)), 1)
    dynconv_bwd_rows_kernel(const BwdRowsParams p) {
  constexpr bool INL = bwd_rows_inline_producer(WT, GV);
  constexpr int NV = kVec;
  constexpr int MAXW = WT > 0 ? WT : -WT;
  constexpr int MAXH = MAXW > 1 ? MAXW - 1 : 1;
  constexpr int MAXP = MAXW <= 2 ? 2 : (MAXW <= 4 ? 4 : 8);  // MAXW rounded up to a power of two
  constexpr int GC = NV / GV;
  constexpr int ES = (int)sizeof(T);
  using PX = Pack<T, NV>;
  using PW = Pack<T, GV>;
  const int W = WT > 0 ? WT : p.W;
  const int H = W - 1;
  const int D = p.D;
  const int G = p.G;
  const long long DC = D / G;
  const float inv_g = 1.f / (float)G;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nconsw = (int)(blockDim.x >> 5) - (INL ? 0 : 1);  // consumer warps
  const int S = p.stages;

  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ __align__(8) unsigned long long bars[2 * kMaxStages];
  const unsigned full0 = smem_addr(&bars[0]), empty0 = smem_addr(&bars[kMaxStages]);
  long long* bnd = reinterpret_cast<long long*>(smem + p.off_bnd);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, nconsw);
    }
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  pdl_wait();
  pdl_trigger();
  const bool packed = p.mode == kModePacked;
  if (packed)
    load_offsets(bnd, p.starts, p.starts_i64, p.nseq, p.T);
  else
    __syncthreads();

  // this CTA's channel slice [c0, c0 + dcta) and token range inside the
  // covered tokens [ulo, uhi), plus its right halo
  const int range = (int)blockIdx.x / p.nsplit, nranges = (int)gridDim.x / p.nsplit;
  const int c0 = ((int)blockIdx.x % p.nsplit) * p.dcta;
  const long long ulo = packed ? bnd[0] : 0;
  const long long uhi = packed ? bnd[p.nseq] : p.T;
  const long long nominal = (uhi - ulo + nranges - 1) / nranges;
  const long long u0 = min(ulo + (long long)range * nominal, uhi);
  const long long u1 = min(u0 + nominal, uhi);
  long long ue = u1;
  if (u1 > u0 && u1 < uhi && H > 0) {
    const long long rb_last = packed ? bnd[seq_of(bnd, p.nseq, u1 - 1) + 1] : uhi;
    ue = min(u1 + (long long)H, rb_last);
  }
  const long long ntiles = ue > u0 ? (ue - u0 + p.BT - 1) / p.BT : 0;

  const T* __restrict__ xg = reinterpret_cast<const T*>(p.x);
  const T* __restrict__ wg = reinterpret_cast<const T*>(p.w);
  const T* __restrict__ gg = reinterpret_cast<const T*>(p.g);
  const T* __restrict__ yrg = reinterpret_cast<const T*>(p.yr);
  const T* __restrict__ dog = reinterpret_cast<const T*>(p.dout);
  // staged row sizes (bytes): a channel slice of x / dout / gate / yr, and the
  // filters (the slice's per tap, or whole rows)
  const int dct = p.dcta;
  const int fct = dct / G;  // filters of the slice
  const unsigned rowx = (unsigned)(dct * ES);
  const unsigned roww = p.wsplit ? (unsigned)(W * fct * ES) : (unsigned)(W * DC * ES);

  // =========================== producer ===========================
  const unsigned per_row = 2u * rowx + roww + (gg != nullptr ? rowx : 0u) + (NORM != kNormNone ? rowx : 0u);
  // Issue tile i's copies into stage i % S (seen empty by the caller).
  auto issue = [&](long long i) {
    // n rows (row stride ld) of a [T, D] tensor's slice, starting at token t:
    // one copy when the slices are whole, contiguous rows, else one per row
    auto copy_rows = [&](unsigned dst, const T* src, long long ld, long long t, int n, unsigned bar) {
      if (p.nsplit == 1 && ld == D) {
        bulk_g2s(dst, src + t * D, (unsigned)n * rowx, bar);
      } else {
        for (int j = 0; j < n; ++j) bulk_g2s(dst + j * rowx, src + (t + j) * ld + c0, rowx, bar);
      }
    };
    const int s = (int)(i % S);
    const long long t0 = u0 + i * p.BT;
    const int n = (int)min((long long)p.BT, ue - t0);
    const unsigned bar = full0 + 8 * s;
    const unsigned sb = smem_addr(smem + p.off_stage) + (unsigned)(s * p.stage_bytes);
    mbar_arrive_expect_tx(bar, (unsigned)n * per_row);
    copy_rows(sb, xg, p.ldx, t0, n, bar);
    if (p.wsplit) {
      const unsigned tapb = (unsigned)(fct * ES);
      for (int j = 0; j < n; ++j)
        for (int k = 0; k < W; ++k)
          bulk_g2s(sb + p.so_w + j * roww + k * tapb, wg + (t0 + j) * p.ldw + k * DC + c0 / G, tapb, bar);
    } else if (p.ldw == W * DC) {
      bulk_g2s(sb + p.so_w, wg + t0 * W * DC, (unsigned)n * roww, bar);
    } else {
      for (int j = 0; j < n; ++j) bulk_g2s(sb + p.so_w + j * roww, wg + (t0 + j) * p.ldw, roww, bar);
    }
    copy_rows(sb + p.so_do, dog, D, t0, n, bar);
    if (gg != nullptr) copy_rows(sb + p.so_g, gg, p.ldg, t0, n, bar);
    if (NORM != kNormNone) copy_rows(sb + p.so_yr, yrg, D, t0, n, bar);
  };
  // bounded wait until the consumers have released the stage use of tile i
  const unsigned wlimit = wait_limit(p.wait_log2);
  auto released = [&](long long i) {
    return mbar_wait(empty0 + 8 * (int)(i % S), (unsigned)((i / S) & 1), wlimit);
  };

  if (!INL && warp == 0) {
    if (lane != 0) return;
    for (long long i = 0; i < ntiles; ++i) {
      if (i >= S && !released(i - S)) {
        atomicOr(&g_tma_errors, kErrTimeout);
        return;
      }
      issue(i);
    }
    return;
  }
  if (INL && threadIdx.x == 0)
    for (long long i = 0; i < min((long long)S, ntiles); ++i) issue(i);

  // =========================== consumers ===========================
  const int cidx = (int)threadIdx.x - (INL ? 0 : 32);
  const int d0 = c0 + cidx * NV;  // first channel of this thread
  const long long f0 = d0 / G;
  // this thread's operands in a stage: channel offset in the slice rows, and
  // filter offset / tap stride (elements) in the staged filter rows
  const int xoff = cidx * NV * ES;
  const int woff = (p.wsplit ? (d0 - c0) / G : d0 / G) * ES;
  const int wtap = p.wsplit ? fct : (int)DC;
  const int lpg = (GV == 1 && G > NV) ? G / NV : 1;
  T* __restrict__ dxg = reinterpret_cast<T*>(p.dx);
  T* __restrict__ dwg = reinterpret_cast<T*>(p.dw);
  T* __restrict__ dgg = reinterpret_cast<T*>(p.dg);

  // current request [ra, rb)
  long long ra = ulo, rb = uhi;
  auto find_request = [&](long long u) {
    if (packed) {
      const long long s = seq_of(bnd, p.nseq, u);
      ra = bnd[s];
      rb = bnd[s + 1];
    }
  };

  // The history window: hw[i] = input at (current token - 1 - i), in the I/O
  // type, or in fp32 (F32WIN: the wide-filter CTAs, whose 255-register budget
  // has room) so that each input is converted once instead of once per tap.
  constexpr bool F32WIN = INL;
  PX hw[F32WIN ? 1 : MAXH];
  float hwf[F32WIN ? MAXH : 1][NV];
  float pend[MAXH][NV];  // pend[j] = partial dx of token (current token - 1 - j)
  auto clear_window = [&]() {
#pragma unroll
    for (int i = 0; i < (F32WIN ? 1 : MAXH); ++i) zero(hw[i]);
#pragma unroll
    for (int i = 0; i < (F32WIN ? MAXH : 1); ++i)
#pragma unroll
      for (int c = 0; c < NV; ++c) hwf[i][c] = 0.f;
  };
  // the input i >= 1 steps back, channel c, in fp32
  auto past = [&](int i, int c) -> float {
    if constexpr (F32WIN) {
      return hwf[i - 1 < MAXH ? i - 1 : 0][c];
    } else {
      return to_f(hw[i - 1 < MAXH ? i - 1 : 0].v[c]);
    }
  };
  auto set_past = [&](int i, const PX& v) {
    if constexpr (F32WIN) {
#pragma unroll
      for (int c = 0; c < NV; ++c) hwf[i][c] = to_f(v.v[c]);
    } else {
      hw[i] = v;
    }
  };
  clear_window();
#pragma unroll
  for (int j = 0; j < MAXH; ++j)
#pragma unroll
    for (int c = 0; c < NV; ++c) pend[j][c] = 0.f;

  if (u0 < ue) {
    find_request(u0);
#pragma unroll
    for (int i = 0; i < MAXH; ++i)
      if (i < H && u0 - 1 - i >= ra) set_past(i, ld<T, NV>(xg + (u0 - 1 - i) * p.ldx + d0));
  }

  // Store the complete dx rows pending at the end of a request (the last
  // token processed was rb - 1): pend[j] is the row of token rb - 1 - j.
  auto flush = [&]() {
    const long long lo = max(ra, u0);
#pragma unroll
    for (int j = 0; j < MAXH; ++j) {
      const long long v = rb - 1 - j;
      if (j < H && v >= lo && v < u1) {
        PX o;
#pragma unroll
        for (int c = 0; c < NV; ++c) o.v[c] = from_f<T>(pend[j][c]);
        st<T, NV>(dxg + v * p.lddx + d0, o);
      }
    }
  };

  int koff[MAXW];  // byte offset of the filter applied to the input i steps back
#pragma unroll
  for (int i = 0; i < MAXW; ++i) koff[i] = (i < W ? (W - 1 - i) : 0) * wtap * ES;
  int s = 0;
  unsigned par = 0;
  long long t0 = u0;
  for (long long it = 0; it < ntiles; ++it, t0 += p.BT) {
    if (!mbar_wait(full0 + 8 * s, par, wlimit)) {
      if (lane == 0) atomicOr(&g_tma_errors, kErrTimeout);
      return;
    }
    const unsigned char* stg = smem + p.off_stage + s * p.stage_bytes;
    const int cur_s = s;
    if (++s == S) {
      s = 0;
      par ^= 1u;
    }
    const int n = (int)min((long long)p.BT, ue - t0);
    const unsigned char* xsp = stg + xoff;
    const unsigned char* wsp = stg + p.so_w + woff;
    const unsigned char* dsp = stg + p.so_do + xoff;
    const unsigned char* gsp = stg + p.so_g + xoff;
    const unsigned char* ysp = stg + p.so_yr + xoff;
    for (int j = 0; j < n; ++j, xsp += rowx, wsp += roww, dsp += rowx, gsp += rowx, ysp += rowx) {
      const long long u = t0 + j;
      if (u >= rb) {  // the next request starts at u: finish the last one
        flush();
        find_request(u);
        clear_window();
#pragma unroll
        for (int q = 0; q < MAXH; ++q)
#pragma unroll
          for (int c = 0; c < NV; ++c) pend[q][c] = 0.f;
      }
      const bool own = u < u1;  // else a right-halo token: dy only
      const PX xr = *reinterpret_cast<const PX*>(xsp);
      const PX dor = *reinterpret_cast<const PX*>(dsp);
      PX gr, yrr;
      zero(gr);
      zero(yrr);
      if (gg != nullptr) gr = *reinterpret_cast<const PX*>(gsp);
      if (NORM != kNormNone) yrr = *reinterpret_cast<const PX*>(ysp);
      PW wr[MAXW];  // wr[i] = w[u, W-1-i]
#pragma unroll
      for (int i = 0; i < MAXW; ++i) {
        zero(wr[i]);
        if (i < W) wr[i] = *reinterpret_cast<const PW*>(wsp + koff[i]);
      }

      float dy[NV], rinv[GV];
#pragma unroll
      for (int gi = 0; gi < GV; ++gi) rinv[gi] = 0.f;
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

      if (own) {  // uniform across the CTA
        // dw[u, k, f] for k = W-1-i: the input i steps back
        float yc[NV];
#pragma unroll
        for (int c = 0; c < NV; ++c) yc[c] = 0.f;
        T* dwrow = dwg + u * p.lddw + f0;
        // GV == 1: this thread's part of the group's dw for the input i steps
        // back, summed over the group's lanes below (GV > 1: stored at once)
        float part[MAXP];
#pragma unroll
        for (int i = MAXP - 1; i >= 0; --i) {
          part[i] = 0.f;
          if (i < W) {
            float xf[NV];
#pragma unroll
            for (int c = 0; c < NV; ++c) xf[c] = (i == 0) ? to_f(xr.v[c]) : past(i, c);
            float sm[GV];
            group_local_dot<NV, GV>(dy, xf, sm);
            if (NORM == kNormNone && gg != nullptr) {
              // the conv recompute, one rounding per tap (fmaf of the converted
              // values is the value fma_io gives on the I/O-type ones)
              const PW& wi = wr[i < MAXW ? i : 0];
              if constexpr (F32WIN) {
#pragma unroll
                for (int c = 0; c < NV; ++c) yc[c] = fmaf(xf[c], to_f(wi.v[c / GC]), yc[c]);
              } else {
                const PX& xs = (i == 0) ? xr : hw[i > 0 && i - 1 < MAXH ? i - 1 : 0];
#pragma unroll
                for (int c = 0; c < NV; ++c) yc[c] = fma_io(xs.v[c], wi.v[c / GC], yc[c]);
              }
            }
            if (GV == 1) {
              part[i] = sm[0];
            } else {
              PW o;
#pragma unroll
              for (int gi = 0; gi < GV; ++gi) o.v[gi] = from_f<T>(sm[gi]);
              st<T, GV>(dwrow + (long long)(W - 1 - i) * DC, o);
            }
          }
        }
        if (GV == 1) {  // one group over lpg lanes: reduce-scatter the W sums
          int base, cnt;
          group_sum_scatter<MAXP>(part, lpg, lane, base, cnt);
          if (lpg >= MAXP) {
            // one total per lane: the group's lanes 0 .. MAXP-1 hold taps base
            if ((cidx & (lpg - 1)) < MAXP && base < W) dwrow[(long long)(W - 1 - base) * DC] = from_f<T>(part[0]);
          } else {
#pragma unroll
            for (int j = 0; j < MAXP; ++j)
              if (j < cnt && base + j < W) dwrow[(long long)(W - 1 - base - j) * DC] = from_f<T>(part[j]);
          }
        }
        if (gg != nullptr) {
          float dv[NV], gf[NV], hat[NV], dgv[NV];
#pragma unroll
          for (int c = 0; c < NV; ++c) {
            dv[c] = to_f(dor.v[c]);
            gf[c] = to_f(gr.v[c]);
            hat[c] = (NORM == kNormNone) ? yc[c] : to_f(yrr.v[c]);
          }
          if (NORM != kNormNone) scale_pairs<NV, GV>(hat, rinv);  // the normed output yr * rinv
          bwd_gate_dg<NV>(dv, gf, hat, dgv);
          PX o;
#pragma unroll
          for (int c = 0; c < NV; ++c) o.v[c] = from_f<T>(dgv[c]);
          st<T, NV>(dgg + u * p.lddg + d0, o);
        }
      }

      // dx: scatter dy[u] into the pending rows u-1 .. u-H; row u-H is complete
      float done[NV];
      if (H == 0) {
#pragma unroll
        for (int c = 0; c < NV; ++c) done[c] = __fmul_rn(dy[c], to_f(wr[0].v[c / GC]));
      } else {
#pragma unroll
        for (int q = 0; q < MAXH; ++q)
          if (q < H) {
            const PW& wq = wr[q + 1 < MAXW ? q + 1 : 0];
#pragma unroll
            for (int c = 0; c < NV; c += 2)
              fma2(pend[q][c], pend[q][c + 1], dy[c], dy[c + 1], to_f(wq.v[c / GC]), to_f(wq.v[(c + 1) / GC]));
          }
#pragma unroll
        for (int c = 0; c < NV; ++c) {
          float v = pend[0][c];
#pragma unroll
          for (int q = 1; q < MAXH; ++q)
            if (q == H - 1) v = pend[q][c];
          done[c] = v;
        }
#pragma unroll
        for (int q = MAXH - 1; q > 0; --q)
#pragma unroll
          for (int c = 0; c < NV; ++c) pend[q][c] = pend[q - 1][c];
#pragma unroll
        for (int c = 0; c < NV; c += 2)
          mul2(pend[0][c], pend[0][c + 1], dy[c], dy[c + 1], to_f(wr[0].v[c / GC]), to_f(wr[0].v[(c + 1) / GC]));
      }
      const long long tc = u - H;
      if (tc >= max(ra, u0) && tc < u1) {
        PX o;
#pragma unroll
        for (int c = 0; c < NV; ++c) o.v[c] = from_f<T>(done[c]);
        st<T, NV>(dxg + tc * p.lddx + d0, o);
      }
      if constexpr (F32WIN) {
#pragma unroll
        for (int i = MAXH - 1; i > 0; --i)
#pragma unroll
          for (int c = 0; c < NV; ++c) hwf[i][c] = hwf[i - 1][c];
      } else {
#pragma unroll
        for (int i = MAXH - 1; i > 0; --i) hw[i] = hw[i - 1];
      }
      set_past(0, xr);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty0 + 8 * cur_s);
    if (INL && warp == 0 && it >= 1 && it - 1 + S < ntiles) {  // refill the stage of tile it - 1
      int ok = 1;
      if (lane == 0) {
        ok = released(it - 1);
        if (ok)
          issue(it - 1 + S);
        else
          atomicOr(&g_tma_errors, kErrTimeout);
      }
      if (!__shfl_sync(0xffffffffu, ok, 0)) return;
    }
  }
  if (ue > u0 && ue == rb) flush();  // the last request ended inside the range or its halo
}

}  // namespace greta
