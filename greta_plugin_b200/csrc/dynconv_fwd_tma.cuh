// Forward of the dynamic convolution over long token streams (training
// forward, HF inference from context, vLLM chunked prefill): row streaming
// through the Tensor Memory Accelerator.
//
// Each persistent CTA (one per SM) owns a contiguous range of tokens and a
// slice of dcta channels: all D channels when D fits one CTA
// (fwd_rows_max_channels), else the channels are split over nsplit CTAs that
// stream the same range. Its producer warp streams the range in stages of BT
// token rows -- x rows, filter rows and gate rows are contiguous in memory, so
// a stage is a few large cp.async.bulk copies (kilobytes each), completion
// counted on the stage's "full" mbarrier. Its dcta/8 consumer threads each own
// 8 channels for the whole range: they keep the last W-1 inputs in registers
// across stages, read the token's operands from shared memory, compute the
// fp32 conv + group norm + gate and store y directly. Consumer warps arrive on
// the stage's "empty" mbarrier when done; the producer refills a stage only
// after that.
//
// Sequences: a range boundary that would fall inside the first W-1 tokens of
// a request is moved to the end of them, so every token whose history
// reaches before its request's start lies in the CTA that holds the request's
// first token (its head CTA). With cache-slot state (vLLM prefill) only the
// head CTA reads the old taps (plain loads at the request's first token) and
// it alone writes the new taps: from its register window at the request's
// last token when the request ends in its range, else right after reading the
// old taps, from the request's last W-1 inputs (then all taps come from the
// chunk). Empty requests are dealt round-robin to CTAs (a slot without
// history is cleared). So no slot is read after it is written.
//
// Every mbarrier wait is bounded; on a timeout the kernel records
// kErrTimeout in the device error word and returns.
#pragma once

#include "dynconv_tma_common.cuh"

namespace greta {

struct RowsParams {
  const void* x;
  const void* w;
  const void* g;
  void* y;
  void* yr;
  const void* starts;
  int starts_i64;
  int mode;        // kModeSingle, kModePacked, kModeContext
  long long nseq;  // sequences (PACKED) or batch rows (CONTEXT)
  long long T;     // tokens (SINGLE / PACKED) or Q (CONTEXT)
  long long U;     // tokens of the launch (T, or nseq * Q for CONTEXT)
  int D, W, G;
  int log2g;          // G = 1 << log2g
  long long nominal;  // tokens per range before boundary moves: U / ranges ...
  int nom_rem;        // ... plus one for the first U % ranges ranges
  int pf_rows;        // rows of the range prefetched into L2 at the start (>= 1)
  int dcta;    // channels per CTA (a multiple of 256 dividing D)
  int nsplit;  // D / dcta: CTAs per token range
  int wsplit;  // 1: stage only the CTA's filters (per tap), 0: whole filter rows
  int BT;      // token rows per stage
  int stages;  // ring depth (<= kMaxStages)
  // cache-slot state (PACKED only)
  void* state;
  long long s_slot, s_d, s_h, num_slots;
  int st_layout;
  const int* slots;
  const signed char* initial;
  int* err;  // slot-range error bits (may be null)
  float eps;
  // row strides (elements) of x and gate rows (D when contiguous) and of the
  // filter rows (W * D/G when contiguous); y and yr are contiguous [U, D]
  long long ldx, ldg, ldw;
  int wait_log2;  // pipeline wait bound: 2^wait_log2 polls (0 = default)
  int withhold;   // test hook: consumer warp 0 of CTA 0 keeps its first stage
  // shared-memory layout (bytes from the dynamic base): sequence offsets
  // [nseq + 1] (int64), request slots [nseq] (int32) and flags [nseq] (int8),
  // then the stages
  int off_bnd, off_meta, off_stage, stage_bytes, so_w, so_g;
};

// ---------------------------------------------------------------------------
// ranges
// ---------------------------------------------------------------------------
// Nominal start of range r (before boundary moves), relative to the first
// covered token: ranges of U / ranges tokens, the first U % ranges of them one
// longer (no division on the device).
__device__ __forceinline__ long long nominal_start(const RowsParams& p, int r) {
  return (long long)r * p.nominal + min(r, p.nom_rem);
}

// Move a range boundary out of the first W-1 tokens of a request, to the
// nearer of the request's start and its (W-1)-th token. The requests cover
// tokens [ulo, uhi). The result is non-decreasing in v, so ranges stay
// ordered and disjoint.
__device__ __forceinline__ long long adjust_boundary(const RowsParams& p, const long long* bnd, long long v, int H,
                                                     long long uhi) {
  if (v >= uhi) return uhi;
  if (p.mode == kModeContext || H == 0) return v;
  long long a = 0, b = uhi;
  if (p.mode == kModePacked) {
    // the non-empty request containing v: the last s with bnd[s] <= v among
    // the requests [0, nseq) has bnd[s + 1] > v
    const long long s = seq_of(bnd, p.nseq, v);
    a = bnd[s];
    b = bnd[s + 1];
  }
  const long long local = v - a;
  if (local > 0 && local < H) v = 2 * local <= H ? a : min(a + H, b);
  return v;
}

// Old taps of this thread's channels, history order (o[i] = input at -1-i).
template <typename T, int NV, int WT, int MAXH>
__device__ __forceinline__ void rows_old_taps(const RowsParams& p, long long slot, int d0, int H,
                                              Pack<T, NV> (&o)[MAXH]) {
  const T* base = reinterpret_cast<const T*>(p.state) + slot * p.s_slot;
  if constexpr (WT > 1) {
    if (p.st_layout == kStDS) {
      constexpr int HH = WT - 1;
      Pack<T, NV> raw[HH];
#pragma unroll
      for (int q = 0; q < HH; ++q) raw[q] = ld<T, NV>(base + (long long)d0 * HH + q * NV);
#pragma unroll
      for (int h = 0; h < HH; ++h)
#pragma unroll
        for (int j = 0; j < NV; ++j) {
          const int e = j * HH + h;
          o[HH - 1 - h].v[j] = raw[e / NV].v[e % NV];
        }
      return;
    }
  }
  if (p.st_layout == kStSD) {
#pragma unroll
    for (int i = 0; i < MAXH; ++i)
      if (i < H) o[i] = ld<T, NV>(base + (long long)(H - 1 - i) * p.s_h + d0);
    return;
  }
#pragma unroll
  for (int i = 0; i < MAXH; ++i)
    if (i < H)
#pragma unroll
      for (int j = 0; j < NV; ++j) o[i].v[j] = base[(long long)(d0 + j) * p.s_d + (long long)(H - 1 - i) * p.s_h];
}

// Write new taps (tap order: taps[h] = tap h) of this thread's channels.
template <typename T, int NV, int WT, int MAXH>
__device__ __forceinline__ void rows_store_taps(const RowsParams& p, long long slot, int d0, int H,
                                                const Pack<T, NV> (&taps)[MAXH]) {
  T* base = reinterpret_cast<T*>(p.state) + slot * p.s_slot;
  if constexpr (WT > 1) {
    if (p.st_layout == kStDS) {
      constexpr int HH = WT - 1;
      Pack<T, NV> raw[HH];
#pragma unroll
      for (int h = 0; h < HH; ++h)
#pragma unroll
        for (int j = 0; j < NV; ++j) {
          const int e = j * HH + h;
          raw[e / NV].v[e % NV] = taps[h].v[j];
        }
#pragma unroll
      for (int q = 0; q < HH; ++q) st<T, NV>(base + (long long)d0 * HH + q * NV, raw[q]);
      return;
    }
  }
  if (p.st_layout == kStSD) {
#pragma unroll
    for (int h = 0; h < MAXH; ++h)
      if (h < H) st<T, NV>(base + (long long)h * p.s_h + d0, taps[h]);
    return;
  }
#pragma unroll
  for (int h = 0; h < MAXH; ++h)
    if (h < H)
#pragma unroll
      for (int j = 0; j < NV; ++j) base[(long long)(d0 + j) * p.s_d + (long long)h * p.s_h] = taps[h].v[j];
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
template <typename T, int WT, int NORM, int GV>
__global__ void __launch_bounds__(32 + fwd_rows_max_channels(WT) / kVec, 1)
    dynconv_fwd_rows_kernel(const RowsParams p) {
  constexpr int NV = kVec;
  constexpr int MAXW = WT > 0 ? WT : -WT;
  constexpr int MAXH = MAXW > 1 ? MAXW - 1 : 1;
  constexpr int GC = NV / GV;
  constexpr int ES = (int)sizeof(T);
  using PX = Pack<T, NV>;
  using PW = Pack<T, GV>;
  // Two tokens per iteration where the CTA has registers to spare (narrow
  // CTAs of wide filters, whose norm and gate work makes them latency bound).
  constexpr bool kPairTokens = fwd_rows_max_channels(WT) <= 2048 && MAXW <= 8;
  const int W = WT > 0 ? WT : p.W;
  const int H = W - 1;
  const int D = p.D;
  const int G = p.G;
  const long long DC = D >> p.log2g;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nconsw = (int)(blockDim.x >> 5) - 1;  // consumer warps
  const int S = p.stages;
  const unsigned wlimit = wait_limit(p.wait_log2);

  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ __align__(8) unsigned long long bars[2 * kMaxStages];
  const unsigned full0 = smem_addr(&bars[0]), empty0 = smem_addr(&bars[kMaxStages]);
  long long* bnd = reinterpret_cast<long long*>(smem + p.off_bnd);

  const int range = (int)blockIdx.x / p.nsplit, nranges = (int)gridDim.x / p.nsplit;
  const int c0 = ((int)blockIdx.x % p.nsplit) * p.dcta;
  const bool has_state = p.state != nullptr;
  int* sslot = reinterpret_cast<int*>(smem + p.off_meta);  // per-request slot and initial flag (PACKED + state)
  signed char* sinit = reinterpret_cast<signed char*>(smem + p.off_meta + 4 * p.nseq);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, nconsw);
    }
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  if (warp == 0 && lane >= 8 && lane < 12 && p.mode != kModeContext) {
    // Start HBM on this CTA's rows before anything else, even before the
    // kernel ahead in the stream has finished (a prefetch returns no data,
    // and L2 stays coherent with that kernel's writes): bulk L2 prefetch of
    // the first pf_rows rows of its nominal range (the range when the
    // requests cover all tokens; boundary moves shift it by < W-1 rows), and
    // a touch of its first output row. The staged copies then hit L2, so the
    // stage ring refills at L2 latency while HBM streams continuously.
    const long long u = min(nominal_start(p, range), p.U - 1);
    const unsigned n = (unsigned)min((long long)p.pf_rows, p.U - u);
    const T* xs = reinterpret_cast<const T*>(p.x) + u * p.ldx;
    const T* gs = p.g != nullptr ? reinterpret_cast<const T*>(p.g) + u * p.ldg : nullptr;
    if (lane == 8 || (lane == 10 && gs != nullptr)) {
      const T* base = lane == 8 ? xs : gs;
      const long long ld = lane == 8 ? p.ldx : p.ldg;
      if (p.nsplit == 1 && ld == D) {
        bulk_prefetch_l2(base, n * (unsigned)(D * ES));
      } else {
        for (unsigned j = 0; j < n; ++j) bulk_prefetch_l2(base + (long long)j * ld + c0, (unsigned)(p.dcta * ES));
      }
    } else if (lane == 9) {
      const T* wb = reinterpret_cast<const T*>(p.w) + u * p.ldw;
      if (p.ldw == W * DC) {
        bulk_prefetch_l2(wb, n * (unsigned)(W * DC * ES));
      } else {
        for (unsigned j = 0; j < n; ++j) bulk_prefetch_l2(wb + (long long)j * p.ldw, (unsigned)(W * DC * ES));
      }
    } else if (lane == 11) {
      prefetch_l2(reinterpret_cast<const T*>(p.y) + u * D + c0);
    }
  }
  if (warp == 0 && lane >= 12 && p.mode == kModePacked) {
    // the request metadata, read by every CTA right after the wait
    const int i = lane - 12, n = 20;
    prefetch_l2_span(p.starts, (p.nseq + 1) << (p.starts_i64 ? 3 : 2), i, n);
    if (has_state) {
      prefetch_l2_span(p.slots, p.nseq * 4, i, n);
      prefetch_l2_span(p.initial, p.nseq, i, n);
    }
  }
  const T* __restrict__ xg = reinterpret_cast<const T*>(p.x);
  const T* __restrict__ wg = reinterpret_cast<const T*>(p.w);
  const T* __restrict__ gg = reinterpret_cast<const T*>(p.g);
  const long long xrow_b = p.mode == kModeContext ? p.T + H : 0;  // context rows per batch row
  // staged row sizes (bytes): a channel slice of x / gate, and the filters
  // (the slice's per tap, or whole rows)
  const int fct = p.dcta >> p.log2g;  // filters of the slice
  const unsigned rowx = (unsigned)(p.dcta * ES);
  const unsigned roww = p.wsplit ? (unsigned)(W * fct * ES) : (unsigned)(W * DC * ES);
  const unsigned sb0 = smem_addr(smem + p.off_stage);
  // one copy for a stage's rows of a tensor when they are whole, contiguous
  // rows; else a copy per row
  const bool xwhole = p.nsplit == 1 && p.ldx == D;
  const bool gwhole = p.nsplit == 1 && p.ldg == D;
  const bool wwhole = p.ldw == W * DC;

  // Stage copies of tokens [t0, t0 + n) into the stage at shared address sb,
  // completing on mbarrier bar: x rows (not in CONTEXT mode, whose rows the
  // producer addresses per batch row), filters and gate rows.
  auto issue_x = [&](long long t0, int n, unsigned sb, unsigned bar) {
    if (xwhole) {
      bulk_g2s(sb, xg + t0 * D, (unsigned)n * rowx, bar);
    } else {
      for (int j = 0; j < n; ++j) bulk_g2s(sb + j * rowx, xg + (t0 + j) * p.ldx + c0, rowx, bar);
    }
  };
  auto issue_wg = [&](long long t0, int n, unsigned sb, unsigned bar) {
    if (p.wsplit) {
      const unsigned tapb = (unsigned)(fct * ES);
      const long long fc0 = c0 >> p.log2g;
      for (int j = 0; j < n; ++j)
        for (int k = 0; k < W; ++k)
          bulk_g2s(sb + p.so_w + j * roww + k * tapb, wg + (t0 + j) * p.ldw + k * DC + fc0, tapb, bar);
    } else if (wwhole) {
      bulk_g2s(sb + p.so_w, wg + t0 * W * DC, (unsigned)n * roww, bar);
    } else {
      for (int j = 0; j < n; ++j) bulk_g2s(sb + p.so_w + j * roww, wg + (t0 + j) * p.ldw, roww, bar);
    }
    if (gg != nullptr) {
      if (gwhole) {
        bulk_g2s(sb + p.so_g, gg + t0 * D, (unsigned)n * rowx, bar);
      } else {
        for (int j = 0; j < n; ++j) bulk_g2s(sb + p.so_g + j * rowx, gg + (t0 + j) * p.ldg + c0, rowx, bar);
      }
    }
  };

  pdl_wait();
  pdl_trigger();

  // Speculative history: when the requests start at token 0, the range most
  // likely starts at its nominal boundary u_spec inside a request, whose W-1
  // previous input rows a consumer thread needs first. They are loaded here,
  // before the sequence offsets arrive, and used if the guess was right.
  const long long u_spec = nominal_start(p, range);
  Pack<T, NV> hspec[MAXH];
#pragma unroll
  for (int i = 0; i < MAXH; ++i) zero(hspec[i]);
  if (threadIdx.x >= 32 && p.mode != kModeContext && u_spec >= H && u_spec <= p.U) {
    const T* xs = reinterpret_cast<const T*>(p.x) + c0 + ((int)threadIdx.x - 32) * NV;
#pragma unroll
    for (int i = 0; i < MAXH; ++i)
      if (i < H) hspec[i] = ld<T, NV>(xs + (u_spec - 1 - i) * p.ldx);
  }

  if (p.mode == kModePacked) {
    // sequence offsets, and with a state the requests' slots and flags, all
    // loaded at once (the slots do not depend on the offsets)
    int dec = 0;  // this thread saw a decreasing offset
    for (long long i = threadIdx.x; i <= p.nseq; i += blockDim.x) {
      const long long v = clampll(load_idx(p.starts, i, p.starts_i64), 0, p.T);
      bnd[i] = v;
      if (i > 0 && v < clampll(load_idx(p.starts, i - 1, p.starts_i64), 0, p.T)) dec = 1;
      if (has_state && i < p.nseq) {
        sslot[i] = p.slots[i];
        sinit[i] = p.initial[i];
      }
    }
    monotone_offsets(bnd, p.nseq, __syncthreads_or(dec));
  } else {
    __syncthreads();
  }

  // this CTA's channel slice [c0, c0 + dcta) and token range inside the
  // covered tokens [ulo, uhi)
  const long long ulo = p.mode == kModePacked ? bnd[0] : 0;
  const long long uhi = p.mode == kModePacked ? bnd[p.nseq] : p.U;
  const long long u0 = adjust_boundary(p, bnd, ulo + nominal_start(p, range), H, uhi);
  const long long u1 = adjust_boundary(p, bnd, ulo + nominal_start(p, range + 1), H, uhi);
  // CONTEXT: batch row and position of token u0 (token counts fit 32 bits)
  const int q0 = p.mode == kModeContext ? (int)((unsigned)u0 % (unsigned)p.T) : 0;
  const long long b0 = p.mode == kModeContext ? (long long)((unsigned)u0 / (unsigned)p.T) : 0;

  if (warp == 0) {
    // =========================== producer ===========================
    if (lane != 0) return;
    int s = 0;
    unsigned par = 0;  // parity of the stage's current use
    long long cb = b0;  // CONTEXT: batch row and position of the next token
    int cq = q0;
    int i = 0;
    for (long long t0 = u0; t0 < u1; t0 += p.BT, ++i) {
      if (i >= S && !mbar_wait(empty0 + 8 * s, par ^ 1u, wlimit)) {
        atomicOr(&g_tma_errors, kErrTimeout);
        return;
      }
      const int n = (int)min((long long)p.BT, u1 - t0);
      const unsigned bar = full0 + 8 * s;
      const unsigned sb = sb0 + (unsigned)(s * p.stage_bytes);
      if (++s == S) {
        s = 0;
        par ^= 1u;
      }
      mbar_arrive_expect_tx(bar, (unsigned)n * (rowx + roww + (gg != nullptr ? rowx : 0u)));
      if (p.mode == kModeContext) {
        for (int j = 0; j < n; ++j) {
          bulk_g2s(sb + j * rowx, xg + (cb * xrow_b + H + cq) * p.ldx + c0, rowx, bar);
          if (++cq == (int)p.T) {
            cq = 0;
            ++cb;
          }
        }
      } else {
        issue_x(t0, n, sb, bar);
      }
      issue_wg(t0, n, sb, bar);
    }
    return;
  }

  // =========================== consumers ===========================
  const int cidx = (int)threadIdx.x - 32;
  const int d0 = c0 + cidx * NV;  // first channel of this thread
  // this thread's operands in a stage: channel offset in the slice rows, and
  // filter offset / tap stride (elements) in the staged filter rows
  const int xoff = cidx * NV * ES;
  const int woff = (p.wsplit ? (d0 - c0) >> p.log2g : d0 >> p.log2g) * ES;
  const int wtap = p.wsplit ? fct : (int)DC;
  const int lpg = (GV == 1 && G > NV) ? G / NV : 1;
  T* __restrict__ yg = reinterpret_cast<T*>(p.y);
  T* __restrict__ yrg = reinterpret_cast<T*>(p.yr);

  // empty requests, dealt round-robin: a slot without history is cleared
  if (has_state)
    for (long long s = range; s < p.nseq; s += nranges)
      if (bnd[s + 1] == bnd[s]) {
        long long sl = sslot[s];
        if (sl >= p.num_slots) {
          if (p.err != nullptr && d0 == 0) atomicOr(p.err, 1);
          sl = -1;
        }
        if (sl >= 0 && sinit[s] == 0) {
          PX z[MAXH];
#pragma unroll
          for (int h = 0; h < MAXH; ++h) zero(z[h]);
          rows_store_taps<T, NV, WT, MAXH>(p, sl, d0, H, z);
        }
      }

  // request bookkeeping (PACKED / SINGLE): current request [ra, rb)
  long long sq = 0, ra = 0, rb = uhi;
  long long slot = -1;
  bool head_here = false;  // the current request's first token is in this CTA
  PX hw[MAXH];             // hw[i] = input at (current token - 1 - i)
#pragma unroll
  for (int i = 0; i < MAXH; ++i) zero(hw[i]);

  auto find_request = [&](long long u) {
    if (p.mode == kModePacked) {
      sq = seq_of(bnd, p.nseq, u);
      ra = bnd[sq];
      rb = bnd[sq + 1];
    }
  };

  // First token of a request: history = old taps (or zeros).
  auto begin_request = [&]() {
    head_here = true;
    slot = -1;
#pragma unroll
    for (int i = 0; i < MAXH; ++i) zero(hw[i]);
    if (!has_state) return;
    long long sl = sslot[sq];
    if (sl >= p.num_slots) {
      if (p.err != nullptr && d0 == 0) atomicOr(p.err, 1);
      sl = -1;
    }
    slot = sl < 0 ? -1 : sl;
    if (slot >= 0 && sinit[sq] != 0) rows_old_taps<T, NV, WT, MAXH>(p, slot, d0, H, hw);
    if (slot >= 0 && rb > u1) {
      // the request continues past this CTA: its new taps are its last W-1
      // inputs (it has more than W-1 tokens), written now, after the old
      // taps were read
      PX taps[MAXH];
#pragma unroll
      for (int h = 0; h < MAXH; ++h) {
        zero(taps[h]);
        if (h < H) taps[h] = ld<T, NV>(xg + (rb - H + h) * p.ldx + d0);
      }
      rows_store_taps<T, NV, WT, MAXH>(p, slot, d0, H, taps);
      slot = -1;  // written
    }
  };

  if (u0 < u1) {
    if (p.mode == kModeContext) {
#pragma unroll
      for (int i = 0; i < MAXH; ++i)
        if (i < H) hw[i] = ld<T, NV>(xg + (b0 * xrow_b + H + q0 - 1 - i) * p.ldx + d0);
    } else {
      find_request(u0);
      if (u0 == ra) {
        begin_request();
      } else if (u0 == u_spec) {
        // mid-request start at the nominal boundary: the rows loaded before
        // the prologue barrier are the history
#pragma unroll
        for (int i = 0; i < MAXH; ++i) hw[i] = hspec[i];
      } else {
        // mid-request start: the boundary rule guarantees u0 - ra >= W-1
#pragma unroll
        for (int i = 0; i < MAXH; ++i)
          if (i < H) hw[i] = ld<T, NV>(xg + (u0 - 1 - i) * p.ldx + d0);
      }
    }
  }

  // The history window stays in the I/O type: the taps multiply with
  // fma_io (for 16-bit types sm_100's mixed-precision FMA), so no input or
  // filter element is converted, and the slot write-back is a bit copy.
  int koff[MAXW];  // byte offset of the filter of the input k steps back
#pragma unroll
  for (int k = 0; k < MAXW; ++k) koff[k] = (k < W ? (W - 1 - k) : 0) * wtap * ES;
  T* yp = yg + u0 * D + d0;
  T* yrp = yrg != nullptr ? yrg + u0 * D + d0 : nullptr;
  int s = 0;
  unsigned par = 0;
  long long cb = b0;  // CONTEXT: batch row and position of the current token
  int cq = q0;
  for (long long t0 = u0; t0 < u1; t0 += p.BT) {
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
    const int n = (int)min((long long)p.BT, u1 - t0);
    const unsigned char* xsp = stg + xoff;
    const unsigned char* wsp = stg + p.so_w + woff;
    const unsigned char* gsp = stg + p.so_g + xoff;
    for (int j = 0; j < n;) {
      const long long u = t0 + j;
      if (p.mode == kModeContext) {
        if (u != u0 && cq == 0) {  // a new batch row: its history is its context
#pragma unroll
          for (int k = 0; k < MAXH; ++k)
            if (k < H) hw[k] = ld<T, NV>(xg + (cb * xrow_b + H - 1 - k) * p.ldx + d0);
        }
        if (++cq == (int)p.T) {  // position of the next token
          cq = 0;
          ++cb;
        }
      } else if (u >= rb) {
        find_request(u);  // skips empty requests
        begin_request();
      }
      const PX xc = *reinterpret_cast<const PX*>(xsp);
      PW wc[MAXW];
#pragma unroll
      for (int k = 0; k < MAXW; ++k) {
        zero(wc[k]);
        if (k < W) wc[k] = *reinterpret_cast<const PW*>(wsp + koff[k]);
      }
      float acc[NV];
#pragma unroll
      for (int c = 0; c < NV; ++c) acc[c] = 0.f;
#pragma unroll
      for (int k = MAXW - 1; k >= 0; --k) {
        if (k < W) {
          const PX& xs = (k == 0) ? xc : hw[k > 0 ? k - 1 : 0];
#pragma unroll
          for (int c = 0; c < NV; ++c) acc[c] = fma_io(xs.v[c], wc[k].v[c / GC], acc[c]);
        }
      }
      if (kPairTokens && p.mode != kModeContext && j + 1 < n && u + 1 < rb) {
        // Token u+1 of the same request alongside token u, so that the two
        // tokens' norm reductions and gates overlap. Its taps, oldest first
        // as for a single token: the window shifted by one, then x[u], x[u+1].
        const PX xn = *reinterpret_cast<const PX*>(xsp + rowx);
#pragma unroll
        for (int k = 0; k < MAXW; ++k) {
          zero(wc[k]);
          if (k < W) wc[k] = *reinterpret_cast<const PW*>(wsp + roww + koff[k]);
        }
        float acn[NV];
#pragma unroll
        for (int c = 0; c < NV; ++c) acn[c] = 0.f;
#pragma unroll
        for (int k = MAXW - 1; k >= 0; --k) {
          if (k < W) {
            const PX& xs = (k == 0) ? xn : (k == 1 ? xc : hw[k > 1 ? k - 2 : 0]);
#pragma unroll
            for (int c = 0; c < NV; ++c) acn[c] = fma_io(xs.v[c], wc[k].v[c / GC], acn[c]);
          }
        }
        if (NORM != kNormNone) {
          if (yrp != nullptr) {
            PX o, q;
#pragma unroll
            for (int c = 0; c < NV; ++c) {
              o.v[c] = from_f<T>(acc[c]);
              q.v[c] = from_f<T>(acn[c]);
            }
            st<T, NV>(yrp, o);
            st<T, NV>(yrp + D, q);
            yrp += 2 * D;
          }
          apply_norm2<NORM, NV, GV>(acc, acn, G, lpg, p.eps);
        }
        if (gg != nullptr) {
          const PX gv = *reinterpret_cast<const PX*>(gsp);
          const PX gw = *reinterpret_cast<const PX*>(gsp + rowx);
          float gf[NV], gn[NV];
#pragma unroll
          for (int c = 0; c < NV; ++c) {
            gf[c] = to_f(gv.v[c]);
            gn[c] = to_f(gw.v[c]);
          }
          gate_pairs<NV>(acc, gf);
          gate_pairs<NV>(acn, gn);
        }
        {
          PX o, q;
#pragma unroll
          for (int c = 0; c < NV; ++c) {
            o.v[c] = from_f<T>(acc[c]);
            q.v[c] = from_f<T>(acn[c]);
          }
          st<T, NV>(yp, o);
          st<T, NV>(yp + D, q);
        }
#pragma unroll
        for (int k = MAXH - 1; k > 1; --k) hw[k] = hw[k - 2];
        if (MAXH > 1) hw[1] = xc;
        hw[0] = xn;
        if (has_state && head_here && slot >= 0 && u + 1 == rb - 1) {
          PX taps[MAXH];
#pragma unroll
          for (int h = 0; h < MAXH; ++h) taps[h] = sel(hw, H - 1 - h);
          rows_store_taps<T, NV, WT, MAXH>(p, slot, d0, H, taps);
          slot = -1;
        }
        j += 2;
        xsp += 2 * rowx;
        wsp += 2 * roww;
        gsp += 2 * rowx;
        yp += 2 * D;
        continue;
      }
      if (NORM != kNormNone) {
        if (yrp != nullptr) {
          PX o;
#pragma unroll
          for (int c = 0; c < NV; ++c) o.v[c] = from_f<T>(acc[c]);
          st<T, NV>(yrp, o);
          yrp += D;
        }
        apply_norm<NORM, NV, GV>(acc, G, lpg, p.eps);
      }
      if (gg != nullptr) {
        const PX gv = *reinterpret_cast<const PX*>(gsp);
        float gf[NV];
#pragma unroll
        for (int c = 0; c < NV; ++c) gf[c] = to_f(gv.v[c]);
        gate_pairs<NV>(acc, gf);
      }
      {
        PX o;
#pragma unroll
        for (int c = 0; c < NV; ++c) o.v[c] = from_f<T>(acc[c]);
        st<T, NV>(yp, o);
      }
#pragma unroll
      for (int k = MAXH - 1; k > 0; --k) hw[k] = hw[k - 1];
      hw[0] = xc;
      if (has_state && head_here && slot >= 0 && u == rb - 1) {
        // the request ends here: the window holds the input at rb-1-k (old
        // taps for positions before ra), so the new tap h is window[H-1-h]
        PX taps[MAXH];
#pragma unroll
        for (int h = 0; h < MAXH; ++h) taps[h] = sel(hw, H - 1 - h);
        rows_store_taps<T, NV, WT, MAXH>(p, slot, d0, H, taps);
        slot = -1;
      }
      ++j;
      xsp += rowx;
      wsp += roww;
      gsp += rowx;
      yp += D;
    }
    __syncwarp();
    // (test hook: consumer warp 0 of CTA 0 keeps the first stage it used, so
    // the producer's refill of it waits until its bound runs out)
    const bool keep = p.withhold != 0 && blockIdx.x == 0 && warp == 1 && t0 == u0;
    if (lane == 0 && !keep) mbar_arrive(empty0 + 8 * cur_s);
  }
}

}  // namespace greta
