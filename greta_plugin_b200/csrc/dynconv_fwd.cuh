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
// Per thread: NV channels x a run of L tokens walked in time order, with the
// last W-1 inputs in registers; see dynconv_fwd_kernel below.
#pragma once

#include "dynconv_common.cuh"

namespace greta {

__device__ __forceinline__ bool resolve_fwd_chunk(const FwdParams& p, ChunkInfo& ci, int W) {
  const long long cid = blockIdx.x / p.nblk;
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
  // PACKED: CTA row cid < nseq is the first chunk of request cid (its offsets,
  // slot and flag are independent loads: no search); the rows after them are
  // the requests' later chunks, found by a block-wide scan.
  SeqHit h;
  if (cid < p.nseq) {
    h.s = cid;
    h.j = 0;
    h.a = clampll(load_idx(p.starts, cid, p.starts_i64), 0, p.T);
    h.b = clampll(load_idx(p.starts, cid + 1, p.starts_i64), 0, p.T);
    if (h.b < h.a) h.b = h.a;
    h.slot_raw = p.slots != nullptr ? p.slots[cid] : -1;
    h.init = p.initial != nullptr ? (int)p.initial[cid] : 0;
  } else if (!block_find_chunk<4>(p.starts, p.starts_i64, p.nseq, p.T, p.chunk, cid - p.nseq, p.slots, p.initial,
                                  h, 1)) {
    return false;
  }
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
      if (p.err != nullptr && threadIdx.x == 0 && threadIdx.y == 0 && blockIdx.x % p.nblk == 0) atomicOr(p.err, 1);
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

// Write the new slot contents, given in tap order (taps[h] = tap h). The
// values are input elements copied as they are, so the state stays bit-exact
// (greta_vllm/triton_conv.py:102-116, greta_vllm/conv.py:61-69).
template <typename T, int NV, int WT, int MAXH>
__device__ __forceinline__ void store_state_taps(const FwdParams& p, const ChunkInfo& ci, int d0, int H,
                                                 const Pack<T, NV> (&taps)[MAXH]) {
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
          raw[e / NV].v[e % NV] = taps[h].v[j];
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
        if (h < H) st<T, NV>(base + (long long)h * p.s_h + d0, taps[h]);
      return;
    }
  }
#pragma unroll
  for (int h = 0; h < MAXH; ++h)
    if (h < H)
#pragma unroll
      for (int j = 0; j < NV; ++j) base[(long long)(d0 + j) * p.s_d + (long long)h * p.s_h] = taps[h].v[j];
}

// One token's operands: the input vector, the W filter taps (reversed:
// w[i] = tap W-1-i, the filter of the input i steps in the past) and the gate.
template <typename T, int NV, int GV, int MAXW>
struct TokenLoads {
  Pack<T, NV> x, g;
  Pack<T, GV> w[MAXW];
};

template <typename T, int NV, int GV, int MAXW>
__device__ __forceinline__ void load_token(TokenLoads<T, NV, GV, MAXW>& o, const T* __restrict__ xg,
                                           const T* __restrict__ wg, const T* __restrict__ gg, long long xrow,
                                           long long orow, const FwdParams& p, int W, long long DC, long long f0,
                                           int d0, bool active) {
  zero(o.x);
  zero(o.g);
#pragma unroll
  for (int i = 0; i < MAXW; ++i) zero(o.w[i]);
  if (!active) return;
  o.x = ld<T, NV>(xg + xrow * p.ldx + d0);
  const T* wrow = wg + orow * p.ldw + f0;
#pragma unroll
  for (int i = 0; i < MAXW; ++i)
    if (i < W) o.w[i] = ld<T, GV>(wrow + (long long)(W - 1 - i) * DC);
  if (gg != nullptr) o.g = ld<T, NV>(gg + orow * p.ldg + d0);
}

// A thread owns NV channels x a run of L consecutive tokens [rs, re) of one
// sequence and walks it in time order: the last W-1 inputs stay in registers
// (each x row is read once, plus a W-1 row halo per run), and the loads of
// token t+1 are issued before the arithmetic of token t.
//
// Cache-slot state: per request and channel vector, ONE thread (row 0 of the
// request's first chunk) touches the slot. It loads the old taps into its
// history window before anything else, and writes the new taps either from
// its final window (the whole request is in its run: decode, short chunks;
// the window then still holds old taps for requests shorter than W-1) or
// from the request's last W-1 inputs loaded up front (longer requests; all
// new taps then come from the chunk). No other thread reads the slot, so no
// barrier is needed.
//
// CTAs are numbered channel block fastest (blockIdx.x = chunk * nblk + block).
template <typename T, int NV, int WT, int NORM, int GV>
__global__ void __launch_bounds__(256) dynconv_fwd_kernel(const FwdParams p) {
  constexpr int MAXW = WT > 0 ? WT : -WT;
  constexpr int MAXH = MAXW > 1 ? MAXW - 1 : 1;
  constexpr int GC = NV / GV;
  const int W = WT > 0 ? WT : p.W;
  const int H = W - 1;
  const int D = p.D;
  const int G = p.G;
  const long long DC = D / G;

  pdl_wait();
  pdl_trigger();
  ChunkInfo ci;
  if (!resolve_fwd_chunk(p, ci, W)) return;

  const int d0 = ((int)(blockIdx.x % p.nblk) * blockDim.x + threadIdx.x) * NV;
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

  // first token's operands: independent of the state, issued first
  TokenLoads<T, NV, GV, MAXW> nxt;
  if (rs < re) load_token(nxt, xg, wg, gg, ci.x_base + rs, ci.o_base + rs, p, W, DC, f0, d0, active);

  const bool state_head = ci.hist == kHistState && ci.head && threadIdx.y == 0;
  const bool write_back = state_head && ci.slot >= 0 && active;
  const bool wb_window = ci.len <= re;  // the whole request is in this thread's run

  Pack<T, NV> hw[MAXH];  // hw[i] = input at (current position - 1 - i)
  if (state_head) {
    Pack<T, NV> tail[MAXH];
    if (write_back && !wb_window) {
      // the request's last W-1 inputs (len > L >= W-1, so all are chunk rows)
#pragma unroll
      for (int h = 0; h < MAXH; ++h) {
        zero(tail[h]);
        if (h < H) tail[h] = ld<T, NV>(xg + (ci.x_base + ci.len - H + h) * p.ldx + d0);
      }
    }
    load_old_state<T, NV, WT, MAXH>(p, ci, d0, active, H, hw);
    if (write_back && !wb_window) store_state_taps<T, NV, WT, MAXH>(p, ci, d0, H, tail);
  } else {
    // only a thread with tokens loads history: the run of a thread past the
    // end of its chunk (rs >= re) may lie past the end of the request, and
    // for the last request past the end of x
#pragma unroll
    for (int i = 0; i < MAXH; ++i) {
      zero(hw[i]);
      if (i < H && active && rs < re) {
        const long long q = rs - 1 - i;
        if (q >= 0 || ci.hist == kHistX) hw[i] = ld<T, NV>(xg + (ci.x_base + q) * p.ldx + d0);
      }
    }
  }

  for (long long t = rs; t < re; ++t) {
    const TokenLoads<T, NV, GV, MAXW> cur = nxt;
    if (t + 1 < re) load_token(nxt, xg, wg, gg, ci.x_base + t + 1, ci.o_base + t + 1, p, W, DC, f0, d0, active);
    float acc[NV];
#pragma unroll
    for (int c = 0; c < NV; ++c) acc[c] = 0.f;
    // taps oldest first: i = distance into the past
#pragma unroll
    for (int i = MAXW - 1; i >= 0; --i) {
      if (i < W) {
        const Pack<T, NV>& xs = (i == 0) ? cur.x : hw[i > 0 ? i - 1 : 0];
#pragma unroll
        for (int c = 0; c < NV; ++c) acc[c] = fma_io(xs.v[c], cur.w[i].v[c / GC], acc[c]);
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
        const float gf = to_f(cur.g.v[c]);
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
    hw[0] = cur.x;
  }

  if (write_back && wb_window) {
    // hw[i] now holds the value at position len-1-i (old taps for negative
    // positions), so the new tap h is hw[H-1-h]
    Pack<T, NV> taps[MAXH];
#pragma unroll
    for (int h = 0; h < MAXH; ++h) taps[h] = sel(hw, H - 1 - h);
    store_state_taps<T, NV, WT, MAXH>(p, ci, d0, H, taps);
  }
}

}  // namespace greta
