// Forward of decode-like vLLM packed batches: one or a few tokens per request
// (greta_vllm/triton_conv.py:28-116 on a batch whose decodes come first,
// greta_vllm/conv.py:84-94 and greta_vllm/model.py:155-161), with the
// cache-slot history and the state write-back fused.
//
// A decode step moves ~100 KB per request in a handful of 16-byte accesses
// per thread, so its time is latency: the request metadata, then the slot's
// old taps, then the stores. This kernel is the register-window forward cut
// down for that case:
//   - CTA row r < num_reqs is request r's first chunk of C tokens; its
//     offsets, slot and flag are direct loads, issued together with the
//     operands of token r (the request's first token when every earlier
//     request has one token, as in a decode batch), so x, w and the gate
//     arrive with the metadata instead of one round trip later.
//   - Rows after num_reqs are later chunks of longer requests, found by the
//     block-wide scan (C >= W-1, so their history is chunk rows, never the
//     slot).
//   - No next-token prefetch: the thread's registers are the window, one
//     token's operands and the accumulators, which keeps it under 64
//     registers so that a 256-request step fits one wave of the GPU.
//   - The slot's old taps stay in the layout they were loaded in (DS: the
//     thread's 8 channels x W-1 taps as one contiguous run; SD: one vector
//     per tap), and a one-token request -- every request of a decode step --
//     convolves them and builds the new taps straight from those registers.
// The slot rules are those of dynconv_fwd_kernel (dynconv_fwd.cuh): the head
// thread of a request alone reads the old taps and writes the new ones, and
// the arithmetic (fp32 sums, taps oldest first) is the same, so both kernels
// give identical bits. W is 4 or 7 (Greta's kernel size) and the state is DS
// or SD; other shapes use dynconv_fwd_kernel.
//
// The same kernel serves the HF single-token decode (FwdParams::mode ROWS):
// batch row r is one token whose history is state row r (DS), shifted in
// place -- no request metadata at all.
#pragma once

#include "dynconv_fwd.cuh"

namespace greta {

// CTAs of 128 threads per SM the register budget is set for: 8 (64 registers
// a thread) for 16-bit types and W = 4, 6 for W = 7, half as many for fp32.
template <typename T>
constexpr int decode_min_ctas(int w) {
  return (w <= 4 ? 8 : 6) / (sizeof(T) == 2 ? 1 : 2);
}

// Slot registers: DS = the slot's [8 channels x HH taps] run as HH packs
// (element c*HH + h is channel c, tap h); SD = one pack per tap.
template <bool DS, typename T, int NV, int HH>
__device__ __forceinline__ T slot_elem(const Pack<T, NV> (&sv)[HH], int c, int h) {
  if constexpr (DS) {
    return sv[(c * HH + h) / NV].v[(c * HH + h) % NV];
  } else {
    return sv[h].v[c];
  }
}

template <bool DS, typename T, int NV, int HH>
__device__ __forceinline__ void set_slot_elem(Pack<T, NV> (&sv)[HH], int c, int h, T v) {
  if constexpr (DS) {
    sv[(c * HH + h) / NV].v[(c * HH + h) % NV] = v;
  } else {
    sv[h].v[c] = v;
  }
}

template <bool DS, typename T, int NV, int HH>
__device__ __forceinline__ void load_slot(const FwdParams& p, long long slot, int d0, Pack<T, NV> (&sv)[HH]) {
  const T* base = reinterpret_cast<const T*>(p.state) + slot * p.s_slot;
#pragma unroll
  for (int q = 0; q < HH; ++q)
    sv[q] = ld<T, NV>(DS ? base + (long long)d0 * HH + q * NV : base + (long long)q * p.s_h + d0);
}

template <bool DS, typename T, int NV, int HH>
__device__ __forceinline__ void store_slot(const FwdParams& p, long long slot, int d0, const Pack<T, NV> (&sv)[HH]) {
  T* base = reinterpret_cast<T*>(p.state) + slot * p.s_slot;
#pragma unroll
  for (int q = 0; q < HH; ++q)
    st<T, NV>(DS ? base + (long long)d0 * HH + q * NV : base + (long long)q * p.s_h + d0, sv[q]);
}

// y of one token: taps oldest first, the W-1 older inputs from old(c, k)
// (tap k), then the current input; norm and gate; stored to row `orow`.
template <typename T, int NV, int GV, int W, int NORM, typename Old>
__device__ __forceinline__ void decode_token(const FwdParams& p, const TokenLoads<T, NV, GV, W>& tok, Old old,
                                             T* yrow, bool active, int lpg) {
  constexpr int GC = NV / GV;
  float acc[NV];
#pragma unroll
  for (int c = 0; c < NV; ++c) {
    float a = 0.f;
#pragma unroll
    for (int k = 0; k < W - 1; ++k) a = fma_io(old(c, k), tok.w[W - 1 - k].v[c / GC], a);
    acc[c] = fma_io(tok.x.v[c], tok.w[0].v[c / GC], a);
  }
  if (NORM != kNormNone) apply_norm<NORM, NV, GV>(acc, p.G, lpg, p.eps);
  if (p.g != nullptr) {
    float gf[NV];
#pragma unroll
    for (int c = 0; c < NV; ++c) gf[c] = to_f(tok.g.v[c]);
    gate_pairs<NV>(acc, gf);
  }
  if (active) {
    Pack<T, NV> o;
#pragma unroll
    for (int c = 0; c < NV; ++c) o.v[c] = from_f<T>(acc[c]);
    st<T, NV>(yrow, o);
  }
}

template <bool DS, bool ROWS, typename T, int W, int NORM, int GV>
__device__ __forceinline__ void decode_run(const FwdParams& p, long long row) {
  constexpr int NV = kVec;
  constexpr int H = W - 1;
  using PX = Pack<T, NV>;
  const int D = p.D;
  const long long DC = D / p.G;
  const int d0 = ((int)(blockIdx.x % p.nblk) * blockDim.x + threadIdx.x) * NV;
  const bool active = d0 < D;
  const long long f0 = d0 / p.G;
  const int lpg = (GV == 1 && p.G > NV) ? p.G / NV : 1;
  const T* __restrict__ xg = reinterpret_cast<const T*>(p.x);
  const T* __restrict__ wg = reinterpret_cast<const T*>(p.w);
  const T* __restrict__ gg = reinterpret_cast<const T*>(p.g);
  T* __restrict__ yg = reinterpret_cast<T*>(p.y);

  // the chunk: tokens [c0, c1) of the request [a, a + len); token counts and
  // slots fit 32 bits (checked on the host)
  int a = 0, len = 0, c0 = 0, c1 = 0;
  bool head = false;
  int slot = -1;
  bool has_old = false;
  TokenLoads<T, NV, GV, W> tok;  // operands of the token being convolved
  bool spec = false;             // tok already holds the request's first token
  if constexpr (ROWS) {
    // HF decode: batch row r is one token with history in state row r,
    // shifted in place (greta/dynamic_conv.py:513-602); no metadata
    if (row >= p.nseq) return;
    const int r = (int)row;
    load_token(tok, xg, wg, gg, r, r, p, W, DC, f0, d0, active);
    a = r;
    len = 1;
    c1 = 1;
    head = true;
    spec = true;
    slot = r;
    has_old = true;
  } else if (row < p.nseq) {
    const int r = (int)row;
    // speculative operands of token r, independent of the metadata
    if (r < p.T) load_token(tok, xg, wg, gg, r, r, p, W, DC, f0, d0, active);
    a = (int)clampll(load_idx(p.starts, r, p.starts_i64), 0, p.T);
    int b = (int)clampll(load_idx(p.starts, r + 1, p.starts_i64), 0, p.T);
    const int slot_raw = p.slots != nullptr ? p.slots[r] : -1;
    const int init = p.initial != nullptr ? (int)p.initial[r] : 0;
    if (b < a) b = a;
    spec = r < p.T && a == r;
    len = b - a;
    c1 = min(p.chunk, len);
    head = true;
    if (p.state != nullptr) {
      if (slot_raw >= p.num_slots && p.err != nullptr && threadIdx.x == 0 && blockIdx.x % p.nblk == 0)
        atomicOr(p.err, 1);
      slot = (slot_raw < 0 || slot_raw >= p.num_slots) ? -1 : slot_raw;
      has_old = init != 0 && slot >= 0;
    }
  } else {
    SeqHit h;
    if (!block_find_chunk<1>(p.starts, p.starts_i64, p.nseq, p.T, p.chunk, row - p.nseq, p.slots, p.initial, h,
                             1))
      return;
    a = (int)h.a;
    len = (int)(h.b - h.a);
    c0 = (int)h.j * p.chunk;
    c1 = min(c0 + p.chunk, len);
  }
  const bool write_back = head && slot >= 0 && active;

  PX sv[H];  // old slot contents in the layout's order (zeros without history)
#pragma unroll
  for (int q = 0; q < H; ++q) zero(sv[q]);
  if (head && has_old && active) load_slot<DS, T, NV, H>(p, slot, d0, sv);

  if (head && spec && len == 1) {
    // one-token request (decode): convolve the old taps in place, then the
    // new taps are (old taps 1 .. W-2, x)
    decode_token<T, NV, GV, W, NORM>(p, tok, [&](int c, int k) { return slot_elem<DS>(sv, c, k); },
                                     yg + (long long)a * D + d0, active, lpg);
    if (write_back) {
      PX nv[H];
#pragma unroll
      for (int c = 0; c < NV; ++c) {
#pragma unroll
        for (int h = 0; h < H - 1; ++h) set_slot_elem<DS>(nv, c, h, slot_elem<DS>(sv, c, h + 1));
        set_slot_elem<DS>(nv, c, H - 1, tok.x.v[c]);
      }
      store_slot<DS, T, NV, H>(p, slot, d0, nv);
    }
    return;
  }

  // general chunk: a register window hw[i] = input at (position - 1 - i)
  PX hw[H];
  if (head) {
#pragma unroll
    for (int i = 0; i < H; ++i)
#pragma unroll
      for (int c = 0; c < NV; ++c) hw[i].v[c] = slot_elem<DS>(sv, c, H - 1 - i);
  } else {
    // a later chunk: c0 >= C >= W-1, so the history is rows of the request
#pragma unroll
    for (int i = 0; i < H; ++i) {
      zero(hw[i]);
      if (active) hw[i] = ld<T, NV>(xg + (long long)(a + c0 - 1 - i) * p.ldx + d0);
    }
  }
  for (int t = c0; t < c1; ++t) {
    if (!(spec && t == 0)) load_token(tok, xg, wg, gg, a + t, a + t, p, W, DC, f0, d0, active);
    decode_token<T, NV, GV, W, NORM>(p, tok, [&](int c, int k) { return hw[H - 1 - k].v[c]; },
                                     yg + (long long)(a + t) * D + d0, active, lpg);
#pragma unroll
    for (int i = H - 1; i > 0; --i) hw[i] = hw[i - 1];
    hw[0] = tok.x;
  }
  if (write_back) {
    // new tap h: from the window when the whole request is in this chunk
    // (hw[i] = input at len-1-i, old taps for negative positions), else the
    // request's last W-1 inputs (len > C >= W-1; the old taps were read above)
    PX nv[H];
    if (len <= c1) {
#pragma unroll
      for (int h = 0; h < H; ++h)
#pragma unroll
        for (int c = 0; c < NV; ++c) set_slot_elem<DS>(nv, c, h, hw[H - 1 - h].v[c]);
    } else {
#pragma unroll
      for (int h = 0; h < H; ++h) {
        const PX v = ld<T, NV>(xg + (long long)(a + len - H + h) * p.ldx + d0);
#pragma unroll
        for (int c = 0; c < NV; ++c) set_slot_elem<DS>(nv, c, h, v.v[c]);
      }
    }
    store_slot<DS, T, NV, H>(p, slot, d0, nv);
  }
}

// ROWS: the HF decode (FwdParams::mode ROWS), a separate instantiation so
// that the packed kernel's register allocation is its own.
template <typename T, int W, int NORM, int GV, bool ROWS>
__global__ void __launch_bounds__(128, decode_min_ctas<T>(W)) dynconv_fwd_decode_kernel(const FwdParams p) {
  const long long row = blockIdx.x / p.nblk;
  if (ROWS && row < p.nseq) {
    // the row's operands, ahead of the wait (see below)
    const int d0 = ((int)(blockIdx.x % p.nblk) * blockDim.x + threadIdx.x) * kVec;
    if (d0 < p.D) {
      prefetch_l2(reinterpret_cast<const T*>(p.x) + row * p.ldx + d0);
      if (p.g != nullptr) prefetch_l2(reinterpret_cast<const T*>(p.g) + row * p.ldg + d0);
      const long long DC = p.D / p.G;
      const T* wr = reinterpret_cast<const T*>(p.w) + row * p.ldw + d0 / p.G;
#pragma unroll
      for (int k = 0; k < W; ++k) prefetch_l2(wr + k * DC);
    }
  } else if (!ROWS && row < p.nseq) {
    // While the kernel ahead in the stream finishes: bring the request's
    // metadata and the speculative first token's operands into L2, so that
    // the loads after the wait are L2 hits.
    const int d0 = ((int)(blockIdx.x % p.nblk) * blockDim.x + threadIdx.x) * kVec;
    if (threadIdx.x == 0) {
      prefetch_l2(reinterpret_cast<const char*>(p.starts) + (row << (p.starts_i64 ? 3 : 2)));
      if (p.slots != nullptr) prefetch_l2(p.slots + row);
      if (p.initial != nullptr) prefetch_l2(p.initial + row);
    }
    if (row < p.T && d0 < p.D) {
      const T* xr = reinterpret_cast<const T*>(p.x) + row * p.ldx;
      prefetch_l2(xr + d0);
      if (p.g != nullptr) prefetch_l2(reinterpret_cast<const T*>(p.g) + row * p.ldg + d0);
      const long long DC = p.D / p.G;
      const T* wr = reinterpret_cast<const T*>(p.w) + row * p.ldw + d0 / p.G;
#pragma unroll
      for (int k = 0; k < W; ++k) prefetch_l2(wr + k * DC);
    }
  }
  pdl_wait();
  pdl_trigger();
  if (p.st_layout == kStSD)
    decode_run<false, ROWS, T, W, NORM, GV>(p, row);
  else
    decode_run<true, ROWS, T, W, NORM, GV>(p, row);
}

}  // namespace greta
