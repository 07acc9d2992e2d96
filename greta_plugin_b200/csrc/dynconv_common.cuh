// Shared device code for the dynamic causal depthwise convolution kernels.
//
// Work decomposition (all kernels):
//   grid.x  = chunks x channel blocks, channel block fastest: a chunk is a
//             run of consecutive tokens of ONE sequence (sequence = packed
//             request, cu_seqlens segment, batch row); a channel block is
//             blockDim.x * NV channels.
//   thread  = NV consecutive channels (one 16-byte vector for 16-bit types)
//             x a run of L consecutive tokens; threadIdx.y picks the run
//             inside the chunk. A thread walks its run in time order and
//             keeps the last W-1 inputs in registers, so every x row is read
//             once from HBM (plus a W-1 row halo per run, which hits L1/L2).
//
// Sequences are resolved on the device from the cumulative offsets (no host
// chunk table, no host synchronisation): each CTA scans the per-sequence chunk
// counts with a block-wide prefix sum and finds its (sequence, chunk) pair.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace greta {

constexpr int kVec = 8;          // channels per thread on the vector path
constexpr int kMaxWGeneric = 16; // largest kernel size handled by the generic-W variant

enum NormKind { kNormNone = 0, kNormPlain = 1, kNormStable = 2 };
enum SeqMode { kModeSingle = 0, kModePacked = 1, kModeContext = 2, kModeRows = 3 };
enum HistKind { kHistZero = 0, kHistX = 1, kHistState = 2 };
enum StateLayout { kStGeneric = 0, kStDS = 1, kStSD = 2 };

// Parameters of the forward family (training fwd, HF inference, HF decode,
// vLLM packed conv + state write-back).
struct FwdParams {
  const void* x;   // [rows, D]
  const void* w;   // [out rows, W, D/G]
  const void* g;   // [out rows, D] or null
  void* y;         // [out rows, D]
  void* yr;        // [out rows, D] or null (pre-norm output)
  const void* starts;  // [nseq + 1] (PACKED) or null
  int starts_i64;
  int mode;            // SeqMode
  long long nseq;      // sequences (PACKED) or batch rows (CONTEXT / ROWS)
  long long T;         // total tokens (SINGLE / PACKED) or Q (CONTEXT)
  int D, W, G;
  int L;               // tokens per thread run
  int chunk;           // tokens per CTA = L * blockDim.y
  int nblk;            // channel blocks; blockIdx.x = chunk * nblk + channel block
  // cache-slot state
  void* state;         // null = no state
  long long s_slot, s_d, s_h, num_slots;
  int st_layout;       // StateLayout
  const int* slots;    // [nseq] or null (ROWS: slot = row)
  const signed char* initial;  // [nseq] or null
  int* err;            // device error bits or null
  float eps;
  // row strides (elements) of the inputs: x and gate rows (D when
  // contiguous), filter rows (W * D/G when contiguous); outputs are
  // contiguous [rows, D]
  long long ldx, ldg, ldw;
};

struct BwdParams {
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
  int mode;  // SINGLE or PACKED
  long long nseq;
  long long T;
  int D, W, G;
  int L;
  int chunk;
  int nblk;  // channel blocks; blockIdx.x = chunk * nblk + channel block
  float eps;
  // row strides (elements): inputs x, gate (D when contiguous) and filters
  // (W * D/G); outputs dx, dg and dw likewise; yr and dout are contiguous
  long long ldx, ldg, ldw, lddx, lddg, lddw;
};

// ---------------------------------------------------------------------------
// element packs and conversions
// ---------------------------------------------------------------------------
template <typename T, int N>
struct alignas(sizeof(T) * N) Pack {
  T v[N];
};

// Programmatic dependent launch. Every kernel here is launched with
// programmatic stream serialization, so it may start while the kernel before
// it in the stream is still running: pdl_wait() blocks until that kernel has
// completed and its writes are visible, and must come before the first access
// to global memory (an L2 prefetch, which returns no data, may precede it).
// pdl_trigger() lets the next kernel in the stream launch once every CTA of
// this grid has triggered or exited, so its launch overlaps this kernel's
// work. Both are no-ops without a dependent or a primary.
// L2 prefetch of the line holding `p` (no data returned; L2 stays coherent
// with the writes of a kernel still running ahead in the stream).
__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];\n" ::"l"(p));
}

// Lines of [p, p + bytes) prefetched into L2 by `n` cooperating threads,
// thread `i` taking every n-th 128-byte line.
__device__ __forceinline__ void prefetch_l2_span(const void* p, long long bytes, int i, int n) {
  const char* a = static_cast<const char*>(p);
  for (long long o = (long long)i * 128; o < bytes; o += (long long)n * 128) prefetch_l2(a + o);
}

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }

__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
__device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }

// a * b + c with a, b in the I/O type and c in fp32, one rounding. For 16-bit
// types this is sm_100's mixed-precision FMA (the operands widen exactly), so
// the result equals fmaf(to_f(a), to_f(b), c) without the two conversions.
__device__ __forceinline__ float fma_io(float a, float b, float c) { return fmaf(a, b, c); }
__device__ __forceinline__ float fma_io(__nv_bfloat16 a, __nv_bfloat16 b, float c) {
  float r;
  asm("fma.rn.f32.bf16 %0, %1, %2, %3;" : "=f"(r) : "h"(__bfloat16_as_ushort(a)), "h"(__bfloat16_as_ushort(b)), "f"(c));
  return r;
}
// Two fp32 lanes per instruction (sm_100's packed fp32 pipe); each lane is
// rounded exactly like fmaf / a * b.
__device__ __forceinline__ unsigned long long pack2(float a, float b) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void unpack2(unsigned long long r, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
// d[c] = a[c] * b[c] + d[c] for c = 0, 1
__device__ __forceinline__ void fma2(float& d0, float& d1, float a0, float a1, float b0, float b1) {
  unsigned long long r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(pack2(a0, a1)), "l"(pack2(b0, b1)), "l"(pack2(d0, d1)));
  unpack2(r, d0, d1);
}
// d[c] = a[c] + b[c] for c = 0, 1
__device__ __forceinline__ void add2(float& d0, float& d1, float a0, float a1, float b0, float b1) {
  unsigned long long r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(pack2(a0, a1)), "l"(pack2(b0, b1)));
  unpack2(r, d0, d1);
}
// d[c] = a[c] * b[c] for c = 0, 1
__device__ __forceinline__ void mul2(float& d0, float& d1, float a0, float a1, float b0, float b1) {
  unsigned long long r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(pack2(a0, a1)), "l"(pack2(b0, b1)));
  unpack2(r, d0, d1);
}

__device__ __forceinline__ float fma_io(__half a, __half b, float c) {
  float r;
  asm("fma.rn.f32.f16 %0, %1, %2, %3;" : "=f"(r) : "h"(__half_as_ushort(a)), "h"(__half_as_ushort(b)), "f"(c));
  return r;
}

template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

template <typename T, int N>
__device__ __forceinline__ void zero(Pack<T, N>& p) {
#pragma unroll
  for (int i = 0; i < N; ++i) p.v[i] = from_f<T>(0.f);
}

template <typename T, int N>
__device__ __forceinline__ Pack<T, N> ld(const T* ptr) {
  return *reinterpret_cast<const Pack<T, N>*>(ptr);
}

template <typename T, int N>
__device__ __forceinline__ void st(T* ptr, const Pack<T, N>& v) {
  *reinterpret_cast<Pack<T, N>*>(ptr) = v;
}

// Runtime-indexed read of a small register array without local memory.
template <int N, typename P>
__device__ __forceinline__ P sel(const P (&a)[N], int idx) {
  P r = a[0];
#pragma unroll
  for (int k = 1; k < N; ++k)
    if (k == idx) r = a[k];
  return r;
}

// 1 / (1 + e^-v) with the fast exponential and reciprocal (a few ulp, like the
// reference kernels' sigmoid); 0 for very negative v, 1 for very positive v.
__device__ __forceinline__ float sigmoidf_(float v) { return __fdividef(1.f, 1.f + __expf(-v)); }

// ---------------------------------------------------------------------------
// group reductions. NV channels per thread; GV groups per thread when G < NV
// (GC = NV / GV channels each), else one group spread over lpg = G / NV lanes.
// ---------------------------------------------------------------------------
// The thread's part: out[gi] = sum of its GC channels of group gi, in order;
// eight channels as two halves of four, each summed in order, then added --
// the sum that a thread of 4 channels and its neighbour lane form at the first
// step of the butterfly below, so that kernels with 8 and with 4 channels per
// thread give the same bits.
template <int NV, int GV>
__device__ __forceinline__ void group_local_sum(const float (&v)[NV], float (&out)[GV]) {
  constexpr int GC = NV / GV;
#pragma unroll
  for (int gi = 0; gi < GV; ++gi) {
    if constexpr (GC == 8) {
      // the two halves in the two lanes of the packed fp32 pipe
      float lo = 0.f, hi = 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) add2(lo, hi, lo, hi, v[gi * GC + c], v[gi * GC + 4 + c]);
      out[gi] = lo + hi;
    } else {
      float s = 0.f;
#pragma unroll
      for (int c = 0; c < GC; ++c) s += v[gi * GC + c];
      out[gi] = s;
    }
  }
}

// out[gi] = the sum over the GC channels of group gi of a[c] * b[c] (the
// thread's part of a group dot product): channel pairs accumulate in the two
// lanes of the packed fp32 pipe -- a product, then a fused multiply-add --
// and the two lanes are added last; eight channels as two halves of four,
// then added (group_local_sum's grouping).
template <int NV, int GV>
__device__ __forceinline__ void group_local_dot(const float (&a)[NV], const float (&b)[NV], float (&out)[GV]) {
  constexpr int GC = NV / GV;
#pragma unroll
  for (int gi = 0; gi < GV; ++gi) {
    const int c0 = gi * GC;
    if constexpr (GC == 1) {
      out[gi] = __fmul_rn(a[c0], b[c0]);
    } else {
      float s[GC >= 8 ? 2 : 1];
#pragma unroll
      for (int h = 0; h < (GC >= 8 ? 2 : 1); ++h) {
        const int c = c0 + 4 * h;
        float e, o;
        mul2(e, o, a[c], a[c + 1], b[c], b[c + 1]);
        if constexpr (GC >= 4) fma2(e, o, a[c + 2], a[c + 3], b[c + 2], b[c + 3]);
        s[h] = e + o;
      }
      out[gi] = GC >= 8 ? s[0] + s[GC >= 8 ? 1 : 0] : s[0];
    }
  }
}

// The butterfly over the lpg lanes of a group: lane bit 0 first, own + partner
// at each step (lpg is warp-uniform; the steps are unrolled so that the
// reductions of independent values can interleave).
__device__ __forceinline__ void group_xlane_sum(float& v, int lpg) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1)
    if (o < lpg) v += __shfl_xor_sync(0xffffffffu, v, o);
}

template <int NV, int GV>
__device__ __forceinline__ void group_sum(const float (&v)[NV], float (&out)[GV], int lpg) {
  group_local_sum<NV, GV>(v, out);
  if (GV == 1) group_xlane_sum(out[0], lpg);
}

// P per-lane values summed over the lpg lanes of a group and left spread over
// them (reduce-scatter): at the step over lane bit o, a lane keeps half of its
// values (the upper half when its bit o is set), sends the partner the other
// half and adds the partner's copy of the kept half; once one value is left the
// steps continue as a butterfly. Afterwards lane r of the group (r < min(lpg, P)
// holds distinct totals; the lanes above repeat them) holds the totals of
// values base .. base + cnt - 1 in v[0 .. cnt). The pairing and the order of
// each addition are group_xlane_sum's, so every total is bit-identical to it,
// with P - 1 shuffles instead of P log2(lpg) when lpg >= P.
template <int P>
__device__ __forceinline__ void group_sum_scatter(float (&v)[P], int lpg, int lane, int& base, int& cnt) {
  base = 0;
  cnt = P;
#pragma unroll
  for (int s = 0; s < 5; ++s) {
    const int o = 1 << s;
    const int m = P >> s;  // values per lane before this step (compile-time once unrolled)
    if (o < lpg) {
      if (m >= 2) {
        const int half = m >> 1;
        const bool hi = (lane & o) != 0;
#pragma unroll
        for (int j = 0; j < half; ++j) {
          const float send = hi ? v[j] : v[half + j];
          const float keep = hi ? v[half + j] : v[j];
          v[j] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
        if (hi) base += half;
        cnt = half;
      } else {
        v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
      }
    }
  }
}

template <int NV, int GV>
__device__ __forceinline__ void group_max(const float (&v)[NV], float (&out)[GV], int lpg) {
  constexpr int GC = NV / GV;
#pragma unroll
  for (int gi = 0; gi < GV; ++gi) {
    float s = v[gi * GC];
#pragma unroll
    for (int c = 1; c < GC; ++c) s = fmaxf(s, v[gi * GC + c]);
    out[gi] = s;
  }
  if (GV == 1) {
#pragma unroll
    for (int o = 1; o < 32; o <<= 1)
      if (o < lpg) out[0] = fmaxf(out[0], __shfl_xor_sync(0xffffffffu, out[0], o));
  }
}

// Group max of a[] and group sum of b[] in one butterfly (each the same
// arithmetic, in the same order, as group_max / group_sum).
template <int NV, int GV>
__device__ __forceinline__ void group_max_sum(const float (&a)[NV], const float (&b)[NV], float (&mx)[GV],
                                              float (&sm)[GV], int lpg) {
  constexpr int GC = NV / GV;
  group_local_sum<NV, GV>(b, sm);
#pragma unroll
  for (int gi = 0; gi < GV; ++gi) {
    float m = a[gi * GC];
#pragma unroll
    for (int c = 1; c < GC; ++c) m = fmaxf(m, a[gi * GC + c]);
    mx[gi] = m;
  }
  if (GV == 1) {
#pragma unroll
    for (int o = 1; o < 32; o <<= 1)
      if (o < lpg) {
        const float pm = __shfl_xor_sync(0xffffffffu, mx[0], o);
        const float ps = __shfl_xor_sync(0xffffffffu, sm[0], o);
        mx[0] = fmaxf(mx[0], pm);
        sm[0] += ps;
      }
  }
}

// The overflow-safe group RMS norm, given the group max of |y| (mx) and the
// group sum of y^2 (ss). Its form s * sqrt(mean((y/s)^2) + eps/s^2), with
// s = max(max|y|, 1), equals sqrt(mean(y^2) + eps): while every group of the
// warp has max|y| < 2^60 that is what is computed; otherwise (or for a NaN)
// the warp takes the rescaled two-pass form. The bound is strict: each square
// is then below 2^120, and a rounded sum of at most 256 of them stays below
// 256 * 2^120 = 2^128, i.e. finite, whereas 256 squares of exactly 2^60 sum
// to 2^128 = inf. For max|y| <= 1 both forms are the same arithmetic. Must be
// called by all 32 lanes.
template <int NV, int GV>
__device__ __forceinline__ void stable_finish(float (&acc)[NV], float (&mx)[GV], float (&ss)[GV], int G, int lpg,
                                              float eps) {
  constexpr int GC = NV / GV;
  const float inv_g = 1.f / (float)G;  // G is a power of two: exact
  bool big = false;
#pragma unroll
  for (int gi = 0; gi < GV; ++gi) big = big || !(mx[gi] < 0x1p60f);
  if (__any_sync(0xffffffffu, big)) {
#pragma unroll
    for (int gi = 0; gi < GV; ++gi) mx[gi] = __frcp_rn(fmaxf(mx[gi], 1.f));  // 1 / s, exact for s up to FLT_MAX
    float sq[NV];
#pragma unroll
    for (int c = 0; c < NV; ++c) {
      const float s = acc[c] * mx[c / GC];
      sq[c] = s * s;
    }
    group_sum<NV, GV>(sq, ss, lpg);
#pragma unroll
    for (int gi = 0; gi < GV; ++gi) ss[gi] = mx[gi] * rsqrtf(ss[gi] * inv_g + eps * mx[gi] * mx[gi]);
  } else {
#pragma unroll
    for (int gi = 0; gi < GV; ++gi) ss[gi] = rsqrtf(ss[gi] * inv_g + eps);
  }
#pragma unroll
  for (int c = 0; c < NV; ++c) acc[c] *= ss[c / GC];
}

// q[c] = a[c] * a[c], channel pairs on the packed fp32 pipe (each lane
// rounded like the scalar product)
template <int NV>
__device__ __forceinline__ void sq_pairs(const float (&a)[NV], float (&q)[NV]) {
  if constexpr (NV % 2 == 0) {
#pragma unroll
    for (int c = 0; c < NV; c += 2) mul2(q[c], q[c + 1], a[c], a[c + 1], a[c], a[c + 1]);
  } else {
#pragma unroll
    for (int c = 0; c < NV; ++c) q[c] = a[c] * a[c];
  }
}
// a[c] *= s[group of c], channel pairs on the packed fp32 pipe
template <int NV, int GV>
__device__ __forceinline__ void scale_pairs(float (&a)[NV], const float (&s)[GV]) {
  constexpr int GC = NV / GV;
  if constexpr (NV % 2 == 0) {
#pragma unroll
    for (int c = 0; c < NV; c += 2) mul2(a[c], a[c + 1], a[c], a[c + 1], s[c / GC], s[(c + 1) / GC]);
  } else {
#pragma unroll
    for (int c = 0; c < NV; ++c) a[c] *= s[c / GC];
  }
}
// a[c] *= g[c] * sigmoid(g[c]) (the SiLU gate), the two products on the
// packed fp32 pipe
template <int NV>
__device__ __forceinline__ void gate_pairs(float (&a)[NV], const float (&g)[NV]) {
  if constexpr (NV % 2 == 0) {
#pragma unroll
    for (int c = 0; c < NV; c += 2) {
      float t0, t1;
      mul2(t0, t1, g[c], g[c + 1], sigmoidf_(g[c]), sigmoidf_(g[c + 1]));
      mul2(a[c], a[c + 1], a[c], a[c + 1], t0, t1);
    }
  } else {
#pragma unroll
    for (int c = 0; c < NV; ++c) a[c] = a[c] * (g[c] * sigmoidf_(g[c]));
  }
}

// Group RMS norm of a thread's NV accumulators, in place.
//   plain : y * 1/sqrt(mean(y^2) + eps)               (greta/dynamic_conv.py:251-255)
//   stable: s = max(max|y|, 1); y / (s * sqrt(mean((y/s)^2) + eps/s^2))
//                                                    (greta_vllm/triton_conv.py:71-77)
// The reciprocal square roots are the hardware's fast form, as the reference
// kernels' tl.rsqrt; 1/s is rounded exactly, so that groups with s above 2^126
// (where a fast reciprocal flushes to zero) stay finite.
template <int NORM, int NV, int GV>
__device__ __forceinline__ void apply_norm(float (&acc)[NV], int G, int lpg, float eps) {
  const float inv_g = 1.f / (float)G;  // G is a power of two: exact
  if (NORM == kNormPlain) {
    float sq[NV], ss[GV];
    sq_pairs<NV>(acc, sq);
    group_sum<NV, GV>(sq, ss, lpg);
#pragma unroll
    for (int gi = 0; gi < GV; ++gi) ss[gi] = rsqrtf(ss[gi] * inv_g + eps);
    scale_pairs<NV, GV>(acc, ss);
  } else if (NORM == kNormStable) {
    float ab[NV], sq[NV], mx[GV], ss[GV];
#pragma unroll
    for (int c = 0; c < NV; ++c) {
      ab[c] = fabsf(acc[c]);
      sq[c] = acc[c] * acc[c];
    }
    group_max_sum<NV, GV>(ab, sq, mx, ss, lpg);
    stable_finish<NV, GV>(acc, mx, ss, G, lpg, eps);
  }
}

// apply_norm on two tokens' accumulators at once: the same arithmetic in the
// same order for each (so each result is bit-identical to apply_norm's), with
// the two tokens' group reductions interleaved so that their shuffle
// latencies overlap.
template <int NV, int GV>
__device__ __forceinline__ void group_sum2(const float (&a)[NV], const float (&b)[NV], float (&oa)[GV],
                                           float (&ob)[GV], int lpg) {
  group_local_sum<NV, GV>(a, oa);
  group_local_sum<NV, GV>(b, ob);
  if (GV == 1) {
#pragma unroll
    for (int o = 1; o < 32; o <<= 1)
      if (o < lpg) {
        const float pa = __shfl_xor_sync(0xffffffffu, oa[0], o);
        const float pb = __shfl_xor_sync(0xffffffffu, ob[0], o);
        oa[0] += pa;
        ob[0] += pb;
      }
  }
}

// group_max_sum for two tokens, their four reductions in one butterfly.
template <int NV, int GV>
__device__ __forceinline__ void group_max_sum2(const float (&a)[NV], const float (&b)[NV], const float (&c2)[NV],
                                               const float (&d)[NV], float (&ma)[GV], float (&sb)[GV],
                                               float (&mc)[GV], float (&sd)[GV], int lpg) {
  constexpr int GC = NV / GV;
  group_local_sum<NV, GV>(b, sb);
  group_local_sum<NV, GV>(d, sd);
#pragma unroll
  for (int gi = 0; gi < GV; ++gi) {
    float m = a[gi * GC], n = c2[gi * GC];
#pragma unroll
    for (int c = 1; c < GC; ++c) {
      m = fmaxf(m, a[gi * GC + c]);
      n = fmaxf(n, c2[gi * GC + c]);
    }
    ma[gi] = m;
    mc[gi] = n;
  }
  if (GV == 1) {
#pragma unroll
    for (int o = 1; o < 32; o <<= 1)
      if (o < lpg) {
        const float p0 = __shfl_xor_sync(0xffffffffu, ma[0], o);
        const float p1 = __shfl_xor_sync(0xffffffffu, sb[0], o);
        const float p2 = __shfl_xor_sync(0xffffffffu, mc[0], o);
        const float p3 = __shfl_xor_sync(0xffffffffu, sd[0], o);
        ma[0] = fmaxf(ma[0], p0);
        sb[0] += p1;
        mc[0] = fmaxf(mc[0], p2);
        sd[0] += p3;
      }
  }
}

template <int NORM, int NV, int GV>
__device__ __forceinline__ void apply_norm2(float (&a)[NV], float (&b)[NV], int G, int lpg, float eps) {
  const float inv_g = 1.f / (float)G;  // G is a power of two: exact
  if (NORM == kNormPlain) {
    float qa[NV], qb[NV], sa[GV], sb[GV];
    sq_pairs<NV>(a, qa);
    sq_pairs<NV>(b, qb);
    group_sum2<NV, GV>(qa, qb, sa, sb, lpg);
#pragma unroll
    for (int gi = 0; gi < GV; ++gi) {
      sa[gi] = rsqrtf(sa[gi] * inv_g + eps);
      sb[gi] = rsqrtf(sb[gi] * inv_g + eps);
    }
    scale_pairs<NV, GV>(a, sa);
    scale_pairs<NV, GV>(b, sb);
  } else if (NORM == kNormStable) {
    float ba[NV], bb[NV], qa[NV], qb[NV], ma[GV], mb[GV], sa[GV], sb[GV];
#pragma unroll
    for (int c = 0; c < NV; ++c) {
      ba[c] = fabsf(a[c]);
      bb[c] = fabsf(b[c]);
      qa[c] = a[c] * a[c];
      qb[c] = b[c] * b[c];
    }
    group_max_sum2<NV, GV>(ba, qa, bb, qb, ma, sa, mb, sb, lpg);
    stable_finish<NV, GV>(a, ma, sa, G, lpg, eps);
    stable_finish<NV, GV>(b, mb, sb, G, lpg, eps);
  }
}

// ---------------------------------------------------------------------------
// Backward pieces shared by both backward kernels, so that they stay
// bit-identical: channel pairs on the packed fp32 pipe, each lane rounded
// like the scalar operation.
// ---------------------------------------------------------------------------
// dy[c] = (dout[c] * g[c]) * sigmoid(g[c]): the gradient through the SiLU gate
template <int NV>
__device__ __forceinline__ void bwd_gate_dy(const float (&dv)[NV], const float (&g)[NV], float (&dy)[NV]) {
  if constexpr (NV % 2 == 0) {
#pragma unroll
    for (int c = 0; c < NV; c += 2) {
      float t0, t1;
      mul2(t0, t1, dv[c], dv[c + 1], g[c], g[c + 1]);
      mul2(dy[c], dy[c + 1], t0, t1, sigmoidf_(g[c]), sigmoidf_(g[c + 1]));
    }
  } else {
#pragma unroll
    for (int c = 0; c < NV; ++c) dy[c] = __fmul_rn(__fmul_rn(dv[c], g[c]), sigmoidf_(g[c]));
  }
}

// The plain group RMS norm's backward, in place on dy, from the saved
// pre-norm output yr: rinv = 1/sqrt(mean(yr^2) + eps), n = yr * rinv,
// dy <- rinv * (dy - n * mean(n * dy)), where mean(n * dy) =
// rinv * mean(yr * dy), so the two group sums (yr^2, yr * dy) run as one
// interleaved reduction. Leaves rinv of each group.
template <int NV, int GV>
__device__ __forceinline__ void bwd_norm(const float (&yr)[NV], float (&dy)[NV], float (&rinv)[GV], float inv_g,
                                         float eps, int lpg) {
  constexpr int GC = NV / GV;
  float sq[NV], py[NV], nk[GV];
  if constexpr (NV % 2 == 0) {
#pragma unroll
    for (int c = 0; c < NV; c += 2) {
      mul2(sq[c], sq[c + 1], yr[c], yr[c + 1], yr[c], yr[c + 1]);
      mul2(py[c], py[c + 1], yr[c], yr[c + 1], dy[c], dy[c + 1]);
    }
  } else {
#pragma unroll
    for (int c = 0; c < NV; ++c) {
      sq[c] = __fmul_rn(yr[c], yr[c]);
      py[c] = __fmul_rn(yr[c], dy[c]);
    }
  }
  group_sum2<NV, GV>(sq, py, rinv, nk, lpg);
#pragma unroll
  for (int gi = 0; gi < GV; ++gi) {
    rinv[gi] = rsqrtf(rinv[gi] * inv_g + eps);
    nk[gi] = -((nk[gi] * rinv[gi]) * inv_g);  // -mean(n * dy)
  }
  if constexpr (NV % 2 == 0) {
#pragma unroll
    for (int c = 0; c < NV; c += 2) {
      const float r0 = rinv[c / GC], r1 = rinv[(c + 1) / GC];
      float n0, n1, t0 = dy[c], t1 = dy[c + 1];
      mul2(n0, n1, yr[c], yr[c + 1], r0, r1);
      fma2(t0, t1, n0, n1, nk[c / GC], nk[(c + 1) / GC]);
      mul2(dy[c], dy[c + 1], r0, r1, t0, t1);
    }
  } else {
#pragma unroll
    for (int c = 0; c < NV; ++c) {
      const float r = rinv[c / GC];
      dy[c] = __fmul_rn(r, __fmaf_rn(__fmul_rn(yr[c], r), nk[c / GC], dy[c]));
    }
  }
}

// dg[c] = (dout[c] * hat[c]) * (s * (1 + g[c] * (1 - s))), s = sigmoid(g[c]):
// the gate's gradient, hat the gated value (the normed or plain conv output)
template <int NV>
__device__ __forceinline__ void bwd_gate_dg(const float (&dv)[NV], const float (&g)[NV], const float (&hat)[NV],
                                            float (&dg)[NV]) {
  if constexpr (NV % 2 == 0) {
#pragma unroll
    for (int c = 0; c < NV; c += 2) {
      const float s0 = sigmoidf_(g[c]), s1 = sigmoidf_(g[c + 1]);
      float o0 = 1.f, o1 = 1.f, q0 = 1.f, q1 = 1.f, a0, a1;
      fma2(o0, o1, -1.f, -1.f, s0, s1);  // 1 - s
      fma2(q0, q1, g[c], g[c + 1], o0, o1);
      mul2(q0, q1, s0, s1, q0, q1);
      mul2(a0, a1, dv[c], dv[c + 1], hat[c], hat[c + 1]);
      mul2(dg[c], dg[c + 1], a0, a1, q0, q1);
    }
  } else {
#pragma unroll
    for (int c = 0; c < NV; ++c) {
      const float sg = sigmoidf_(g[c]);
      const float q = __fmul_rn(sg, __fmaf_rn(g[c], __fmaf_rn(-1.f, sg, 1.f), 1.f));
      dg[c] = __fmul_rn(__fmul_rn(dv[c], hat[c]), q);
    }
  }
}

// ---------------------------------------------------------------------------
// chunk resolution
// ---------------------------------------------------------------------------
struct ChunkInfo {
  long long x_base;  // row of local position 0 in x
  long long o_base;  // row of local position 0 in w / g / y / yr
  long long len;     // sequence length
  long long c0, c1;  // chunk token range [c0, c1), local positions
  long long slot;    // cache slot, -1 = none
  int hist;          // HistKind for positions < 0
  int has_state;     // old slot contents are used
  int head;          // first chunk of its sequence
};

__device__ __forceinline__ long long load_idx(const void* p, long long i, int is64) {
  return is64 ? reinterpret_cast<const long long*>(p)[i] : (long long)reinterpret_cast<const int*>(p)[i];
}

__device__ __forceinline__ long long clampll(long long v, long long lo, long long hi) {
  return v < lo ? lo : (v > hi ? hi : v);
}

// Block-wide search of chunk `cid` among sequences described by cumulative
// offsets `starts` (clamped to [0, T]). Sequence i owns max(1, ceil(len_i /
// chunk)) chunks (an empty sequence keeps one chunk for its state write-back).
// All threads of the block must call this. Returns false when cid is past the
// last chunk. Each thread handles kItems consecutive sequences per pass.
struct SeqHit {
  long long s, j, a, b;
  int slot_raw;
  int init;
};

//
// With skip = 1 only the chunks after each sequence's first are numbered
// (chunk j >= 1 of sequence i is number j - 1 + the count of earlier
// sequences' later chunks); the first chunks are then addressed directly.
template <int kItems>
__device__ bool block_find_chunk(const void* starts, int is64, long long nseq, long long T,
                                 int chunk, long long cid, const int* slots,
                                 const signed char* initial, SeqHit& hit, int skip = 0) {
  __shared__ long long sh_warp[32];
  __shared__ SeqHit sh_hit;
  __shared__ int sh_found;
  const int nthr = blockDim.x * blockDim.y;
  const int tid = threadIdx.y * blockDim.x + threadIdx.x;
  const int lane = tid & 31, wid = tid >> 5, nw = (nthr + 31) >> 5;
  if (tid == 0) sh_found = 0;
  __syncthreads();
  long long running = 0;
  for (long long base = 0; base < nseq; base += (long long)nthr * kItems) {
    const long long i0 = base + (long long)tid * kItems;
    long long bnd[kItems + 1];
    long long cnt[kItems];
    long long tot = 0;
#pragma unroll
    for (int k = 0; k <= kItems; ++k) {
      const long long i = i0 + k;
      bnd[k] = (i <= nseq) ? clampll(load_idx(starts, i, is64), 0, T) : 0;
    }
#pragma unroll
    for (int k = 0; k < kItems; ++k) {
      long long n = 0;
      if (i0 + k < nseq) {
        n = bnd[k + 1] - bnd[k];
        if (n < 0) n = 0;
        n = n > 0 ? (n + chunk - 1) / chunk : 1;
        n -= skip;
      }
      cnt[k] = n;
      tot += n;
    }
    // block exclusive scan of tot
    long long incl = tot;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const long long t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += t;
    }
    if (lane == 31 || tid == nthr - 1) sh_warp[wid] = incl;
    __syncthreads();
    if (wid == 0) {
      long long v = lane < nw ? sh_warp[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const long long t = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += t;
      }
      if (lane < nw) sh_warp[lane] = v;
    }
    __syncthreads();
    long long ex = running + (wid > 0 ? sh_warp[wid - 1] : 0) + incl - tot;
    const long long block_total = sh_warp[nw - 1];
#pragma unroll
    for (int k = 0; k < kItems; ++k) {
      if (i0 + k < nseq && cid >= ex && cid < ex + cnt[k]) {
        SeqHit h;
        h.s = i0 + k;
        h.j = cid - ex + skip;
        h.a = bnd[k];
        h.b = bnd[k + 1] < bnd[k] ? bnd[k] : bnd[k + 1];
        h.slot_raw = slots ? slots[i0 + k] : -1;
        h.init = initial ? (int)initial[i0 + k] : 0;
        sh_hit = h;
        sh_found = 1;
      }
      ex += cnt[k];
    }
    running += block_total;
    __syncthreads();
    if (running > cid) break;  // uniform: running is the same in every thread
  }
  const bool found = sh_found != 0;
  if (found) hit = sh_hit;
  return found;
}

}  // namespace greta


namespace greta {

// ---------------------------------------------------------------------------
// per-thread asynchronous global->shared copies (cp.async). A thread stages
// its own operands in shared memory; only the thread that issued a copy reads
// it (after cp.async.wait_group), so no barrier is involved. With pred false
// nothing is read and the destination is zero-filled.
// ---------------------------------------------------------------------------
__device__ __forceinline__ unsigned smem_addr(const void* p) {
  return static_cast<unsigned>(__cvta_generic_to_shared(p));
}

template <int BYTES>
__device__ __forceinline__ void cp_async(void* dst, const void* src, bool pred) {
  static_assert(BYTES == 4 || BYTES == 8 || BYTES == 16, "cp.async moves 4, 8 or 16 bytes");
  const unsigned n = pred ? BYTES : 0;
  if constexpr (BYTES == 16) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_addr(dst)), "l"(src), "r"(n)
                 : "memory");
  } else {
    asm volatile("cp.async.ca.shared.global [%0], [%1], %2, %3;\n" ::"r"(smem_addr(dst)), "l"(src), "n"(BYTES),
                 "r"(n)
                 : "memory");
  }
}

// Copy one pack of BYTES (a multiple of 16, or 4 / 8). Smaller packs are
// never staged (callers keep them in registers); the empty branch only lets
// such instantiations compile.
template <int BYTES>
__device__ __forceinline__ void cp_async_pack(void* dst, const void* src, bool pred) {
  if constexpr (BYTES >= 16) {
#pragma unroll
    for (int o = 0; o < BYTES; o += 16)
      cp_async<16>(static_cast<char*>(dst) + o, static_cast<const char*>(src) + o, pred);
  } else if constexpr (BYTES == 4 || BYTES == 8) {
    cp_async<BYTES>(dst, src, pred);
  }
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }

template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// wait until at most `pending` (runtime, 0..3) of this thread's groups are in flight
__device__ __forceinline__ void cp_async_wait_rt(int pending) {
  switch (pending) {
    case 0: cp_async_wait<0>(); break;
    case 1: cp_async_wait<1>(); break;
    case 2: cp_async_wait<2>(); break;
    default: cp_async_wait<3>(); break;
  }
}

}  // namespace greta
