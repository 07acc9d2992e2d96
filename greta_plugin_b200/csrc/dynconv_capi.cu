// C ABI of libgreta_dynconv.so: argument validation, vector-path selection,
// launch shapes, and dispatch to the per-dtype kernel instantiations.
// Declarations and the contract of every entry point: include/greta_dynconv.h.
#include <stdint.h>

#include <climits>
#include <initializer_list>

#include "dynconv_fwd_wide.cuh"
#include "dynconv_launch.cuh"
#include "greta_dynconv.h"

using namespace greta;

namespace {

constexpr int kAbiVersion = 10100;  // 1.1.0: per-call options (_ex), wide groups on the packed call

int esize(int dtype) {
  switch (dtype) {
    case GRETA_DT_F32: return 4;
    case GRETA_DT_F16: return 2;
    case GRETA_DT_BF16: return 2;
    default: return 0;
  }
}

bool is_pow2(int64_t v) { return v > 0 && (v & (v - 1)) == 0; }

bool aligned(const void* p, int64_t a) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// max_g: the widest group the entry point takes (256, or D for the packed
// call, whose wide groups run on dynconv_fwd_wide_kernel)
int check_common(int dtype, int64_t D, int64_t W, int64_t G, int norm, int64_t max_g = 256) {
  if (esize(dtype) == 0) return GRETA_ERR_UNSUPPORTED;
  if (D <= 0 || W <= 0 || G <= 0) return GRETA_ERR_INVALID_ARG;
  if (D > (int64_t)INT_MAX / 2) return GRETA_ERR_INVALID_ARG;
  if (D % G != 0) return GRETA_ERR_INVALID_ARG;
  if (!is_pow2(G) || G > max_g) return GRETA_ERR_UNSUPPORTED;
  if (W > kMaxWGeneric) return GRETA_ERR_UNSUPPORTED;
  if (norm < GRETA_NORM_NONE || norm > GRETA_NORM_STABLE) return GRETA_ERR_UNSUPPORTED;
  return GRETA_OK;
}

int group_vec(int nv, int64_t G) { return nv == 1 ? 1 : (G >= kVec ? 1 : (int)(kVec / G)); }

// kVec channels per thread when every row is a whole number of aligned
// vectors; one channel per thread otherwise (only possible for G <= 32,
// since one group must fit the lanes of one warp).
int pick_nv(int dtype, int64_t D, int64_t G, std::initializer_list<const void*> rows, const void* w) {
  const int es = esize(dtype);
  bool ok = D % kVec == 0;
  for (const void* p : rows) ok = ok && aligned(p, (int64_t)kVec * es);
  ok = ok && aligned(w, (int64_t)group_vec(kVec, G) * es);
  if (ok) return kVec;
  if (G > 32) return 0;
  return 1;
}

// Row strides usable by the vector kernels: every row of a [T, D] tensor
// starts on a whole kVec-element vector (a thread loads its kVec channels as
// one aligned pack: 16 bytes for 16-bit types, 32 for fp32), every filter row
// on a whole group vector.
bool strides_vec_ok(int dtype, int64_t G, std::initializer_list<int64_t> rows, std::initializer_list<int64_t> wrows) {
  (void)dtype;
  for (int64_t ld : rows)
    if (ld % kVec != 0) return false;
  for (int64_t ld : wrows)
    if (ld % group_vec(kVec, G) != 0) return false;
  return true;
}

// 1-D grid of chunks x channel blocks, channel block fastest.
LaunchShape make_shape(long long chunks, int64_t D, int nv, int tx, int ty) {
  const long long lanes = (D + nv - 1) / nv;
  const long long need = ((lanes + 31) / 32) * 32;
  if (tx > need) tx = (int)need;
  LaunchShape s;
  s.block = dim3(tx, ty, 1);
  s.nblk = (int)((lanes + tx - 1) / tx);
  s.grid = dim3((unsigned)(chunks * s.nblk), 1, 1);
  return s;
}

int finish(cudaError_t e) { return e == cudaSuccess ? GRETA_OK : GRETA_ERR_LAUNCH; }

// Row strides of the inputs: 0 means a contiguous tensor (x and gate rows of
// D elements, filter rows of W * D/G).
template <typename P>
P with_strides(P p) {
  if (p.ldx == 0) p.ldx = p.D;
  if (p.ldg == 0) p.ldg = p.D;
  if (p.ldw == 0) p.ldw = (long long)p.W * (p.D / p.G);
  return p;
}

// The same for the backward's outputs dx, dg and dw.
template <typename P>
P with_bwd_strides(P p) {
  p = with_strides(p);
  if (p.lddx == 0) p.lddx = p.D;
  if (p.lddg == 0) p.lddg = p.D;
  if (p.lddw == 0) p.lddw = (long long)p.W * (p.D / p.G);
  return p;
}

cudaError_t run_fwd(int dtype, const FwdParams& p, int nv, int norm, const LaunchShape& s, void* stream) {
  const int gv = group_vec(nv, p.G);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case GRETA_DT_F32: return launch_fwd_f32(with_strides(p), nv, norm, gv, s, st);
    case GRETA_DT_F16: return launch_fwd_f16(with_strides(p), nv, norm, gv, s, st);
    default: return launch_fwd_bf16(with_strides(p), nv, norm, gv, s, st);
  }
}

cudaError_t run_bwd(int dtype, const BwdParams& p, int nv, int norm, const LaunchShape& s, void* stream) {
  const int gv = group_vec(nv, p.G);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case GRETA_DT_F32: return launch_bwd_f32(with_bwd_strides(p), nv, norm, gv, s, st);
    case GRETA_DT_F16: return launch_bwd_f16(with_bwd_strides(p), nv, norm, gv, s, st);
    default: return launch_bwd_bf16(with_bwd_strides(p), nv, norm, gv, s, st);
  }
}

cudaError_t run_fwd_decode(int dtype, const FwdParams& p, int norm, const LaunchShape& s, void* stream) {
  const int gv = group_vec(kVec, p.G);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case GRETA_DT_F32: return launch_fwd_decode_f32(with_strides(p), norm, gv, s, st);
    case GRETA_DT_F16: return launch_fwd_decode_f16(with_strides(p), norm, gv, s, st);
    default: return launch_fwd_decode_bf16(with_strides(p), norm, gv, s, st);
  }
}

cudaError_t run_fwd_wide(int dtype, const FwdParams& p, int norm, dim3 grid, dim3 block, int groups, void* stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case GRETA_DT_F32: return launch_fwd_wide_f32(with_strides(p), norm, grid, block, groups, st);
    case GRETA_DT_F16: return launch_fwd_wide_f16(with_strides(p), norm, grid, block, groups, st);
    default: return launch_fwd_wide_bf16(with_strides(p), norm, grid, block, groups, st);
  }
}

long long cdiv(long long a, long long b) { return (a + b - 1) / b; }

// Built-in CTA shapes per launch path: {threads along channels (tx), token
// runs per CTA (ty), tokens per run (L)}; a CTA owns tx*8 channels of ty*L
// consecutive tokens and each thread walks one run. Long streams use 32x4
// CTAs; the backward uses longer runs to amortise its W-1 row right halo;
// packed prefill uses short runs so a ~1k-token batch spreads over the GPU;
// decode has one token per request and uses 128-thread CTAs (the decode
// kernel's limit) with chunks of 8 tokens for the occasional longer request.
struct Shape {
  int tx, ty, L;
};
enum Path { kPathFwd = 0, kPathBwd, kPathInference, kPathDecodeRows, kPathPackedPrefill, kPathPackedDecode, kPaths };
constexpr Shape kDefaultShape[kPaths] = {
    {32, 4, 16},   // training forward
    {32, 4, 32},   // training backward
    {32, 4, 16},   // HF inference from context
    {128, 1, 1},   // HF decode rows
    {32, 2, 8},    // packed batches with more than 2 tokens per request
    {128, 1, 8},   // packed batches with at most 2 tokens per request
};

// Per-call launch choices (greta_dynconv_options); the library keeps no
// process-wide settings.
struct Opts {
  int kernel = GRETA_KERNEL_AUTO;  // GRETA_KERNEL_*
  Shape shape{0, 0, 0};  // register-kernel CTA shape (tx == 0: built-in)
  int wait_log2 = 0;   // pipeline wait bound of the row-streaming kernels
  int withhold = 0;    // test hook of the row-streaming forward
  int rows_channels = 0;  // row-streaming kernels: channel-slice cap (0: built-in)
  int rows_ranges = 0;    // row-streaming kernels: token ranges (0: SMs / slices)
  int rows_smem = 200 * 1024;  // row-streaming kernels: stage-ring budget (bytes)
};

// GRETA_OK and the parsed options, or GRETA_ERR_INVALID_ARG for a bad struct.
int parse_opts(const greta_dynconv_options* o, Opts& out) {
  out = Opts{};
  if (o == nullptr) return GRETA_OK;
  if (o->size != (int)sizeof(greta_dynconv_options)) return GRETA_ERR_INVALID_ARG;
  if (o->kernel < GRETA_KERNEL_AUTO || o->kernel > GRETA_KERNEL_ROWS) return GRETA_ERR_INVALID_ARG;
  out.kernel = o->kernel;
  if (o->block_x > 0 && o->block_y > 0 && o->tokens > 0) {
    if (o->block_x % 32 != 0 || o->block_x * o->block_y > 256) return GRETA_ERR_INVALID_ARG;
    out.shape = Shape{o->block_x, o->block_y, o->tokens};
  }
  if (o->wait_limit_log2 != 0 && (o->wait_limit_log2 < 8 || o->wait_limit_log2 > 24)) return GRETA_ERR_INVALID_ARG;
  out.wait_log2 = o->wait_limit_log2;
  out.withhold = o->test_withhold_release != 0 ? 1 : 0;
  if (o->rows_channels < 0 || (o->rows_channels > 0 && o->rows_channels < 256)) return GRETA_ERR_INVALID_ARG;
  if (o->rows_ranges < 0 || o->rows_ranges > (1 << 20)) return GRETA_ERR_INVALID_ARG;
  if (o->rows_smem_kb != 0 && (o->rows_smem_kb < 32 || o->rows_smem_kb > 200)) return GRETA_ERR_INVALID_ARG;
  out.rows_channels = o->rows_channels;
  out.rows_ranges = o->rows_ranges;
  if (o->rows_smem_kb != 0) out.rows_smem = o->rows_smem_kb * 1024;
  return GRETA_OK;
}

// ---------------------------------------------------------------------------
// TMA forward (dynconv_fwd_tma.cuh): applicability and shared-memory plan
// ---------------------------------------------------------------------------

int num_sms() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  static int cache[64] = {0};
  if (dev >= 0 && dev < 64 && cache[dev] > 0) return cache[dev];
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  if (dev >= 0 && dev < 64) cache[dev] = n;
  return n;
}

size_t a128(size_t v) { return (v + 127) & ~(size_t)127; }

cudaError_t run_rows(int dtype, const RowsParams& p, int norm, int gv, dim3 grid, dim3 block, size_t smem,
                     void* stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case GRETA_DT_F32: return launch_fwd_rows_f32(with_strides(p), norm, gv, grid, block, smem, st);
    case GRETA_DT_F16: return launch_fwd_rows_f16(with_strides(p), norm, gv, grid, block, smem, st);
    default: return launch_fwd_rows_bf16(with_strides(p), norm, gv, grid, block, smem, st);
  }
}

// Channels per CTA of a row-streaming kernel: the widest multiple of 256 that
// divides D and is at most max_c (0 when there is none).
int64_t slice_channels(int64_t D, int64_t max_c) {
  for (int64_t n = 1; n <= D / 256; ++n)
    if (D % n == 0 && (D / n) % 256 == 0 && D / n <= max_c) return D / n;
  return 0;
}

// Launch the row-streaming TMA forward when it applies: rows of whole
// 256-channel blocks (split over CTAs of at most fwd_rows_max_channels),
// 16-byte aligned tensors and copies, DS / SD state, at most kMaxSeqsTma
// sequences, and room for at least two token rows in flight. Returns -1 when
// it does not.
int try_rows_fwd(int dtype, RowsParams p, bool gate, int norm, void* stream, const Opts& o) {
  if (o.kernel != GRETA_KERNEL_AUTO && o.kernel != GRETA_KERNEL_ROWS) return -1;
  p = with_strides(p);
  p.wait_log2 = o.wait_log2;
  p.withhold = o.withhold;
  const int es = esize(dtype);
  // every bulk copy starts on a 16-byte boundary: row strides too
  if ((p.ldx * es) % 16 != 0 || (p.ldg * es) % 16 != 0 || (p.ldw * es) % 16 != 0) return -1;
  const int64_t D = p.D, W = p.W, G = p.G, DC = D / G;
  if (D % 256 != 0 || W > kMaxWGeneric) return -1;
  if (p.mode == kModePacked && p.nseq > kMaxSeqsTma) return -1;
  if (p.state != nullptr && p.st_layout != kStDS && p.st_layout != kStSD) return -1;
  if (p.U >= ((int64_t)1 << 31)) return -1;  // token positions are 32-bit inside the kernel
  for (const void* q : {p.x, p.w, p.g, (const void*)p.y, (const void*)p.yr})
    if (!aligned(q, 16)) return -1;
  // the W template launch_fwd_rows picks: 4, 7, -8 or -kMaxWGeneric
  const int wt = W == 4 ? 4 : (W == 7 ? 7 : (W <= 8 ? -8 : -kMaxWGeneric));
  int64_t cmax = fwd_rows_max_channels(wt);
  if (o.rows_channels > 0 && o.rows_channels < cmax) cmax = o.rows_channels;
  const int64_t dcta = slice_channels(D, cmax);
  if (dcta == 0) return -1;
  const int64_t nsplit = D / dcta;
  if ((W * DC * es) % 16 != 0) return -1;
  const bool wsplit = nsplit > 1 && W * DC * es > 2048;
  if (wsplit && ((dcta / G) * es) % 16 != 0) return -1;
  const int64_t rowx = dcta * es, roww = wsplit ? W * (dcta / G) * es : W * DC * es;
  const bool packed = p.mode == kModePacked;
  // offsets [nseq + 1] x 8 B, then (with a state) slots [nseq] x 4 B and flags [nseq] x 1 B
  const size_t off_meta = packed ? (size_t)(p.nseq + 1) * 8 : 0;
  const size_t meta = packed && p.state != nullptr ? (size_t)p.nseq * 5 : 0;
  const size_t off_stage = packed ? a128(off_meta + meta) : 0;
  const size_t budget = (size_t)o.rows_smem;
  if (off_stage >= budget) return -1;
  const int64_t per_token = rowx + roww + (gate ? rowx : 0);
  const int64_t inflight = (int64_t)(budget - off_stage) / per_token;
  if (inflight < 2) return -1;
  int S, BT;
  if (inflight >= 8) {
    S = 4;
    BT = (int)(inflight / 4 < 16 ? inflight / 4 : 16);
  } else {
    S = (int)(inflight < kMaxStages ? inflight : kMaxStages);
    BT = 1;
  }
  size_t so_w, so_g, stage;
  for (;;) {
    so_w = a128((size_t)BT * rowx);
    so_g = so_w + a128((size_t)BT * roww);
    stage = so_g + (gate ? a128((size_t)BT * rowx) : 0);
    if (off_stage + S * stage <= budget || (BT == 1 && S == 2)) break;
    if (BT > 1) --BT; else --S;
  }
  if (off_stage + S * stage > budget) return -1;
  p.BT = BT;
  p.stages = S;
  p.off_bnd = 0;
  p.off_meta = (int)off_meta;
  p.off_stage = (int)off_stage;
  p.stage_bytes = (int)stage;
  p.so_w = (int)so_w;
  p.so_g = (int)so_g;
  p.dcta = (int)dcta;
  p.nsplit = (int)nsplit;
  p.wsplit = wsplit ? 1 : 0;
  p.log2g = 0;
  while ((1 << p.log2g) < G) ++p.log2g;
  long long ranges = o.rows_ranges > 0 ? o.rows_ranges : num_sms() / nsplit;
  if (ranges < 1) ranges = 1;
  if (p.U < ranges) ranges = p.U;
  if (ranges <= 0) return GRETA_OK;
  // balanced ranges: U / ranges tokens, the first U % ranges one longer
  p.nominal = p.U / ranges;
  p.nom_rem = (int)(p.U % ranges);
  // L2 prefetch at the start: the first rows of every range, about 48 MB in
  // all (a whole short prefill; the head of each range of a long stream)
  const int64_t full_row = D * es * (gate ? 2 : 1) + W * DC * es;
  int64_t pf = ((int64_t)48 << 20) / (ranges * full_row);
  if (pf > p.nominal + (p.nom_rem > 0)) pf = p.nominal + (p.nom_rem > 0);
  p.pf_rows = (int)(pf < 1 ? 1 : pf);
  const size_t smem = off_stage + S * stage;
  return finish(run_rows(dtype, p, norm, group_vec(kVec, G), dim3((unsigned)(ranges * nsplit)),
                         dim3((unsigned)(32 + dcta / kVec)), smem, stream));
}

cudaError_t run_bwd_rows(int dtype, const BwdRowsParams& p, int norm, int gv, dim3 grid, dim3 block, size_t smem,
                         void* stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case GRETA_DT_F32: return launch_bwd_rows_f32(with_bwd_strides(p), norm, gv, grid, block, smem, st);
    case GRETA_DT_F16: return launch_bwd_rows_f16(with_bwd_strides(p), norm, gv, grid, block, smem, st);
    default: return launch_bwd_rows_bf16(with_bwd_strides(p), norm, gv, grid, block, smem, st);
  }
}

// Launch the row-streaming TMA backward when it applies: rows of whole
// 256-channel blocks (split over CTAs of at most bwd_rows_max_channels),
// W <= kMaxWBwdRows, 16-byte aligned tensors and copies, at most kMaxSeqsTma
// sequences, and room for two stages of token rows (x, filters, dout, gate,
// saved pre-norm output). Returns -1 when it does not.
int try_rows_bwd(int dtype, BwdRowsParams p, int norm, void* stream, const Opts& o) {
  if (o.kernel != GRETA_KERNEL_AUTO && o.kernel != GRETA_KERNEL_ROWS) return -1;
  p = with_bwd_strides(p);
  p.wait_log2 = o.wait_log2;
  const int es = esize(dtype);
  // bulk copies and vector stores start on 16-byte boundaries: row strides too
  for (long long ld : {p.ldx, p.ldg, p.ldw, p.lddx, p.lddg})
    if ((ld * es) % 16 != 0) return -1;
  const int64_t D = p.D, W = p.W, G = p.G, DC = D / G;
  if (D % 256 != 0 || W > kMaxWBwdRows) return -1;
  if (p.mode == kModePacked && p.nseq > kMaxSeqsTma) return -1;
  for (const void* q : {p.x, p.w, p.g, p.yr, p.dout, (const void*)p.dx, (const void*)p.dw, (const void*)p.dg})
    if (!aligned(q, 16)) return -1;
  // the W template launch_bwd_rows picks: 4, 7 or -kMaxWBwdRows
  const int wt = W == 4 ? 4 : (W == 7 ? 7 : -kMaxWBwdRows);
  int64_t cmax = bwd_rows_max_channels(wt, group_vec(kVec, G));
  if (o.rows_channels > 0 && o.rows_channels < cmax) cmax = o.rows_channels;
  const int64_t dcta = slice_channels(D, cmax);
  if (dcta == 0) return -1;
  const int64_t nsplit = D / dcta;
  if ((W * DC * es) % 16 != 0) return -1;
  // split filter rows per tap when whole rows would be re-read by many CTAs
  const bool wsplit = nsplit > 1 && W * DC * es > 2048;
  if (wsplit && ((dcta / G) * es) % 16 != 0) return -1;
  const int64_t rowx = dcta * es, roww = wsplit ? W * (dcta / G) * es : W * DC * es;
  const bool gate = p.g != nullptr, has_yr = norm != GRETA_NORM_NONE;
  const bool packed = p.mode == kModePacked;
  const size_t off_stage = packed ? a128((size_t)(p.nseq + 1) * 8) : 0;
  const size_t budget = (size_t)o.rows_smem;
  if (off_stage >= budget) return -1;
  const int64_t per_token = 2 * rowx + roww + (gate ? rowx : 0) + (has_yr ? rowx : 0);
  const int64_t inflight = (int64_t)(budget - off_stage) / per_token;
  if (inflight < 2) return -1;
  int S, BT;
  if (inflight >= 8) {
    S = 4;
    BT = (int)(inflight / 4 < 16 ? inflight / 4 : 16);
  } else {
    S = (int)(inflight < kMaxStages ? inflight : kMaxStages);
    BT = 1;
  }
  size_t so_w, so_do, so_g, so_yr, stage;
  for (;;) {
    so_w = a128((size_t)BT * rowx);
    so_do = so_w + a128((size_t)BT * roww);
    so_g = so_do + a128((size_t)BT * rowx);
    so_yr = so_g + (gate ? a128((size_t)BT * rowx) : 0);
    stage = so_yr + (has_yr ? a128((size_t)BT * rowx) : 0);
    if (off_stage + S * stage <= budget || (BT == 1 && S == 2)) break;
    if (BT > 1) --BT; else --S;
  }
  if (off_stage + S * stage > budget) return -1;
  p.BT = BT;
  p.stages = S;
  p.off_bnd = 0;
  p.off_stage = (int)off_stage;
  p.stage_bytes = (int)stage;
  p.so_w = (int)so_w;
  p.so_do = (int)so_do;
  p.so_g = (int)so_g;
  p.so_yr = (int)so_yr;
  p.dcta = (int)dcta;
  p.nsplit = (int)nsplit;
  p.wsplit = wsplit ? 1 : 0;
  long long ranges = o.rows_ranges > 0 ? o.rows_ranges : num_sms() / nsplit;
  if (ranges < 1) ranges = 1;
  if (p.T < ranges) ranges = p.T;
  if (ranges <= 0) return GRETA_OK;
  const size_t smem = off_stage + S * stage;
  return finish(run_bwd_rows(dtype, p, norm, group_vec(kVec, G), dim3((unsigned)(ranges * nsplit)),
                             dim3((unsigned)bwd_rows_threads(wt, group_vec(kVec, G), (int)dcta)), smem, stream));
}

// A run must cover the W-1 history positions: a request's old slot taps are
// then only read by row 0 of its first chunk.
Shape shape_for(int path, int H, const Opts& o) {
  Shape s = o.shape.tx > 0 ? o.shape : kDefaultShape[path];
  if (s.L < H) s.L = H;
  if (s.L < 1) s.L = 1;
  return s;
}

}  // namespace

extern "C" {

int greta_dynconv_fwd_ex(int dtype, const void* x, const void* w, const void* gate, void* y, void* yr,
                         const void* cu_seqlens, int cu_seqlens_int64, int64_t num_seqs, int64_t T,
                         int64_t D, int64_t W, int64_t G, int norm, float eps, void* stream,
                         const greta_dynconv_options* opt) {
  return greta_dynconv_fwd_ld_ex(dtype, x, D, w, W * (G > 0 ? D / G : 0), gate, D, y, yr, cu_seqlens,
                                 cu_seqlens_int64, num_seqs, T, D, W, G, norm, eps, stream, opt);
}

int greta_dynconv_fwd_ld_ex(int dtype, const void* x, int64_t ldx, const void* w, int64_t ldw, const void* gate,
                            int64_t ldg, void* y, void* yr, const void* cu_seqlens, int cu_seqlens_int64,
                            int64_t num_seqs, int64_t T, int64_t D, int64_t W, int64_t G, int norm, float eps,
                            void* stream, const greta_dynconv_options* opt) {
  Opts o;
  int rc = parse_opts(opt, o);
  if (rc) return rc;
  rc = check_common(dtype, D, W, G, norm);
  if (rc) return rc;
  if (T < 0 || (cu_seqlens && num_seqs < 0)) return GRETA_ERR_INVALID_ARG;
  if (ldx < D || ldg < D || ldw < W * (D / G)) return GRETA_ERR_INVALID_ARG;
  if (T == 0 || (cu_seqlens && num_seqs == 0)) return GRETA_OK;  // empty tensors may have null pointers
  if (!x || !w || !y) return GRETA_ERR_INVALID_ARG;
  int nv = pick_nv(dtype, D, G, {x, gate, y, yr}, w);
  if (nv == kVec && !strides_vec_ok(dtype, G, {ldx, gate ? ldg : D}, {ldw})) nv = G > 32 ? 0 : 1;
  if (nv == 0) return GRETA_ERR_ALIGNMENT;
  if (nv == kVec) {
    RowsParams tp{};
    tp.x = x; tp.w = w; tp.g = gate; tp.y = y; tp.yr = norm != GRETA_NORM_NONE ? yr : nullptr;
    tp.starts = cu_seqlens; tp.starts_i64 = cu_seqlens_int64 ? 1 : 0;
    tp.mode = cu_seqlens ? kModePacked : kModeSingle;
    tp.nseq = cu_seqlens ? num_seqs : 1;
    tp.T = T; tp.U = T; tp.D = (int)D; tp.W = (int)W; tp.G = (int)G;
    tp.eps = eps;
    tp.ldx = ldx; tp.ldg = ldg; tp.ldw = ldw;
    const int r = try_rows_fwd(dtype, tp, gate != nullptr, norm, stream, o);
    if (r >= 0) return r;
  }
  const Shape sh = shape_for(kPathFwd, (int)W - 1, o);
  FwdParams p{};
  p.x = x; p.w = w; p.g = gate; p.y = y; p.yr = norm != GRETA_NORM_NONE ? yr : nullptr;
  p.starts = cu_seqlens; p.starts_i64 = cu_seqlens_int64 ? 1 : 0;
  p.mode = cu_seqlens ? kModePacked : kModeSingle;
  p.nseq = cu_seqlens ? num_seqs : 1;
  p.T = T; p.D = (int)D; p.W = (int)W; p.G = (int)G;
  p.L = sh.L; p.chunk = sh.L * sh.ty;
  p.eps = eps;
  p.ldx = ldx; p.ldg = ldg; p.ldw = ldw;
  const long long chunks = cdiv(T, p.chunk) + (cu_seqlens ? num_seqs : 0);
  if (chunks * (D / 8 + 1) > INT_MAX) return GRETA_ERR_INVALID_ARG;
  return finish(run_fwd(dtype, p, nv, norm, make_shape(chunks, D, nv, sh.tx, sh.ty), stream));
}

int greta_dynconv_bwd_ex(int dtype, const void* x, const void* w, const void* gate, const void* yr,
                         const void* dout, void* dx, void* dw, void* dg, const void* cu_seqlens,
                         int cu_seqlens_int64, int64_t num_seqs, int64_t T, int64_t D, int64_t W,
                         int64_t G, int norm, float eps, void* stream, const greta_dynconv_options* opt) {
  const int64_t wr = W * (G > 0 ? D / G : 0);
  return greta_dynconv_bwd_ld_ex(dtype, x, D, w, wr, gate, D, yr, dout, dx, D, dw, wr, dg, D, cu_seqlens,
                                 cu_seqlens_int64, num_seqs, T, D, W, G, norm, eps, stream, opt);
}

int greta_dynconv_bwd_ld_ex(int dtype, const void* x, int64_t ldx, const void* w, int64_t ldw, const void* gate,
                            int64_t ldg, const void* yr, const void* dout, void* dx, int64_t lddx, void* dw,
                            int64_t lddw, void* dg, int64_t lddg, const void* cu_seqlens, int cu_seqlens_int64,
                            int64_t num_seqs, int64_t T, int64_t D, int64_t W, int64_t G, int norm, float eps,
                            void* stream, const greta_dynconv_options* opt) {
  Opts o;
  int rc = parse_opts(opt, o);
  if (rc) return rc;
  rc = check_common(dtype, D, W, G, norm);
  if (rc) return rc;
  if (norm == GRETA_NORM_STABLE) return GRETA_ERR_UNSUPPORTED;
  if (T < 0 || (cu_seqlens && num_seqs < 0)) return GRETA_ERR_INVALID_ARG;
  if (ldx < D || ldg < D || lddx < D || lddg < D || ldw < W * (D / G) || lddw < W * (D / G))
    return GRETA_ERR_INVALID_ARG;
  if (T == 0 || (cu_seqlens && num_seqs == 0)) return GRETA_OK;  // empty tensors may have null pointers
  if (!x || !w || !dout || !dx || !dw) return GRETA_ERR_INVALID_ARG;
  if ((gate == nullptr) != (dg == nullptr)) return GRETA_ERR_INVALID_ARG;
  if (norm != GRETA_NORM_NONE && yr == nullptr) return GRETA_ERR_INVALID_ARG;
  int nv = pick_nv(dtype, D, G, {x, gate, yr, dout, dx, dg}, w);
  if (nv == kVec && !aligned(dw, (int64_t)group_vec(kVec, G) * esize(dtype))) nv = G > 32 ? 0 : 1;
  if (nv == kVec && !strides_vec_ok(dtype, G, {ldx, gate ? ldg : D, lddx, gate ? lddg : D}, {ldw, lddw}))
    nv = G > 32 ? 0 : 1;
  if (nv == 0) return GRETA_ERR_ALIGNMENT;
  if (nv == kVec) {
    BwdRowsParams tp{};
    tp.x = x; tp.w = w; tp.g = gate; tp.yr = norm != GRETA_NORM_NONE ? yr : nullptr; tp.dout = dout;
    tp.dx = dx; tp.dw = dw; tp.dg = dg;
    tp.starts = cu_seqlens; tp.starts_i64 = cu_seqlens_int64 ? 1 : 0;
    tp.mode = cu_seqlens ? kModePacked : kModeSingle;
    tp.nseq = cu_seqlens ? num_seqs : 1;
    tp.T = T; tp.D = (int)D; tp.W = (int)W; tp.G = (int)G;
    tp.eps = eps;
    tp.ldx = ldx; tp.ldg = ldg; tp.ldw = ldw; tp.lddx = lddx; tp.lddg = lddg; tp.lddw = lddw;
    const int r = try_rows_bwd(dtype, tp, norm, stream, o);
    if (r >= 0) return r;
  }
  const Shape sh = shape_for(kPathBwd, (int)W - 1, o);
  BwdParams p{};
  p.x = x; p.w = w; p.g = gate; p.yr = norm != GRETA_NORM_NONE ? yr : nullptr; p.dout = dout;
  p.dx = dx; p.dw = dw; p.dg = dg;
  p.starts = cu_seqlens; p.starts_i64 = cu_seqlens_int64 ? 1 : 0;
  p.mode = cu_seqlens ? kModePacked : kModeSingle;
  p.nseq = cu_seqlens ? num_seqs : 1;
  p.T = T; p.D = (int)D; p.W = (int)W; p.G = (int)G;
  p.L = sh.L; p.chunk = sh.L * sh.ty;
  p.eps = eps;
  p.ldx = ldx; p.ldg = ldg; p.ldw = ldw; p.lddx = lddx; p.lddg = lddg; p.lddw = lddw;
  const long long chunks = cdiv(T, p.chunk) + (cu_seqlens ? num_seqs : 0);
  if (chunks * (D / 8 + 1) > INT_MAX) return GRETA_ERR_INVALID_ARG;
  return finish(run_bwd(dtype, p, nv, norm, make_shape(chunks, D, nv, sh.tx, sh.ty), stream));
}

int greta_dynconv_inference_ex(int dtype, const void* context, const void* w, const void* gate, void* y,
                               int64_t B, int64_t Q, int64_t D, int64_t W, int64_t G, int norm, float eps,
                               void* stream, const greta_dynconv_options* opt) {
  Opts o;
  int rc = parse_opts(opt, o);
  if (rc) return rc;
  rc = check_common(dtype, D, W, G, norm);
  if (rc) return rc;
  if (B < 0 || Q < 0) return GRETA_ERR_INVALID_ARG;
  if (B == 0 || Q == 0) return GRETA_OK;  // empty tensors may have null pointers
  if (!context || !w || !y) return GRETA_ERR_INVALID_ARG;
  const int nv = pick_nv(dtype, D, G, {context, gate, y}, w);
  if (nv == 0) return GRETA_ERR_ALIGNMENT;
  if (nv == kVec) {
    RowsParams tp{};
    tp.x = context; tp.w = w; tp.g = gate; tp.y = y; tp.yr = nullptr;
    tp.mode = kModeContext;
    tp.nseq = B;
    tp.T = Q; tp.U = B * Q; tp.D = (int)D; tp.W = (int)W; tp.G = (int)G;
    tp.eps = eps;
    const int r = try_rows_fwd(dtype, tp, gate != nullptr, norm, stream, o);
    if (r >= 0) return r;
  }
  const Shape sh = shape_for(kPathInference, (int)W - 1, o);
  FwdParams p{};
  p.x = context; p.w = w; p.g = gate; p.y = y; p.yr = nullptr;
  p.mode = kModeContext;
  p.nseq = B;
  p.T = Q; p.D = (int)D; p.W = (int)W; p.G = (int)G;
  p.L = sh.L; p.chunk = sh.L * sh.ty;
  p.eps = eps;
  const long long chunks = B * cdiv(Q, p.chunk);
  if (chunks * (D / 8 + 1) > INT_MAX) return GRETA_ERR_INVALID_ARG;
  return finish(run_fwd(dtype, p, nv, norm, make_shape(chunks, D, nv, sh.tx, sh.ty), stream));
}

int greta_dynconv_decode_rows_ex(int dtype, const void* x, const void* w, const void* gate, void* conv_state,
                                 void* y, int64_t B, int64_t D, int64_t W, int64_t G, int norm, float eps,
                                 void* stream, const greta_dynconv_options* opt) {
  Opts o;
  int rc = parse_opts(opt, o);
  if (rc) return rc;
  rc = check_common(dtype, D, W, G, norm);
  if (rc) return rc;
  if (B < 0 || W < 2) return GRETA_ERR_INVALID_ARG;
  if (B == 0) return GRETA_OK;  // empty tensors may have null pointers
  if (!x || !w || !conv_state || !y) return GRETA_ERR_INVALID_ARG;
  if (B > INT_MAX) return GRETA_ERR_INVALID_ARG;
  const int nv = pick_nv(dtype, D, G, {x, gate, y}, w);
  if (nv == 0) return GRETA_ERR_ALIGNMENT;
  const int H = (int)W - 1;
  const int es = esize(dtype);
  FwdParams p{};
  p.x = x; p.w = w; p.g = gate; p.y = y; p.yr = nullptr;
  p.mode = kModeRows;
  p.nseq = B;
  p.T = B; p.D = (int)D; p.W = (int)W; p.G = (int)G;
  p.L = 1; p.chunk = 1;  // one token per request
  p.state = conv_state;
  p.s_slot = D * H; p.s_d = H; p.s_h = 1; p.num_slots = B;
  p.st_layout = (nv == kVec && aligned(conv_state, (int64_t)kVec * es)) ? kStDS : kStGeneric;
  p.eps = eps;
  const Shape sh = shape_for(kPathDecodeRows, H, o);
  if (nv == kVec && (W == 4 || W == 7) && p.st_layout == kStDS && sh.tx <= 128)
    return finish(run_fwd_decode(dtype, p, norm, make_shape(B, D, nv, sh.tx, 1), stream));
  return finish(run_fwd(dtype, p, nv, norm, make_shape(B, D, nv, sh.tx, 1), stream));
}

int greta_dynconv_packed_state_ex(int dtype, const void* x, const void* w, const void* gate, void* y,
                                  void* state, int64_t num_slots, int64_t s_slot, int64_t s_d, int64_t s_h,
                                  const int32_t* starts, const int32_t* slots, const int8_t* has_initial,
                                  int64_t num_reqs, int64_t T, int64_t D, int64_t W, int64_t G, int norm,
                                  float eps, int32_t* error_flags, void* stream, const greta_dynconv_options* opt) {
  return greta_dynconv_packed_state_ld_ex(dtype, x, D, w, W * (G > 0 ? D / G : 0), gate, D, y, state, num_slots,
                                          s_slot, s_d, s_h, starts, slots, has_initial, num_reqs, T, D, W, G, norm,
                                          eps, error_flags, stream, opt);
}

int greta_dynconv_packed_state_ld_ex(int dtype, const void* x, int64_t ldx, const void* w, int64_t ldw,
                                     const void* gate, int64_t ldg, void* y, void* state, int64_t num_slots,
                                     int64_t s_slot, int64_t s_d, int64_t s_h, const int32_t* starts,
                                     const int32_t* slots, const int8_t* has_initial, int64_t num_reqs, int64_t T,
                                     int64_t D, int64_t W, int64_t G, int norm, float eps, int32_t* error_flags,
                                     void* stream, const greta_dynconv_options* opt) {
  Opts o;
  int rc = parse_opts(opt, o);
  if (rc) return rc;
  rc = check_common(dtype, D, W, G, norm, D);
  if (rc) return rc;
  const int H = (int)W - 1;
  if (T < 0 || num_reqs < 0 || num_slots < 0) return GRETA_ERR_INVALID_ARG;
  if (ldx < D || ldg < D || ldw < W * (D / G)) return GRETA_ERR_INVALID_ARG;
  if (T == 0 || num_reqs == 0) return GRETA_OK;  // empty tensors may have null pointers
  if (!x || !w || !y || !starts || !slots || !has_initial) return GRETA_ERR_INVALID_ARG;
  if (H > 0 && !state && num_slots > 0) return GRETA_ERR_INVALID_ARG;
  int nv = pick_nv(dtype, D, G, {x, gate, y}, w);
  if (nv == kVec && !strides_vec_ok(dtype, G, {ldx, gate ? ldg : D}, {ldw})) nv = G > 32 ? 0 : 1;
  if (nv == 0) return GRETA_ERR_ALIGNMENT;
  const int es = esize(dtype);
  const bool decode_like = T <= 2 * num_reqs;
  const Shape sh = shape_for(decode_like ? kPathPackedDecode : kPathPackedPrefill, H, o);
  FwdParams p{};
  p.x = x; p.w = w; p.g = gate; p.y = y; p.yr = nullptr;
  p.starts = starts; p.starts_i64 = 0;
  p.mode = kModePacked;
  p.nseq = num_reqs;
  p.T = T; p.D = (int)D; p.W = (int)W; p.G = (int)G;
  p.L = sh.L; p.chunk = sh.L * sh.ty;
  p.slots = slots;
  p.initial = reinterpret_cast<const signed char*>(has_initial);
  p.err = error_flags;
  p.eps = eps;
  p.ldx = ldx; p.ldg = ldg; p.ldw = ldw;
  if (H > 0 && state != nullptr && num_slots > 0) {
    p.state = state;
    p.s_slot = s_slot; p.s_d = s_d; p.s_h = s_h; p.num_slots = num_slots;
    const bool base_ok = nv == kVec && aligned(state, (int64_t)kVec * es) && s_slot % kVec == 0;
    if (base_ok && s_h == 1 && s_d == H)
      p.st_layout = kStDS;
    else if (base_ok && s_d == 1 && s_h % kVec == 0)
      p.st_layout = kStSD;
    else
      p.st_layout = kStGeneric;
  } else {
    // No history storage (W == 1, or an empty cache): every slot reads as
    // "no history" and nothing is written back.
    p.state = nullptr;
    p.num_slots = 0;
  }
  if (G > 256) {
    // groups wider than one warp's 256 channels: each CTA owns one whole
    // group of a chunk of kWideChunk tokens (dynconv_fwd_wide.cuh)
    if (nv != kVec) return GRETA_ERR_ALIGNMENT;
    p.L = p.chunk = kWideChunk;
    const long long groups = D / G;
    const long long rows = cdiv(T, p.chunk) + num_reqs;
    if (rows * groups > INT_MAX) return GRETA_ERR_INVALID_ARG;
    const int threads = (int)(G / kVec < kWideThreads ? G / kVec : kWideThreads);
    return finish(run_fwd_wide(dtype, p, norm, dim3((unsigned)(rows * groups)), dim3((unsigned)threads), (int)groups,
                               stream));
  }
  if (!decode_like && nv == kVec) {
    RowsParams tp{};
    tp.x = x; tp.w = w; tp.g = gate; tp.y = y; tp.yr = nullptr;
    tp.starts = starts; tp.starts_i64 = 0;
    tp.mode = kModePacked;
    tp.nseq = num_reqs;
    tp.T = T; tp.U = T; tp.D = (int)D; tp.W = (int)W; tp.G = (int)G;
    tp.state = p.state; tp.s_slot = p.s_slot; tp.s_d = p.s_d; tp.s_h = p.s_h; tp.num_slots = p.num_slots;
    tp.st_layout = p.st_layout; tp.slots = slots; tp.initial = p.initial; tp.err = error_flags;
    tp.eps = eps;
    tp.ldx = ldx; tp.ldg = ldg; tp.ldw = ldw;
    const int r = try_rows_fwd(dtype, tp, gate != nullptr, norm, stream, o);
    if (r >= 0) return r;
  }
  if (decode_like && nv == kVec && (W == 4 || W == 7) && sh.ty == 1 && sh.tx <= 128 && T < INT_MAX &&
      num_slots < INT_MAX && (p.state == nullptr || p.st_layout == kStDS || p.st_layout == kStSD)) {
    // decode kernel: each request's first chunk of C tokens (C >= W-1) on CTA
    // row r < num_reqs, then at most (T-1)/C later chunks of longer requests
    p.L = p.chunk = sh.L;
    const long long chunks = num_reqs + (T - 1) / p.chunk;
    if (chunks * (D / 8 + 1) > INT_MAX) return GRETA_ERR_INVALID_ARG;
    return finish(run_fwd_decode(dtype, p, norm, make_shape(chunks, D, nv, sh.tx, 1), stream));
  }
  const long long chunks = cdiv(T, p.chunk) + num_reqs;
  if (chunks * (D / 8 + 1) > INT_MAX) return GRETA_ERR_INVALID_ARG;
  return finish(run_fwd(dtype, p, nv, norm, make_shape(chunks, D, nv, sh.tx, sh.ty), stream));
}

int greta_dynconv_fwd(int dtype, const void* x, const void* w, const void* gate, void* y, void* yr,
                      const void* cu_seqlens, int cu_seqlens_int64, int64_t num_seqs, int64_t T, int64_t D,
                      int64_t W, int64_t G, int norm, float eps, void* stream) {
  return greta_dynconv_fwd_ex(dtype, x, w, gate, y, yr, cu_seqlens, cu_seqlens_int64, num_seqs, T, D, W, G, norm,
                              eps, stream, nullptr);
}

int greta_dynconv_bwd(int dtype, const void* x, const void* w, const void* gate, const void* yr, const void* dout,
                      void* dx, void* dw, void* dg, const void* cu_seqlens, int cu_seqlens_int64, int64_t num_seqs,
                      int64_t T, int64_t D, int64_t W, int64_t G, int norm, float eps, void* stream) {
  return greta_dynconv_bwd_ex(dtype, x, w, gate, yr, dout, dx, dw, dg, cu_seqlens, cu_seqlens_int64, num_seqs, T, D,
                              W, G, norm, eps, stream, nullptr);
}

int greta_dynconv_inference(int dtype, const void* context, const void* w, const void* gate, void* y, int64_t B,
                            int64_t Q, int64_t D, int64_t W, int64_t G, int norm, float eps, void* stream) {
  return greta_dynconv_inference_ex(dtype, context, w, gate, y, B, Q, D, W, G, norm, eps, stream, nullptr);
}

int greta_dynconv_decode_rows(int dtype, const void* x, const void* w, const void* gate, void* conv_state, void* y,
                              int64_t B, int64_t D, int64_t W, int64_t G, int norm, float eps, void* stream) {
  return greta_dynconv_decode_rows_ex(dtype, x, w, gate, conv_state, y, B, D, W, G, norm, eps, stream, nullptr);
}

int greta_dynconv_packed_state(int dtype, const void* x, const void* w, const void* gate, void* y, void* state,
                               int64_t num_slots, int64_t s_slot, int64_t s_d, int64_t s_h, const int32_t* starts,
                               const int32_t* slots, const int8_t* has_initial, int64_t num_reqs, int64_t T,
                               int64_t D, int64_t W, int64_t G, int norm, float eps, int32_t* error_flags,
                               void* stream) {
  return greta_dynconv_packed_state_ex(dtype, x, w, gate, y, state, num_slots, s_slot, s_d, s_h, starts, slots,
                                       has_initial, num_reqs, T, D, W, G, norm, eps, error_flags, stream, nullptr);
}

int greta_dynconv_device_errors(int clear) {
  const bool cl = clear != 0;
  const int v[6] = {device_errors_f32(cl),           device_errors_f16(cl),           device_errors_bf16(cl),
                    device_errors_bwd_rows_f32(cl), device_errors_bwd_rows_f16(cl), device_errors_bwd_rows_bf16(cl)};
  int all = 0;
  for (int e : v) {
    if (e < 0) return -1;
    all |= e;
  }
  return all;
}

int greta_dynconv_supports(int64_t group_size, int64_t channels) {
  return (is_pow2(group_size) && channels > 0 && channels % group_size == 0) ? 1 : 0;
}

const char* greta_dynconv_status_string(int status) {
  switch (status) {
    case GRETA_OK: return "ok";
    case GRETA_ERR_INVALID_ARG: return "invalid argument (null pointer, negative size or shape mismatch)";
    case GRETA_ERR_UNSUPPORTED: return "unsupported configuration (dtype, group size, kernel size or norm kind)";
    case GRETA_ERR_ALIGNMENT: return "misaligned pointer for the vector path with group size > 32";
    case GRETA_ERR_LAUNCH: return "CUDA kernel launch failed";
    default: return "unknown status";
  }
}

int greta_dynconv_version(void) { return kAbiVersion; }

}  // extern "C"
