/*
 * greta_dynconv.h -- C ABI of the B200 (sm_100a) dynamic causal depthwise
 * convolution library (libgreta_dynconv.so).
 *
 * The operator, for token t, channel d, taps k = 0..W-1 and G channels per
 * shared filter:
 *
 *   y[t,d]   = sum_k w[t, k, d / G] * x[t + k - W + 1, d]   (tap W-1 = current token)
 *   out[t,d] = GroupRMSNorm_G(y)[t,d] * SiLU(g[t,d])          (norm and gate optional)
 *
 * History before a sequence's first token is zero (training), comes from an
 * explicit context (HF inference), or from a per-request cache slot holding
 * the previous W-1 inputs (vLLM packed batches, HF decode).
 *
 * Conventions shared by every entry point:
 *   - All tensor pointers are DEVICE pointers on the current CUDA device.
 *     Tensors are dense row-major (the innermost dimension is contiguous)
 *     unless explicit strides are passed.
 *   - `dtype` is one of GRETA_DT_*; x, w, gate, outputs and state all have
 *     that element type. Accumulation is fp32; every output is rounded once
 *     (round-to-nearest-even).
 *   - `stream` is a cudaStream_t (NULL = legacy default stream). Calls only
 *     enqueue kernels: no allocation, no host synchronisation, so they can be
 *     issued while a stream is being captured into a CUDA graph.
 *   - Return value: GRETA_OK or one of the GRETA_ERR_* codes below. On an
 *     argument error nothing is launched.
 *   - The group size G must be a power of two dividing D, with G <= 256,
 *     except for greta_dynconv_packed_state, which takes any power of two
 *     dividing D (as the reference's vLLM path does). The kernel size W must
 *     be in [1, 16] (the decode entry points need W >= 2).
 *   - Every entry point has an `_ex` form with a trailing
 *     `const greta_dynconv_options*` (NULL = the plain form's behaviour):
 *     per-call launch choices for tests and tuning sweeps. The library keeps
 *     no process-wide settings.
 *   - Weights are compact and tap-major: w[t, k, f] with f = d / G.
 */
#ifndef GRETA_DYNCONV_H
#define GRETA_DYNCONV_H

#include <stdint.h>

#if defined(__GNUC__)
#define GRETA_API __attribute__((visibility("default")))
#else
#define GRETA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* element types */
#define GRETA_DT_F32 0
#define GRETA_DT_F16 1
#define GRETA_DT_BF16 2

/* group RMS-norm variants */
#define GRETA_NORM_NONE 0
/* y * rsqrt(mean_G(y^2) + eps): greta/dynamic_conv.py:251-255 (training and HF kernels) */
#define GRETA_NORM_PLAIN 1
/* overflow-safe max-abs rescaled form: greta_vllm/triton_conv.py:71-77 (vLLM path) */
#define GRETA_NORM_STABLE 2

/* status codes */
#define GRETA_OK 0
#define GRETA_ERR_INVALID_ARG 1 /* null pointer, negative size, shape mismatch */
#define GRETA_ERR_UNSUPPORTED 2 /* G not a power of two (or > 256 where noted), W out of range, dtype */
#define GRETA_ERR_ALIGNMENT 3   /* a pointer or stride breaks the vector-path alignment */
#define GRETA_ERR_LAUNCH 4      /* the CUDA launch itself failed */

/*
 * Packed variable-length forward (training and plain inference).
 * Replaces dynconv_fwd / dynconv_fwd_kernel, greta/dynamic_conv.py:786-823 and
 * :179-261 (called by DynamicCausalConv1dFunction.forward, :867-882, and
 * dynamic_causal_conv1d, :896-931).
 *
 *   x, gate, y, yr : [T, D]   (the reference's [1, T, D])
 *   w              : [T, W, D/G]
 *   cu_seqlens     : [num_seqs + 1] cumulative sequence offsets (int32, or
 *                    int64 when cu_seqlens_int64 != 0); NULL = one sequence of
 *                    T tokens. Offsets are clamped to [0, T] on the device.
 *   gate           : NULL = no gate
 *   yr             : NULL, or receives the pre-norm conv output (saved for the
 *                    backward when norm != NONE; the reference's SAVE_PRE)
 *   norm           : GRETA_NORM_NONE or GRETA_NORM_PLAIN
 */
GRETA_API int greta_dynconv_fwd(int dtype, const void* x, const void* w, const void* gate, void* y,
                      void* yr, const void* cu_seqlens, int cu_seqlens_int64,
                      int64_t num_seqs, int64_t T, int64_t D, int64_t W, int64_t G,
                      int norm, float eps, void* stream);

/*
 * Packed variable-length backward: dx, compact dw and dg in one pass.
 * Replaces dynconv_bwd / dynconv_bwd_kernel, greta/dynamic_conv.py:826-864 and
 * :271-428 (called by DynamicCausalConv1dFunction.backward, :884-893).
 *
 *   dout, dx, dg : [T, D];  dw : [T, W, D/G] (same element type as w)
 *   yr           : pre-norm output from the forward; required when norm != NONE
 *   gate / dg    : both NULL or both non-NULL
 */
GRETA_API int greta_dynconv_bwd(int dtype, const void* x, const void* w, const void* gate,
                      const void* yr, const void* dout, void* dx, void* dw, void* dg,
                      const void* cu_seqlens, int cu_seqlens_int64, int64_t num_seqs,
                      int64_t T, int64_t D, int64_t W, int64_t G, int norm, float eps,
                      void* stream);

/*
 * Batched forward from an explicit context (HF prefill with cache).
 * Replaces dynamic_causal_conv1d_inference / dynconv_inference_kernel,
 * greta/dynamic_conv.py:643-687 and :435-506.
 *
 *   context : [B, Q + W - 1, D]  (W-1 history tokens, then the Q query tokens)
 *   w       : [B, Q, W, D/G];  gate, y : [B, Q, D]
 *   norm    : GRETA_NORM_NONE or GRETA_NORM_PLAIN
 */
GRETA_API int greta_dynconv_inference(int dtype, const void* context, const void* w, const void* gate,
                            void* y, int64_t B, int64_t Q, int64_t D, int64_t W, int64_t G,
                            int norm, float eps, void* stream);

/*
 * Single-token decode keyed by batch row, with the in-place state shift.
 * Replaces dynamic_causal_conv1d_decode / dynconv_decode_kernel,
 * greta/dynamic_conv.py:722-765 and :513-602.
 *
 *   x, gate, y : [B, D];  w : [B, W, D/G]
 *   conv_state : [B, D, W-1] contiguous, chronological; updated in place to
 *                (old[1:], x). Requires W >= 2.
 *   norm       : GRETA_NORM_NONE or GRETA_NORM_PLAIN
 */
GRETA_API int greta_dynconv_decode_rows(int dtype, const void* x, const void* w, const void* gate,
                              void* conv_state, void* y, int64_t B, int64_t D, int64_t W,
                              int64_t G, int norm, float eps, void* stream);

/*
 * vLLM packed batch (chunked prefill and decode) with cache-slot history and
 * the fused state write-back. Replaces packed_dynamic_conv_triton and its two
 * kernels _conv_kernel / _state_kernel, greta_vllm/triton_conv.py:128-173,
 * :28-84 and :87-116 (torch form: greta_vllm/conv.py:10-70).
 *
 *   x, gate, y : [T, D];  w : [T, W, D/G]
 *   state      : [num_slots, D, W-1] addressed through element strides
 *                (s_slot, s_d, s_h), so both vLLM orientations (dim-first
 *                "DS" and the transposed "SD" view) are read in place.
 *   starts     : [num_reqs + 1] int32 cumulative token offsets (decodes first)
 *   slots      : [num_reqs] int32 cache slot per request; < 0 = no history and
 *                no write-back (padding). A slot >= num_slots is treated the
 *                same way and flagged in *error_flags (bit 0) when non-NULL.
 *   has_initial: [num_reqs] int8; 0 = ignore the slot's old contents (zeros)
 *   norm       : GRETA_NORM_NONE, GRETA_NORM_PLAIN or GRETA_NORM_STABLE
 *                (the vLLM plugin uses STABLE)
 *   G          : any power of two dividing D; groups wider than 256 channels
 *                run on a kernel that gives each CTA one whole group
 *   error_flags: NULL, or a device int32 that receives OR-ed error bits
 *
 * After the call, each request's slot holds its last W-1 inputs (taken from
 * the chunk, or shifted from the old state when the chunk is shorter than
 * W-1) -- bit-exact copies of the input elements.
 */
GRETA_API int greta_dynconv_packed_state(int dtype, const void* x, const void* w, const void* gate,
                               void* y, void* state, int64_t num_slots, int64_t s_slot,
                               int64_t s_d, int64_t s_h, const int32_t* starts,
                               const int32_t* slots, const int8_t* has_initial,
                               int64_t num_reqs, int64_t T, int64_t D, int64_t W, int64_t G,
                               int norm, float eps, int32_t* error_flags, void* stream);

/*
 * Per-call launch options (no counterpart in the reference, whose Triton
 * kernels are autotuned). Pass to the `_ex` entry points; NULL, or a zeroed
 * struct with `size` set, means the built-in choices. Nothing here changes
 * results beyond floating-point summation order, except the test hooks,
 * which make a kernel stop early on purpose.
 */
/* kernel families, for greta_dynconv_options.kernel */
#define GRETA_KERNEL_AUTO 0     /* the library's choice per call */
#define GRETA_KERNEL_REGISTER 1 /* register-staged kernels only */
#define GRETA_KERNEL_ROWS 2     /* row-streaming (bulk-copy) kernels where the shape allows */

typedef struct greta_dynconv_options {
  int size;          /* sizeof(greta_dynconv_options); other sizes are rejected */
  int kernel;        /* GRETA_KERNEL_*: a family that does not apply to the call falls
                        back to the register-staged kernels; all give the same bits */
  int block_x;       /* register-kernel CTA shape: threads along channels (multiple of 32), */
  int block_y;       /* token runs per CTA (block_x * block_y <= 256) and */
  int tokens;        /* tokens per run (raised to at least W-1); any <= 0 = built-in shape */
  int wait_limit_log2; /* bound of each pipeline (mbarrier) wait in the row-streaming
                          kernels: 2^n polls, 8 <= n <= 24; 0 = 2^24 (about a second) */
  int test_withhold_release; /* test hook: != 0 makes consumer warp 0 of CTA 0 of the
                                row-streaming forward keep its first stage, so that the
                                producer's bounded wait runs out (device error bit 1, see
                                greta_dynconv_device_errors); the launch still returns */
  int rows_channels; /* row-streaming kernels: at most this many channels per CTA (the
                        widest multiple of 256 dividing D that fits); 0 = built-in */
  int rows_ranges;   /* row-streaming kernels: token ranges (CTAs = ranges x channel
                        slices); 0 = SMs / slices */
  int rows_smem_kb;  /* row-streaming kernels: shared-memory budget of the stage ring in
                        KiB (32..200); 0 = 200 */
} greta_dynconv_options;

GRETA_API int greta_dynconv_fwd_ex(int dtype, const void* x, const void* w, const void* gate, void* y,
                                   void* yr, const void* cu_seqlens, int cu_seqlens_int64,
                                   int64_t num_seqs, int64_t T, int64_t D, int64_t W, int64_t G,
                                   int norm, float eps, void* stream, const greta_dynconv_options* opt);
GRETA_API int greta_dynconv_bwd_ex(int dtype, const void* x, const void* w, const void* gate,
                                   const void* yr, const void* dout, void* dx, void* dw, void* dg,
                                   const void* cu_seqlens, int cu_seqlens_int64, int64_t num_seqs,
                                   int64_t T, int64_t D, int64_t W, int64_t G, int norm, float eps,
                                   void* stream, const greta_dynconv_options* opt);
GRETA_API int greta_dynconv_inference_ex(int dtype, const void* context, const void* w, const void* gate,
                                         void* y, int64_t B, int64_t Q, int64_t D, int64_t W, int64_t G,
                                         int norm, float eps, void* stream, const greta_dynconv_options* opt);
GRETA_API int greta_dynconv_decode_rows_ex(int dtype, const void* x, const void* w, const void* gate,
                                           void* conv_state, void* y, int64_t B, int64_t D, int64_t W,
                                           int64_t G, int norm, float eps, void* stream,
                                           const greta_dynconv_options* opt);
GRETA_API int greta_dynconv_packed_state_ex(int dtype, const void* x, const void* w, const void* gate,
                                            void* y, void* state, int64_t num_slots, int64_t s_slot,
                                            int64_t s_d, int64_t s_h, const int32_t* starts,
                                            const int32_t* slots, const int8_t* has_initial,
                                            int64_t num_reqs, int64_t T, int64_t D, int64_t W, int64_t G,
                                            int norm, float eps, int32_t* error_flags, void* stream,
                                            const greta_dynconv_options* opt);

/*
 * greta_dynconv_fwd / greta_dynconv_bwd with row strides (elements between
 * consecutive token rows): ldx, ldg, ldw for the inputs x, gate and filters,
 * and in the backward lddx, lddg, lddw for the outputs dx, dg and dw (y, yr
 * and dout stay contiguous [T, D]). With x, gate and filters the column
 * blocks of ONE projection GEMM's output [T, ld] (in_proj | gate_proj |
 * kernel_proj concatenated) and dx, dg, dw written into the matching column
 * blocks of one gradient buffer, the three projections' backward is one
 * GEMM for the hidden states' gradient and one for the weights'. Contiguous
 * strides make these the plain calls. No counterpart in the reference, which
 * runs three projections and their three backward GEMMs
 * (greta/modeling_greta.py:452-459).
 */
GRETA_API int greta_dynconv_fwd_ld_ex(int dtype, const void* x, int64_t ldx, const void* w, int64_t ldw,
                                      const void* gate, int64_t ldg, void* y, void* yr, const void* cu_seqlens,
                                      int cu_seqlens_int64, int64_t num_seqs, int64_t T, int64_t D, int64_t W,
                                      int64_t G, int norm, float eps, void* stream,
                                      const greta_dynconv_options* opt);
GRETA_API int greta_dynconv_bwd_ld_ex(int dtype, const void* x, int64_t ldx, const void* w, int64_t ldw,
                                      const void* gate, int64_t ldg, const void* yr, const void* dout, void* dx,
                                      int64_t lddx, void* dw, int64_t lddw, void* dg, int64_t lddg,
                                      const void* cu_seqlens, int cu_seqlens_int64, int64_t num_seqs, int64_t T,
                                      int64_t D, int64_t W, int64_t G, int norm, float eps, void* stream,
                                      const greta_dynconv_options* opt);

/*
 * greta_dynconv_packed_state with row strides for its inputs: ldx, ldg and ldw
 * are the distances in elements between consecutive token rows of x, gate and
 * the filters (x[t, d] at x + t*ldx + d, w[t, k, f] at w + t*ldw + k*(D/G) + f).
 * With ldx = ldg = D and ldw = W*D/G it is greta_dynconv_packed_state. Strided
 * inputs let x, gate and filters be column blocks of ONE projection GEMM's
 * output [T, ld] (in_proj | gate_proj | kernel_proj concatenated), read in
 * place instead of split into three tensors first. Requires ldx, ldg >= D,
 * ldw >= W*D/G; the vector kernels also need 16-byte aligned rows. y stays
 * contiguous [T, D]. No counterpart in the reference, which calls three
 * separate projections (greta_vllm/model.py:115-124).
 */
GRETA_API int greta_dynconv_packed_state_ld_ex(int dtype, const void* x, int64_t ldx, const void* w, int64_t ldw,
                                               const void* gate, int64_t ldg, void* y, void* state,
                                               int64_t num_slots, int64_t s_slot, int64_t s_d, int64_t s_h,
                                               const int32_t* starts, const int32_t* slots,
                                               const int8_t* has_initial, int64_t num_reqs, int64_t T, int64_t D,
                                               int64_t W, int64_t G, int norm, float eps, int32_t* error_flags,
                                               void* stream, const greta_dynconv_options* opt);

/*
 * Device-side error bits recorded by earlier kernels of this library on the
 * current device (bit 1, value 2: a pipeline wait of a row-streaming kernel
 * timed out and the kernel returned early, leaving part of its outputs
 * unwritten). Synchronises the device; clear != 0 resets the bits. Returns
 * the bits, or -1 when they cannot be read. For debugging and tests.
 */
GRETA_API int greta_dynconv_device_errors(int clear);

/* supports() of greta_vllm/triton_conv.py:119-121: G a power of two dividing
 * `channels` (the packed entry point's rule). */
GRETA_API int greta_dynconv_supports(int64_t group_size, int64_t channels);

/* Human-readable text for a status code (static storage). */
GRETA_API const char* greta_dynconv_status_string(int status);

/* Library ABI version: major * 10000 + minor * 100 + patch. */
GRETA_API int greta_dynconv_version(void);

#ifdef __cplusplus
}
#endif

#endif /* GRETA_DYNCONV_H */
