/*
 * dynconv_oracle.c -- CPU restatement of Greta's dynamic causal depthwise
 * convolution, used ONLY as test infrastructure: the parity checker of the
 * CUDA library and the timed CPU baseline. Nothing in the product path calls
 * it.
 *
 * Restated from the reference (Garbo-AI/greta-plugin):
 *   oracle_fwd         greta/dynamic_conv.py:937-962 torch_dynamic_causal_conv1d
 *                      (+ the pre-norm save of dynconv_fwd_kernel, :247-249)
 *   oracle_bwd         greta/dynamic_conv.py:319-428 dynconv_bwd_kernel math
 *                      (equal to autograd through torch_dynamic_causal_conv1d)
 *   oracle_inference   greta/dynamic_conv.py:467-506 dynconv_inference_kernel
 *   oracle_decode_rows greta/dynamic_conv.py:536-602 dynconv_decode_kernel
 *   oracle_packed      greta_vllm/triton_conv.py:41-116 (_conv_kernel followed
 *                      by _state_kernel); torch form greta_vllm/conv.py:10-70
 *
 * Every tensor is fp32, dense row-major, with the reference layouts:
 *   x [T, D], w [T, W, D/G] (compact, tap-major), gate [T, D], state
 *   [slots, D, W-1] through element strides. Arithmetic is double precision
 *   and the result is rounded to fp32 once, so the oracle is at least as exact
 *   as the reference's fp32 torch path it stands in for.
 *
 * Norm kinds: 0 none, 1 plain  y / sqrt(mean(y^2) + eps)
 *             (greta/dynamic_conv.py:251-255, :957-959),
 *             2 stable  s = max(max|y|, 1); y / (s sqrt(mean((y/s)^2) + eps/s^2))
 *             (greta_vllm/triton_conv.py:71-77, greta/modeling_greta.py:149-158).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static double sigmoid_d(double v) { return 1.0 / (1.0 + exp(-v)); }

/* Group RMS norm of one token row (D values), in place. */
static void norm_row(double* y, int64_t D, int64_t G, int kind, double eps) {
  if (kind == 0) return;
  for (int64_t f = 0; f < D / G; ++f) {
    double* v = y + f * G;
    if (kind == 1) {
      double ss = 0;
      for (int64_t c = 0; c < G; ++c) ss += v[c] * v[c];
      const double rinv = 1.0 / sqrt(ss / (double)G + eps);
      for (int64_t c = 0; c < G; ++c) v[c] *= rinv;
    } else {
      double mx = 0;
      for (int64_t c = 0; c < G; ++c) mx = fabs(v[c]) > mx ? fabs(v[c]) : mx;
      const double s = mx > 1.0 ? mx : 1.0;
      double ss = 0;
      for (int64_t c = 0; c < G; ++c) ss += (v[c] / s) * (v[c] / s);
      const double den = s * sqrt(ss / (double)G + eps / (s * s));
      for (int64_t c = 0; c < G; ++c) v[c] /= den;
    }
  }
}

static void set_threads(int threads) {
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#else
  (void)threads;
#endif
}

/* Sequence index of every token from cumulative offsets (clamped to [0, T]). */
static int64_t* seq_of_tokens(const int64_t* cu, int64_t nseq, int64_t T, int64_t* starts_out) {
  int64_t* seq = (int64_t*)malloc(sizeof(int64_t) * (T > 0 ? T : 1));
  for (int64_t t = 0; t < T; ++t) seq[t] = -1;
  for (int64_t s = 0; s < nseq; ++s) {
    int64_t a = cu[s] < 0 ? 0 : (cu[s] > T ? T : cu[s]);
    int64_t b = cu[s + 1] < 0 ? 0 : (cu[s + 1] > T ? T : cu[s + 1]);
    starts_out[s] = a;
    for (int64_t t = a; t < b; ++t) seq[t] = s;
  }
  return seq;
}

/*
 * Training forward. cu == NULL: one sequence of T tokens. yr (pre-norm output)
 * may be NULL. Tokens outside every sequence are left untouched.
 */
void oracle_fwd(const float* x, const float* w, const float* gate, const int64_t* cu, int64_t nseq,
                int64_t T, int64_t D, int64_t W, int64_t G, int norm, double eps, float* y, float* yr,
                int threads) {
  set_threads(threads);
  const int64_t H = W - 1, DC = D / G;
  int64_t one[2] = {0, T};
  if (!cu) {
    cu = one;
    nseq = 1;
  }
  int64_t* starts = (int64_t*)malloc(sizeof(int64_t) * (nseq > 0 ? nseq : 1));
  int64_t* seq = seq_of_tokens(cu, nseq, T, starts);
#pragma omp parallel
  {
    double* acc = (double*)malloc(sizeof(double) * D);
#pragma omp for schedule(static)
    for (int64_t t = 0; t < T; ++t) {
      if (seq[t] < 0) continue;
      const int64_t a = starts[seq[t]];
      for (int64_t d = 0; d < D; ++d) acc[d] = 0;
      for (int64_t k = 0; k < W; ++k) {
        const int64_t src = t + k - H;
        if (src < a) continue;
        const float* xr = x + src * D;
        const float* wr = w + (t * W + k) * DC;
        for (int64_t d = 0; d < D; ++d) acc[d] += (double)xr[d] * (double)wr[d / G];
      }
      if (yr && norm)
        for (int64_t d = 0; d < D; ++d) yr[t * D + d] = (float)acc[d];
      norm_row(acc, D, G, norm, eps);
      for (int64_t d = 0; d < D; ++d) {
        double v = acc[d];
        if (gate) {
          const double g = gate[t * D + d];
          v *= g * sigmoid_d(g);
        }
        y[t * D + d] = (float)v;
      }
    }
    free(acc);
  }
  free(seq);
  free(starts);
}

/*
 * Training backward: dx [T, D], dw [T, W, D/G], dg [T, D] (dg only with gate).
 * norm 0 or 1 (plain), as in the reference training path. With norm, `yr`
 * (may be NULL) is the pre-norm output saved by the forward, in the I/O
 * precision: the reference backward kernel reads it from memory
 * (greta/dynamic_conv.py:328-342) instead of recomputing it, and with 16-bit
 * I/O its rounding matters for groups whose RMS is tiny. NULL recomputes it
 * exactly (the autograd-through-torch form, :937-962).
 */
void oracle_bwd(const float* x, const float* w, const float* gate, const float* dout, const float* yr,
                const int64_t* cu, int64_t nseq, int64_t T, int64_t D, int64_t W, int64_t G, int norm, double eps,
                float* dx, float* dw, float* dg, int threads) {
  set_threads(threads);
  const int64_t H = W - 1, DC = D / G;
  int64_t one[2] = {0, T};
  if (!cu) {
    cu = one;
    nseq = 1;
  }
  int64_t* starts = (int64_t*)malloc(sizeof(int64_t) * (nseq > 0 ? nseq : 1));
  int64_t* seq = seq_of_tokens(cu, nseq, T, starts);
  double* dy = (double*)malloc(sizeof(double) * (T > 0 ? T : 1) * D);
  double* hat = (double*)malloc(sizeof(double) * (T > 0 ? T : 1) * D); /* pre-gate output */
  /* pass 1: conv output, norm, dy = d out / d (pre-norm conv) */
#pragma omp parallel
  {
    double* acc = (double*)malloc(sizeof(double) * D);
    double* dn = (double*)malloc(sizeof(double) * D);
#pragma omp for schedule(static)
    for (int64_t t = 0; t < T; ++t) {
      double* dyr = dy + t * D;
      double* hr = hat + t * D;
      if (seq[t] < 0) {
        for (int64_t d = 0; d < D; ++d) dyr[d] = hr[d] = 0;
        continue;
      }
      const int64_t a = starts[seq[t]];
      if (norm && yr) {
        for (int64_t d = 0; d < D; ++d) acc[d] = yr[t * D + d];
      } else {
        for (int64_t d = 0; d < D; ++d) acc[d] = 0;
        for (int64_t k = 0; k < W; ++k) {
          const int64_t src = t + k - H;
          if (src < a) continue;
          for (int64_t d = 0; d < D; ++d) acc[d] += (double)x[src * D + d] * (double)w[(t * W + k) * DC + d / G];
        }
      }
      for (int64_t d = 0; d < D; ++d) {
        const double o = dout[t * D + d];
        if (gate) {
          const double g = gate[t * D + d];
          dn[d] = o * g * sigmoid_d(g);
        } else {
          dn[d] = o;
        }
      }
      if (norm) {
        for (int64_t f = 0; f < DC; ++f) {
          double ss = 0, cs = 0;
          for (int64_t c = 0; c < G; ++c) ss += acc[f * G + c] * acc[f * G + c];
          const double rinv = 1.0 / sqrt(ss / (double)G + eps);
          for (int64_t c = 0; c < G; ++c) cs += acc[f * G + c] * rinv * dn[f * G + c];
          cs /= (double)G;
          for (int64_t c = 0; c < G; ++c) {
            const double n = acc[f * G + c] * rinv;
            hr[f * G + c] = n;
            dyr[f * G + c] = rinv * (dn[f * G + c] - n * cs);
          }
        }
      } else {
        for (int64_t d = 0; d < D; ++d) {
          hr[d] = acc[d];
          dyr[d] = dn[d];
        }
      }
    }
    free(acc);
    free(dn);
  }
  /* pass 2: dx, dw, dg */
#pragma omp parallel
  {
    double* accx = (double*)malloc(sizeof(double) * D);
#pragma omp for schedule(static)
    for (int64_t t = 0; t < T; ++t) {
      if (seq[t] < 0) continue;
      const int64_t a = starts[seq[t]];
      const int64_t e = cu[seq[t] + 1] > T ? T : cu[seq[t] + 1];
      (void)a;
      /* dx[t] = sum_i dy[t+i] * w[t+i, W-1-i] within the sequence */
      for (int64_t d = 0; d < D; ++d) accx[d] = 0;
      for (int64_t i = 0; i < W; ++i) {
        const int64_t u = t + i;
        if (u >= e) break;
        for (int64_t d = 0; d < D; ++d) accx[d] += dy[u * D + d] * (double)w[(u * W + (W - 1 - i)) * DC + d / G];
      }
      for (int64_t d = 0; d < D; ++d) dx[t * D + d] = (float)accx[d];
      /* dw[t, k, f] = sum_{d in f} dy[t, d] * x[t+k-W+1, d] */
      for (int64_t k = 0; k < W; ++k) {
        const int64_t src = t + k - H;
        for (int64_t f = 0; f < DC; ++f) {
          double s = 0;
          if (src >= starts[seq[t]])
            for (int64_t c = 0; c < G; ++c) s += dy[t * D + f * G + c] * (double)x[src * D + f * G + c];
          dw[(t * W + k) * DC + f] = (float)s;
        }
      }
      if (gate && dg) {
        for (int64_t d = 0; d < D; ++d) {
          const double g = gate[t * D + d], sg = sigmoid_d(g);
          dg[t * D + d] = (float)((double)dout[t * D + d] * hat[t * D + d] * (sg * (1.0 + g * (1.0 - sg))));
        }
      }
    }
    free(accx);
  }
  free(dy);
  free(hat);
  free(seq);
  free(starts);
}

/* HF inference from context [B, Q+W-1, D]; w [B, Q, W, D/G]; gate, y [B, Q, D]. */
void oracle_inference(const float* ctx, const float* w, const float* gate, int64_t B, int64_t Q, int64_t D,
                      int64_t W, int64_t G, int norm, double eps, float* y, int threads) {
  set_threads(threads);
  const int64_t DC = D / G, CL = Q + W - 1;
#pragma omp parallel
  {
    double* acc = (double*)malloc(sizeof(double) * D);
#pragma omp for collapse(2) schedule(static)
    for (int64_t b = 0; b < B; ++b)
      for (int64_t q = 0; q < Q; ++q) {
        for (int64_t d = 0; d < D; ++d) acc[d] = 0;
        for (int64_t k = 0; k < W; ++k) {
          const float* xr = ctx + (b * CL + q + k) * D;
          const float* wr = w + ((b * Q + q) * W + k) * DC;
          for (int64_t d = 0; d < D; ++d) acc[d] += (double)xr[d] * (double)wr[d / G];
        }
        norm_row(acc, D, G, norm, eps);
        for (int64_t d = 0; d < D; ++d) {
          double v = acc[d];
          if (gate) {
            const double g = gate[(b * Q + q) * D + d];
            v *= g * sigmoid_d(g);
          }
          y[(b * Q + q) * D + d] = (float)v;
        }
      }
    free(acc);
  }
}

/* HF decode by batch row; state [B, D, W-1] contiguous, shifted in place. */
void oracle_decode_rows(const float* x, const float* w, const float* gate, float* state, int64_t B, int64_t D,
                        int64_t W, int64_t G, int norm, double eps, float* y, int threads) {
  set_threads(threads);
  const int64_t H = W - 1, DC = D / G;
#pragma omp parallel
  {
    double* acc = (double*)malloc(sizeof(double) * D);
#pragma omp for schedule(static)
    for (int64_t b = 0; b < B; ++b) {
      float* st = state + b * D * H;
      for (int64_t d = 0; d < D; ++d) {
        double s = 0;
        for (int64_t k = 0; k < H; ++k) s += (double)st[d * H + k] * (double)w[(b * W + k) * DC + d / G];
        s += (double)x[b * D + d] * (double)w[(b * W + H) * DC + d / G];
        acc[d] = s;
      }
      norm_row(acc, D, G, norm, eps);
      for (int64_t d = 0; d < D; ++d) {
        double v = acc[d];
        if (gate) {
          const double g = gate[b * D + d];
          v *= g * sigmoid_d(g);
        }
        y[b * D + d] = (float)v;
        for (int64_t k = 0; k + 1 < H; ++k) st[d * H + k] = st[d * H + k + 1];
        st[d * H + H - 1] = x[b * D + d];
      }
    }
    free(acc);
  }
}

/*
 * vLLM packed batch with cache-slot history and state write-back.
 * starts [N+1], slots [N] (< 0 or >= num_slots: no history, no write-back),
 * has_initial [N]. state is addressed as state[slot*s_slot + d*s_d + h*s_h].
 * Each request reads its slot before writing it (slots are distinct).
 */
void oracle_packed(const float* x, const float* w, const float* gate, float* state, int64_t num_slots,
                   int64_t s_slot, int64_t s_d, int64_t s_h, const int64_t* starts, const int64_t* slots,
                   const int64_t* has_initial, int64_t N, int64_t T, int64_t D, int64_t W, int64_t G, int norm,
                   double eps, float* y, int threads) {
  set_threads(threads);
  const int64_t H = W - 1, DC = D / G;
#pragma omp parallel
  {
    double* acc = (double*)malloc(sizeof(double) * D);
    float* old = (float*)malloc(sizeof(float) * (H > 0 ? H : 1) * D);
#pragma omp for schedule(dynamic, 1)
    for (int64_t n = 0; n < N; ++n) {
      int64_t a = starts[n] < 0 ? 0 : (starts[n] > T ? T : starts[n]);
      int64_t b = starts[n + 1] < 0 ? 0 : (starts[n + 1] > T ? T : starts[n + 1]);
      if (b < a) b = a;
      const int64_t len = b - a;
      int64_t slot = slots[n];
      if (slot >= num_slots || !state) slot = -1;
      const int has = has_initial[n] != 0 && slot >= 0;
      /* snapshot of the old slot contents (zeros without history) */
      for (int64_t d = 0; d < D; ++d)
        for (int64_t h = 0; h < H; ++h) old[d * H + h] = has ? state[slot * s_slot + d * s_d + h * s_h] : 0.f;
      for (int64_t t = a; t < b; ++t) {
        const int64_t local = t - a;
        for (int64_t d = 0; d < D; ++d) acc[d] = 0;
        for (int64_t k = 0; k < W; ++k) {
          const int64_t src = local + k - H;
          const float* wr = w + (t * W + k) * DC;
          for (int64_t d = 0; d < D; ++d) {
            const double v = src >= 0 ? (double)x[(a + src) * D + d] : (double)old[d * H + src + H];
            acc[d] += v * (double)wr[d / G];
          }
        }
        norm_row(acc, D, G, norm, eps);
        for (int64_t d = 0; d < D; ++d) {
          double v = acc[d];
          if (gate) {
            const double g = gate[t * D + d];
            v *= g * sigmoid_d(g);
          }
          y[t * D + d] = (float)v;
        }
      }
      if (slot >= 0) {
        for (int64_t h = 0; h < H; ++h) {
          const int64_t local = len - H + h;
          for (int64_t d = 0; d < D; ++d)
            state[slot * s_slot + d * s_d + h * s_h] = local >= 0 ? x[(a + local) * D + d] : old[d * H + local + H];
        }
      }
    }
    free(acc);
    free(old);
  }
}

int oracle_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
