/*
 * CPU oracle for the causal depthwise conv1d path.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the checker that the CUDA path is compared against, and
 * the timed CPU baseline. Only tests/, __graft_entry__.smoke() and bench.py (its cpu_baseline leg
 * and its `--impl reference` arm) may load it. The product package never imports, links or calls
 * it. A missing CUDA extension is an error there, never a reason to come here.
 *
 * It restates the reference's algorithm, jxiong21029/causal-conv1d-triton,
 * causal_conv1d_triton/causal_conv1d.py (abbreviated cc.py below), element by element in fp32,
 * in the reference's order of operations:
 *
 *   out[b,t,d] = act(bias[d] + sum_k weight[d,k] * x[b, t-(W-1)+k, d])
 *
 * with rows t < 0 read from initial_states (or zero), seq_idx masking of taps that cross a
 * sequence boundary, padding rows (seq id < 0) forced to zero, and SiLU. Multiply-add pairs that
 * the compiled reference contracts into one FMA (Triton enables fp fusion) use fmaf() here. A tap
 * that reads a zero row (outside concat(initial_states, x)) or that the sequence mask removes is
 * skipped, which equals adding w * 0 except for the sign of an exact zero.
 *
 * Loops run over whole channels-last rows so that the compiler vectorises them along D; the
 * order of operations per element is unchanged by that.
 *
 * Layouts (all contiguous, fp32 unless stated):
 *   x, out, dout, dx : (B, T, D)          weight, dweight : (D, W)        bias, dbias : (D)
 *   initial_states, final_states, dfinal, dinit : (B, W-1, D)            seq_idx : int32 (B, T)
 *
 * The weight/bias gradients are accumulated in double and rounded once at the end, which makes
 * this a tighter reference for them than the reference's own fp32 two-stage sum (cc.py:313-374).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* Row t of concat(initial_states, x): rows in [-PAD, 0) are the initial states, other rows
 * outside [0, T) are zero (returned as NULL). Follows _load_row, cc.py:28-41. */
static inline const float* row_ptr(const float* x, const float* init, int64_t b, int64_t t,
                                   int64_t T, int64_t D, int64_t PAD) {
  if (t >= 0 && t < T) return x + (b * T + t) * D;
  if (init && t < 0 && t >= -PAD) return init + (b * PAD + (t + PAD)) * D;
  return NULL;
}

/* Sequence id at row t: the initial states belong to seq_idx[b, 0]'s sequence, every other row
 * outside [0, T) gets -1. Follows _load_seq, cc.py:17-25. */
static inline int32_t seq_val(const int32_t* seq, int64_t b, int64_t t, int64_t T, int has_init) {
  if (has_init) return t < T ? seq[b * T + (t > 0 ? t : 0)] : -1;
  return (t >= 0 && t < T) ? seq[b * T + t] : -1;
}

static inline float sigmoid_f(float z) { return 1.0f / (1.0f + expf(-z)); }

/* weight (D, W) -> wt (W, D), so that tap k of every channel is one contiguous row. */
static float* transpose_w(const float* w, int64_t D, int64_t W) {
  float* wt = (float*)malloc((size_t)(W * D) * sizeof(float));
  for (int64_t d = 0; d < D; ++d)
    for (int64_t k = 0; k < W; ++k) wt[k * D + d] = w[d * W + k];
  return wt;
}

/* Pre-activation row z[0..D) at (b, t) in the forward's order (cc.py:129-136): the tap on x[t]
 * first, then taps k = 0..W-2 oldest first, each masked to the same sequence, then the bias. */
static void preact_row(const float* x, const float* wt, const float* bias, const float* init,
                       const int32_t* seq, int64_t b, int64_t t, int64_t T, int64_t D, int64_t W,
                       int32_t seq_t, float* z) {
  const int64_t PAD = W - 1;
  const float* xr = row_ptr(x, init, b, t, T, D, PAD);
  const float* wl = wt + PAD * D;
  if (xr) {
    for (int64_t d = 0; d < D; ++d) z[d] = wl[d] * xr[d];
  } else {
    for (int64_t d = 0; d < D; ++d) z[d] = 0.0f;
  }
  for (int64_t k = 0; k < PAD; ++k) {
    const int64_t tt = t - PAD + k;
    const float* r = row_ptr(x, init, b, tt, T, D, PAD);
    if (!r) continue;
    if (seq && seq_val(seq, b, tt, T, init != NULL) != seq_t) continue;
    const float* wk = wt + k * D;
    for (int64_t d = 0; d < D; ++d) z[d] = fmaf(wk[d], r[d], z[d]);
  }
  if (bias)
    for (int64_t d = 0; d < D; ++d) z[d] += bias[d];
}

/* Forward: cc.py:105-164. */
void cc1d_oracle_fwd(const float* x, const float* w, const float* bias, const float* init,
                     const int32_t* seq, float* out, float* final_states, int64_t B, int64_t T,
                     int64_t D, int64_t W, int silu, int nthreads) {
  const int64_t PAD = W - 1;
  float* wt = transpose_w(w, D, W);
#ifdef _OPENMP
  if (nthreads <= 0) nthreads = omp_get_max_threads();
#pragma omp parallel for collapse(2) schedule(static) num_threads(nthreads)
#endif
  for (int64_t b = 0; b < B; ++b) {
    for (int64_t t = 0; t < T; ++t) {
      const int32_t seq_t = seq ? seq_val(seq, b, t, T, init != NULL) : 0;
      float* o = out + (b * T + t) * D;
      preact_row(x, wt, bias, init, seq, b, t, T, D, W, seq_t, o);
      if (seq && seq_t < 0) {
        for (int64_t d = 0; d < D; ++d) o[d] = 0.0f;
      } else if (silu) {
        for (int64_t d = 0; d < D; ++d) o[d] = o[d] * sigmoid_f(o[d]);
      }
    }
  }
  free(wt);
  /* Final states: the last PAD rows of concat(initial_states, x), cc.py:153-164. */
  if (final_states) {
    for (int64_t b = 0; b < B; ++b)
      for (int64_t p = 0; p < PAD; ++p) {
        const float* r = row_ptr(x, init, b, T - PAD + p, T, D, PAD);
        float* f = final_states + (b * PAD + p) * D;
        for (int64_t d = 0; d < D; ++d) f[d] = r ? r[d] : 0.0f;
      }
  }
}

/* Gradient of the pre-activation for row t (cc.py:274-288): dy times SiLU'(z) with z recomputed
 * in the forward's order, zero on padding rows and outside [0, T). */
static void dz_row(const float* x, const float* wt, const float* bias, const float* init,
                   const int32_t* seq, const float* dy, int64_t b, int64_t t, int64_t T,
                   int64_t D, int64_t W, int silu, float* dz, float* zbuf) {
  if (t < 0 || t >= T) {
    for (int64_t d = 0; d < D; ++d) dz[d] = 0.0f;
    return;
  }
  const int32_t seq_t = seq ? seq_val(seq, b, t, T, init != NULL) : 0;
  if (seq && seq_t < 0) {
    for (int64_t d = 0; d < D; ++d) dz[d] = 0.0f;
    return;
  }
  const float* g = dy + (b * T + t) * D;
  if (!silu) {
    memcpy(dz, g, (size_t)D * sizeof(float));
    return;
  }
  preact_row(x, wt, bias, init, seq, b, t, T, D, W, seq_t, zbuf);
  for (int64_t d = 0; d < D; ++d) {
    const float z = zbuf[d];
    const float s = sigmoid_f(z);
    dz[d] = g[d] * s * fmaf(z, 1.0f - s, 1.0f);
  }
}

/* Backward: cc.py:253-341 (per-element math) with the partial sums of cc.py:313-321 and
 * cc.py:344-374 done as one double-precision sum. dinit may be NULL (need_dinit false), dfinal
 * may be NULL. dweight and dbias are always written. */
void cc1d_oracle_bwd(const float* x, const float* w, const float* bias, const float* init,
                     const int32_t* seq, const float* dy, const float* dfinal, float* dx,
                     float* dweight, float* dbias, float* dinit, int64_t B, int64_t T, int64_t D,
                     int64_t W, int silu, int nthreads) {
  const int64_t PAD = W - 1;
  const int64_t TB = 128; /* rows per task */
  const int64_t nblk = (T + TB - 1) / TB;
  const int64_t ntask = B * nblk;
  float* wt = transpose_w(w, D, W);
#ifdef _OPENMP
  if (nthreads <= 0) nthreads = omp_get_max_threads();
#else
  nthreads = 1;
#endif
  const size_t nacc = (size_t)(W + 1) * (size_t)D;
  const size_t nrow = (size_t)(TB + 2 * PAD);
  double* acc = (double*)calloc((size_t)nthreads * nacc, sizeof(double));
  float* dzbuf = (float*)malloc((size_t)nthreads * (nrow + 1) * (size_t)D * sizeof(float));

#ifdef _OPENMP
#pragma omp parallel num_threads(nthreads)
#endif
  {
#ifdef _OPENMP
    const int tid = omp_get_thread_num();
#else
    const int tid = 0;
#endif
    double* a = acc + (size_t)tid * nacc;
    float* dzb = dzbuf + (size_t)tid * (nrow + 1) * (size_t)D;
    float* zbuf = dzb + nrow * (size_t)D;
#ifdef _OPENMP
#pragma omp for schedule(static)
#endif
    for (int64_t task = 0; task < ntask; ++task) {
      const int64_t b = task / nblk;
      const int64_t t0 = (task % nblk) * TB;
      const int64_t t1 = t0 + TB < T ? t0 + TB : T;
      /* Rows whose dx this task produces; block 0 also produces dinit rows [-PAD, 0). */
      const int64_t lo = (t0 == 0 && dinit) ? -PAD : t0;
      /* dz over [lo, t1 + PAD), row r stored at dzb[(r - lo) * D]. */
      for (int64_t r = lo; r < t1 + PAD; ++r)
        dz_row(x, wt, bias, init, seq, dy, b, r, T, D, W, silu, dzb + (r - lo) * D, zbuf);
      for (int64_t t = lo; t < t1; ++t) {
        const int32_t seq_t = seq ? seq_val(seq, b, t, T, init != NULL) : 0;
        float* g = (t >= 0) ? dx + (b * T + t) * D : dinit + (b * PAD + (t + PAD)) * D;
        const float* dz = dzb + (t - lo) * D;
        /* x[t] feeds out[t + j] through weight[PAD - j] (cc.py:290-296). */
        const float* wl = wt + PAD * D;
        for (int64_t d = 0; d < D; ++d) g[d] = wl[d] * dz[d];
        for (int64_t j = 1; j <= PAD; ++j) {
          if (seq && seq_val(seq, b, t + j, T, init != NULL) != seq_t) continue;
          const float* dzj = dzb + (t + j - lo) * D;
          const float* wj = wt + (PAD - j) * D;
          for (int64_t d = 0; d < D; ++d) g[d] = fmaf(wj[d], dzj[d], g[d]);
        }
        /* final_states[p] = concat(initial_states, x)[T - PAD + p] (cc.py:297-302). */
        if (dfinal) {
          const int64_t f = t - (T - PAD);
          if (f >= 0 && f < PAD) {
            const float* df = dfinal + (b * PAD + f) * D;
            for (int64_t d = 0; d < D; ++d) g[d] += df[d];
          }
        }
        if (t < 0) continue;
        /* Weight and bias gradients from the rows this task owns (cc.py:313-321). */
        for (int64_t k = 0; k < W; ++k) {
          const int64_t tt = t - PAD + k;
          if (seq && k < PAD && seq_val(seq, b, tt, T, init != NULL) != seq_t) continue;
          const float* r = row_ptr(x, init, b, tt, T, D, PAD);
          if (!r) continue;
          double* ak = a + k * D;
          for (int64_t d = 0; d < D; ++d) ak[d] += (double)dz[d] * (double)r[d];
        }
        double* ab = a + W * D;
        for (int64_t d = 0; d < D; ++d) ab[d] += (double)dz[d];
      }
    }
  }
  /* Fixed-order sum over threads. */
  for (int64_t k = 0; k <= W; ++k) {
    for (int64_t d = 0; d < D; ++d) {
      double s = 0.0;
      for (int i = 0; i < nthreads; ++i) s += acc[(size_t)i * nacc + (size_t)(k * D + d)];
      if (k < W)
        dweight[d * W + k] = (float)s;
      else if (dbias)
        dbias[d] = (float)s;
    }
  }
  free(wt);
  free(acc);
  free(dzbuf);
}

/* Single-step state update for decoding. The reference has no decode kernel; the state is its
 * (B, W-1, D) layout, the inputs preceding x[:, 0] (cc.py:597-599). For each of the L new rows
 * the window is concat(state, x_new) and out = act(bias + sum_k w[k] * window[k]) in the
 * forward's order; afterwards the state holds the last W-1 rows of concat(state, x_new). state is
 * updated in place. x_new and out are (B, L, D). */
void cc1d_oracle_update(const float* x, float* state, const float* w, const float* bias,
                        float* out, int64_t B, int64_t L, int64_t D, int64_t W, int silu) {
  const int64_t PAD = W - 1;
  float* win = (float*)malloc((size_t)(PAD + L) * sizeof(float));
  for (int64_t b = 0; b < B; ++b) {
    for (int64_t d = 0; d < D; ++d) {
      for (int64_t p = 0; p < PAD; ++p) win[p] = state[(b * PAD + p) * D + d];
      for (int64_t l = 0; l < L; ++l) win[PAD + l] = x[(b * L + l) * D + d];
      const float* wd = w + d * W;
      for (int64_t l = 0; l < L; ++l) {
        float z = wd[PAD] * win[l + PAD];
        for (int64_t k = 0; k < PAD; ++k) z = fmaf(wd[k], win[l + k], z);
        if (bias) z += bias[d];
        if (silu) z = z * sigmoid_f(z);
        out[(b * L + l) * D + d] = z;
      }
      for (int64_t p = 0; p < PAD; ++p) state[(b * PAD + p) * D + d] = win[L + p];
    }
  }
  free(win);
}
