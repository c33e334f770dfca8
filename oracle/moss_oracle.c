/*
 * moss_oracle.c -- CPU oracle for the MOSS Audio Tokenizer v2 hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file restates, in plain C with IEEE-754
 * round-to-nearest arithmetic (compiled with -ffp-contract=off, so every `*`
 * and `+` rounds on its own and only explicit fmaf() fuses), the algorithms
 * the reference runs on the hot path.  It is the checker the tests, the smoke
 * check and the CPU baseline of the benchmark compare against; the product
 * (fast_moss_b200) never links or calls it.
 *
 * Pinning (how each restatement is tied to the reference):
 *   scale_add, rotate, select  -- golden vectors produced by the reference's
 *                                 own Triton kernels (run under the Triton
 *                                 interpreter) in tests/golden/;
 *   lfq_prepare                -- the reference's kernel source compiled for
 *                                 the host (oracle/build_ref.py) and golden
 *                                 vectors in tests/golden/;
 *   layer_norm                 -- golden vectors from torch's CUDA layer norm
 *                                 (the op the reference calls) captured on a
 *                                 B200 by tests/golden/make_golden_gpu.py;
 *   rvq                        -- per-stage selection checked against the
 *                                 reference's `_select` kernel on the golden
 *                                 case; the loop itself is upstream code that
 *                                 is not in the reference, its dot/norm order
 *                                 is this project's documented definition.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define EXPORT __attribute__((visibility("default")))

/* ----------------------------------------------------------------- helpers */
static float bf16_round(float f) {
  /* Round-to-nearest-even to bfloat16, returned as float (NaN kept quiet). */
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) {
    u = (u | 0x00400000u) & 0xffff0000u;
  } else {
    uint32_t lsb = (u >> 16) & 1u;
    u = (u + 0x7fffu + lsb) & 0xffff0000u;
  }
  memcpy(&f, &u, 4);
  return f;
}

static float round_dtype(float v, int bf16) { return bf16 ? bf16_round(v) : v; }

EXPORT void oracle_bf16_round(const float* x, float* y, int64_t n) {
  for (int64_t i = 0; i < n; ++i) y[i] = bf16_round(x[i]);
}

/* ------------------------------------------------------- residual update
 * fast_moss/v2_pointwise.py:92-98 (_scale_add): y = x + u*s[i % c], the
 * product and the sum rounded separately. */
EXPORT void oracle_scale_add(const float* x, const float* u, const float* s, float* y, int64_t n,
                             int64_t c) {
  for (int64_t i = 0; i < n; ++i) {
    float p = u[i] * s[i % c];
    y[i] = x[i] + p;
  }
}

/* ---------------------------------------------------------------- layer norm
 * torch.nn.LayerNorm on CUDA as called by fast_moss/v2_runtime.py:259: the
 * vectorised float32 forward of PyTorch (128 threads = 4 warps per row,
 * float4 loads, per-thread Welford with float count, shuffle-down tree per
 * warp, two-level tree across warps, var = m2/n, rstd = rsqrt(var + eps),
 * y = fma(gamma, rstd*(x-mean), beta)).  mean_variant selects how the merge
 * "nA*meanA + nB*meanB" is fused: 0 fma(nA,meanA,nB*meanB), 1 fma(nB,meanB,
 * nA*meanA), 2 no fusion; 0 is the form the B200 golden vectors confirm. */
typedef struct {
  float mean, m2, count;
} welford_t;

static welford_t w_push(welford_t w, float v) {
  float delta = v - w.mean;
  float count = w.count + 1.0f;
  float mean = fmaf(delta, 1.0f / count, w.mean);
  float m2 = fmaf(delta, v - mean, w.m2);
  welford_t r = {mean, m2, count};
  return r;
}

static welford_t w_merge(welford_t b, welford_t a, int mean_variant) {
  float delta = b.mean - a.mean;
  float count = a.count + b.count;
  welford_t r = {0.0f, 0.0f, count};
  if (count > 0.0f) {
    float coef = 1.0f / count;
    float na = a.count * coef;
    float nb = b.count * coef;
    if (mean_variant == 0) {
      float t = nb * b.mean;
      r.mean = fmaf(na, a.mean, t);
    } else if (mean_variant == 1) {
      float t = na * a.mean;
      r.mean = fmaf(nb, b.mean, t);
    } else {
      float t1 = na * a.mean, t2 = nb * b.mean;
      r.mean = t1 + t2;
    }
    float dd = delta * delta;
    float dda = dd * a.count;
    float sum = a.m2 + b.m2;
    r.m2 = fmaf(dda, nb, sum);
  }
  return r;
}

/* Row statistics of one row of width n (n % 4 == 0). */
static void ln_row_stats(const float* x, int64_t n, int mean_variant, float* mean_out,
                         float* m2_out) {
  welford_t th[128];
  int64_t nvec = n / 4;
  for (int t = 0; t < 128; ++t) {
    welford_t w = {0.0f, 0.0f, 0.0f};
    for (int64_t i = t; i < nvec; i += 128) {
      for (int e = 0; e < 4; ++e) w = w_push(w, x[4 * i + e]);
    }
    th[t] = w;
  }
  welford_t warp_res[4];
  for (int wp = 0; wp < 4; ++wp) {
    welford_t lane[32];
    for (int l = 0; l < 32; ++l) lane[l] = th[wp * 32 + l];
    for (int off = 16; off > 0; off >>= 1) {
      welford_t next[32];
      for (int l = 0; l < 32; ++l) {
        /* __shfl_down returns the caller's own value past the warp end */
        welford_t other = (l + off < 32) ? lane[l + off] : lane[l];
        next[l] = w_merge(lane[l], other, mean_variant);
      }
      memcpy(lane, next, sizeof(lane));
    }
    warp_res[wp] = lane[0];
  }
  welford_t w0 = w_merge(warp_res[0], warp_res[2], mean_variant);
  welford_t w1 = w_merge(warp_res[1], warp_res[3], mean_variant);
  w0 = w_merge(w0, w1, mean_variant);
  *mean_out = w0.mean;
  *m2_out = w0.m2;
}

/* var_eps_out[r] = m2/n + eps (the argument of rsqrt).  If rstd_in is given
 * those per-row values are used (the device rsqrtf is an approximation whose
 * exact bits are hardware-defined); otherwise rstd = 1/sqrt(var+eps) rounded
 * from double.  Any output pointer may be NULL except y. */
EXPORT void oracle_layer_norm(const float* x, const float* gamma, const float* beta, float eps,
                              int64_t rows, int64_t n, int mean_variant, const float* rstd_in,
                              float* y, float* mean_out, float* var_eps_out, float* rstd_out) {
  for (int64_t r = 0; r < rows; ++r) {
    const float* xr = x + r * n;
    float mean, m2;
    ln_row_stats(xr, n, mean_variant, &mean, &m2);
    float var = m2 / (float)n;
    float ve = var + eps;
    float rstd = rstd_in ? rstd_in[r] : (float)(1.0 / sqrt((double)ve));
    for (int64_t j = 0; j < n; ++j) {
      float diff = xr[j] - mean;
      float t = rstd * diff;
      float o;
      if (gamma && beta) o = fmaf(gamma[j], t, beta[j]);
      else if (gamma) o = gamma[j] * t;
      else if (beta) o = fmaf(rstd, diff, beta[j]);
      else o = t;
      y[r * n + j] = o;
    }
    if (mean_out) mean_out[r] = mean;
    if (var_eps_out) var_eps_out[r] = ve;
    if (rstd_out) rstd_out[r] = rstd;
  }
}

/* ------------------------------------------------------------------- rotary
 * fast_moss/v2_pointwise.py:8-47 (_rotate).  q, k hold float values (of the
 * input dtype) with element strides qs/ks; cos/sin [b,t,d/2]; outputs are
 * contiguous [b,h,t,d], rounded to bf16 when bf16 != 0. */
EXPORT void oracle_rotate(const float* q, const float* k, const int64_t* qs, const int64_t* ks,
                          const float* cs, const float* sn, int64_t b, int64_t h, int64_t t,
                          int64_t d, int bf16, float* oq, float* ok) {
  int64_t half = d / 2;
  for (int64_t bi = 0; bi < b; ++bi)
    for (int64_t hi = 0; hi < h; ++hi)
      for (int64_t ti = 0; ti < t; ++ti)
        for (int64_t p = 0; p < half; ++p) {
          int64_t qi = bi * qs[0] + hi * qs[1] + ti * qs[2] + 2 * p * qs[3];
          int64_t ki = bi * ks[0] + hi * ks[1] + ti * ks[2] + 2 * p * ks[3];
          float c = cs[(bi * t + ti) * half + p], s = sn[(bi * t + ti) * half + p];
          float qr = q[qi], qj = q[qi + qs[3]], kr = k[ki], kj = k[ki + ks[3]];
          int64_t o = ((bi * h + hi) * t + ti) * d + 2 * p;
          float a1 = qr * c, a2 = qj * s, a3 = qr * s, a4 = qj * c;
          oq[o] = round_dtype(a1 - a2, bf16);
          oq[o + 1] = round_dtype(a3 + a4, bf16);
          a1 = kr * c; a2 = kj * s; a3 = kr * s; a4 = kj * c;
          ok[o] = round_dtype(a1 - a2, bf16);
          ok[o + 1] = round_dtype(a3 + a4, bf16);
        }
}

/* Rotary tables of fast_moss/v2_runtime.py:209-222 evaluated with double
 * precision libm and rounded to float (the device uses CUDA's expf/cosf/sinf,
 * so these agree to a few float ulps, not bit for bit). */
EXPORT void oracle_rope_tables(const float* offset, int64_t b, int64_t t, int64_t d, float coef,
                               float* cs, float* sn) {
  int64_t half = d / 2;
  for (int64_t bi = 0; bi < b; ++bi)
    for (int64_t ti = 0; ti < t; ++ti)
      for (int64_t j = 0; j < half; ++j) {
        float arg = (float)j * coef;
        float freq = (float)exp((double)arg);
        float ts = offset[bi] + (float)ti;
        float phase = freq * ts;
        cs[(bi * t + ti) * half + j] = (float)cos((double)phase);
        sn[(bi * t + ti) * half + j] = (float)sin((double)phase);
      }
}

/* ------------------------------------------------------ gated activation
 * Eager PyTorch chain (no reference kernel; upstream FFN): h = round(x + b),
 * a = round(act(h_gate)), y = round(a * h_up).  act evaluated in float with
 * double-precision libm for exp/erf/tanh rounded to float. */
static float act_eval(float v, int act) {
  if (act == 0) {
    float e = (float)exp(-(double)v);
    float den = 1.0f + e;
    return v / den;
  } else if (act == 1) {
    float arg = v * 0.70710678118654752440f;
    float er = (float)erf((double)arg);
    float h = v * 0.5f;
    return h * (1.0f + er);
  } else {
    float cube = (v * v) * v;
    float inner = 0.79788456080286535588f * fmaf(0.044715f, cube, v);
    float th = (float)tanh((double)inner);
    float h = 0.5f * v;
    return h * (1.0f + th);
  }
}

EXPORT void oracle_gated_act(const float* x, const float* bias, float* y, int64_t rows,
                             int64_t width, int act, int gated, int bf16) {
  int64_t out_w = gated ? width / 2 : width;
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t c = 0; c < out_w; ++c) {
      /* without a bias there is no add (so -0 stays -0, as in torch) */
      float hg = bias ? round_dtype(x[r * width + c] + bias[c], bf16) : x[r * width + c];
      float a = round_dtype(act_eval(hg, act), bf16);
      if (gated) {
        float hu = bias ? round_dtype(x[r * width + out_w + c] + bias[out_w + c], bf16)
                        : x[r * width + out_w + c];
        y[r * out_w + c] = round_dtype(a * hu, bf16);
      } else {
        y[r * out_w + c] = a;
      }
    }
}

/* ----------------------------------------------------------- LFQ prepare
 * fast_moss/quantizer_prepare.py:17-57.  transposed = (b == 1 && t > 1). */
static float sum8(const float* v, int transposed) {
  if (transposed) {
    float a = v[0] + v[4], b = v[1] + v[5], c = v[2] + v[6], d = v[3] + v[7];
    float ab = a + b;
    float abc = ab + c;
    return abc + d;
  }
  float p01 = v[0] + v[1], p23 = v[2] + v[3], p45 = v[4] + v[5], p67 = v[6] + v[7];
  float l = p01 + p23, r = p45 + p67;
  return l + r;
}

/* The preparation of one 8-value latent v; `transposed` selects the order
 * the reference uses for a [1, 8, t > 1] batch. */
static void prepare_values(const float* v, int transposed, float* e, float* tw, float* norm,
                           float* denom) {
  float sq[8], es[8];
  for (int d = 0; d < 8; ++d) sq[d] = v[d] * v[d];
  float total;
  if (transposed) {
    float a = fmaf(v[4], v[4], sq[0]), bb = fmaf(v[5], v[5], sq[1]);
    float c = fmaf(v[6], v[6], sq[2]), dd = fmaf(v[7], v[7], sq[3]);
    float ab = a + bb;
    float abc = ab + c;
    total = abc + dd;
  } else {
    total = sum8(sq, 0);
  }
  float den = sqrtf(total);
  den = den < 1.0e-12f ? 1.0e-12f : den;
  for (int d = 0; d < 8; ++d) {
    e[d] = v[d] / den;
    tw[d] = 2.0f * e[d];
    es[d] = e[d] * e[d];
  }
  *norm = sum8(es, transposed);
  *denom = den;
}

static void prepare_one(const float* x, int64_t row, int64_t b, int64_t t, float* e, float* tw,
                        float* norm, float* denom) {
  int64_t bi = row / t, ti = row % t;
  float v[8];
  for (int d = 0; d < 8; ++d) v[d] = x[bi * 8 * t + d * t + ti];
  prepare_values(v, b == 1 && t > 1, e, tw, norm, denom);
}

EXPORT void oracle_lfq_prepare(const float* x, int64_t b, int64_t t, float* e, float* norm,
                               float* twice, float* denom) {
  int transposed = (b == 1 && t > 1);
  for (int64_t row = 0; row < b * t; ++row) {
    float ev[8], tv[8];
    prepare_one(x, row, b, t, ev, tv, &norm[row], &denom[row]);
    for (int d = 0; d < 8; ++d) {
      int64_t o = transposed ? d * t + row : row * 8 + d;
      e[o] = ev[d];
      twice[o] = tv[d];
    }
  }
}

/* ------------------------------------------------------------ LFQ select
 * fast_moss/quantizer.py:29-49: distance = (norm - dots) + cnorm, first NaN
 * index wins, otherwise the first minimum. */
static int64_t select_first(const float* dist, int64_t k) {
  int64_t best_i = 0;
  float best = INFINITY;
  int have = 0;
  for (int64_t j = 0; j < k; ++j) {
    if (isnan(dist[j])) return j;
  }
  for (int64_t j = 0; j < k; ++j) {
    if (!have || dist[j] < best) {
      best = dist[j];
      best_i = j;
      have = 1;
    }
  }
  return best_i;
}

EXPORT void oracle_lfq_select(const float* dots, const float* norm, const float* cnorm,
                              const float* book, const float* lat, const int64_t* ls, int64_t b,
                              int64_t d, int64_t t, int64_t k, int ste, float* out,
                              int64_t* indices) {
  float* dist = (float*)malloc(sizeof(float) * (size_t)k);
  for (int64_t row = 0; row < b * t; ++row) {
    for (int64_t j = 0; j < k; ++j) {
      float diff = norm[row] - dots[row * k + j];
      dist[j] = diff + cnorm[j];
    }
    int64_t idx = select_first(dist, k);
    indices[row] = idx;
    int64_t bi = row / t, ti = row % t;
    for (int64_t c = 0; c < d; ++c) {
      float value = book[idx * d + c];
      if (ste) {
        float latent = lat[bi * ls[0] + c * ls[1] + ti * ls[2]];
        float diff = value - latent;
        out[bi * d * t + c * t + ti] = latent + diff;
      } else {
        out[row * d + c] = value;
      }
    }
  }
  free(dist);
}

/* LFQ decode (fast_moss/v2_runtime.py:143-181) with the dot products as a
 * sequential FMA over the eight channels (first term a plain product). */
EXPORT void oracle_lfq_decode(const float* x, const float* book_normed, const float* cnorm,
                              const float* weight, int64_t b, int64_t t, int64_t k, float* out,
                              int64_t* indices) {
  float* dist = (float*)malloc(sizeof(float) * (size_t)k);
  for (int64_t row = 0; row < b * t; ++row) {
    float e[8], tw[8], norm, den;
    prepare_one(x, row, b, t, e, tw, &norm, &den);
    for (int64_t j = 0; j < k; ++j) {
      const float* c = book_normed + j * 8;
      float dot = tw[0] * c[0];
      for (int q = 1; q < 8; ++q) dot = fmaf(tw[q], c[q], dot);
      float diff = norm - dot;
      dist[j] = diff + cnorm[j];
    }
    int64_t idx = select_first(dist, k);
    indices[row] = idx;
    for (int q = 0; q < 8; ++q) out[row * 8 + q] = weight[idx * 8 + q];
  }
  free(dist);
}

/* ------------------------------------------------ multi-stage LFQ quantizer
 * The stage loop of the real codec's quantizer (the upstream module called at
 * fast_moss/v2_codec.py:45), every stage: the 8-wide input projection, the
 * LFQ decode above (prepare with the reference's orders, dots, select:
 * fast_moss/v2_runtime.py:143-181), the output projection and r -= o.  The
 * projections' summation order is defined here (the upstream module that
 * fixes it is not available):
 *   z_j = dot_lanes(w_in[s, j], r) + b_in[s, j]; dot_lanes = 32 partial
 *         sums p_l (sequential FMA from +0 over d = l, l + 32, ...) added as
 *         p_l = p_l + p_(l ^ off) for off = 16, 8, 4, 2, 1, result p_0;
 *   o_d = fma chain over j of w_out[s, d, j] c_j from +0, plus b_out[s, d]. */
static float dot_lanes(const float* w, const float* r, int64_t d) {
  float p[32];
  for (int l = 0; l < 32; ++l) {
    float acc = 0.0f;
    for (int64_t i = l; i < d; i += 32) acc = fmaf(w[i], r[i], acc);
    p[l] = acc;
  }
  for (int off = 16; off > 0; off >>= 1) {
    float q[32];
    for (int l = 0; l < 32; ++l) q[l] = p[l] + p[l ^ off];
    for (int l = 0; l < 32; ++l) p[l] = q[l];
  }
  return p[0];
}

EXPORT void oracle_lfq_rvq_encode(const float* x, int64_t b, int64_t d, int64_t t,
                                  int64_t stages, int64_t k, const float* w_in, const float* b_in,
                                  const float* book_normed, const float* cnorm,
                                  const float* weight, const float* w_out, const float* b_out,
                                  int64_t* codes, float* residual) {
  const int64_t rows = b * t;
  const int transposed_b = (b == 1 && t > 1) ? 1 : 0;
  float* r = (float*)malloc(sizeof(float) * (size_t)d);
  float* dist = (float*)malloc(sizeof(float) * (size_t)k);
  for (int64_t row = 0; row < rows; ++row) {
    const int64_t bi = row / t, ti = row % t;
    for (int64_t c = 0; c < d; ++c) r[c] = x[(bi * d + c) * t + ti];
    for (int64_t s = 0; s < stages; ++s) {
      float z[8], e[8], tw[8], norm, den;
      for (int j = 0; j < 8; ++j)
        z[j] = dot_lanes(w_in + (s * 8 + j) * d, r, d) + b_in[s * 8 + j];
      /* z is one latent of the stage's [b, 8, t] tensor */
      prepare_values(z, transposed_b, e, tw, &norm, &den);
      const float* bn = book_normed + s * k * 8;
      const float* cn = cnorm + s * k;
      for (int64_t j = 0; j < k; ++j) {
        const float* c = bn + j * 8;
        float dot = tw[0] * c[0];
        for (int q = 1; q < 8; ++q) dot = fmaf(tw[q], c[q], dot);
        float diff = norm - dot;
        dist[j] = diff + cn[j];
      }
      const int64_t idx = select_first(dist, k);
      codes[s * rows + row] = idx;
      const float* cw = weight + (s * k + idx) * 8;
      for (int64_t c = 0; c < d; ++c) {
        const float* wo = w_out + (s * d + c) * 8;
        float o = 0.0f;
        for (int j = 0; j < 8; ++j) o = fmaf(wo[j], cw[j], o);
        o = o + b_out[s * d + c];
        r[c] = r[c] - o;
      }
    }
    if (residual)
      for (int64_t c = 0; c < d; ++c) residual[(bi * d + c) * t + ti] = r[c];
  }
  free(dist);
  free(r);
}

/* ------------------------------------------------------ residual VQ
 * Stage loop (the upstream quantizer called at fast_moss/v2_codec.py:45),
 * each stage selecting with the rule of fast_moss/quantizer.py:33-39:
 *   norm = sum_d r_d^2, dot_j = sum_d (2 r_d) c_jd   (sequential FMA from +0,
 *   d ascending), dist_j = (norm - dot_j) + cnorm_j, cnorm_j = sum_d c_jd^2
 *   (same order); first NaN else first minimum; r -= c; recon += c. */
EXPORT void oracle_rvq_code_norms(const float* books, int64_t stages, int64_t k, int64_t d,
                                  float* cnorm) {
  for (int64_t s = 0; s < stages; ++s)
    for (int64_t j = 0; j < k; ++j) {
      const float* c = books + (s * k + j) * d;
      float n = 0.0f;
      for (int64_t q = 0; q < d; ++q) n = fmaf(c[q], c[q], n);
      cnorm[s * k + j] = n;
    }
}

/* dot[j] = sequential FMA of tw against column j of the transposed book
 * bt[d][k]; vectorisable across j while each j keeps the d-ascending order. */
__attribute__((target_clones("arch=skylake-avx512", "arch=haswell", "default"))) static void stage_dots(
    const float* tw, const float* bt, int64_t k, int64_t d, float* dot) {
  for (int64_t j = 0; j < k; ++j) dot[j] = 0.0f;
  for (int64_t q = 0; q < d; ++q) {
    const float a = tw[q];
    const float* col = bt + q * k;
    for (int64_t j = 0; j < k; ++j) dot[j] = fmaf(a, col[j], dot[j]);
  }
}

EXPORT void oracle_rvq_encode(const float* x, int64_t rows, int64_t d, const float* books,
                              const float* cnorm, int64_t stages, int64_t k, int32_t* codes,
                              float* recon, float* residual_out, int nthreads) {
  /* transposed books for the vectorisable dot loop */
  float* bt = (float*)malloc(sizeof(float) * (size_t)(stages * k * d));
  for (int64_t s = 0; s < stages; ++s)
    for (int64_t j = 0; j < k; ++j)
      for (int64_t q = 0; q < d; ++q) bt[(s * d + q) * k + j] = books[(s * k + j) * d + q];
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel
#endif
  {
    float* r = (float*)malloc(sizeof(float) * (size_t)d);
    float* rc = (float*)malloc(sizeof(float) * (size_t)d);
    float* tw = (float*)malloc(sizeof(float) * (size_t)d);
    float* dot = (float*)malloc(sizeof(float) * (size_t)k);
    float* dist = (float*)malloc(sizeof(float) * (size_t)k);
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 16)
#endif
    for (int64_t row = 0; row < rows; ++row) {
      for (int64_t q = 0; q < d; ++q) {
        r[q] = x[row * d + q];
        rc[q] = 0.0f;
      }
      for (int64_t s = 0; s < stages; ++s) {
        float n = 0.0f;
        for (int64_t q = 0; q < d; ++q) {
          n = fmaf(r[q], r[q], n);
          tw[q] = 2.0f * r[q];
        }
        stage_dots(tw, bt + s * d * k, k, d, dot);
        for (int64_t j = 0; j < k; ++j) {
          float diff = n - dot[j];
          dist[j] = diff + cnorm[s * k + j];
        }
        int64_t idx = select_first(dist, k);
        codes[s * rows + row] = (int32_t)idx;
        const float* c = books + (s * k + idx) * d;
        for (int64_t q = 0; q < d; ++q) {
          r[q] = r[q] - c[q];
          rc[q] = rc[q] + c[q];
        }
      }
      for (int64_t q = 0; q < d; ++q) {
        recon[row * d + q] = rc[q];
        if (residual_out) residual_out[row * d + q] = r[q];
      }
    }
    free(r);
    free(rc);
    free(tw);
    free(dot);
    free(dist);
  }
  free(bt);
}

/* Per-stage distances of one row (for checking a stage against the
 * reference's selection kernel): norm and dots in the pinned order. */
EXPORT void oracle_rvq_stage_terms(const float* r, int64_t d, const float* book, int64_t k,
                                   float* norm_out, float* dots_out) {
  float n = 0.0f;
  float* tw = (float*)malloc(sizeof(float) * (size_t)d);
  for (int64_t q = 0; q < d; ++q) {
    n = fmaf(r[q], r[q], n);
    tw[q] = 2.0f * r[q];
  }
  for (int64_t j = 0; j < k; ++j) {
    float dot = 0.0f;
    for (int64_t q = 0; q < d; ++q) dot = fmaf(tw[q], book[j * d + q], dot);
    dots_out[j] = dot;
  }
  *norm_out = n;
  free(tw);
}

EXPORT void oracle_rvq_decode(const int32_t* codes, int64_t rows, const float* books,
                              int64_t stages, int64_t k, int64_t d, float* recon) {
  for (int64_t row = 0; row < rows; ++row)
    for (int64_t q = 0; q < d; ++q) {
      float acc = 0.0f;
      for (int64_t s = 0; s < stages; ++s) {
        int32_t c = codes[s * rows + row];
        if (c < 0 || c >= k) continue;
        acc = acc + books[(s * k + c) * d + q];
      }
      recon[row * d + q] = acc;
    }
}

EXPORT int oracle_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
