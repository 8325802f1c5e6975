/*
 * gsv_oracle.c -- CPU restatement of the gpt-sovits-rs SoVITS v2 Generator
 * (HiFi-GAN style decoder), used ONLY as test infrastructure: the parity
 * checker for the CUDA library, the golden-fixture cross-check and the timed
 * CPU baseline ("port").  Nothing in the product links or calls this file.
 *
 * Every function restates the reference algorithm and cites the reference
 * file:line (paths inside the gpt-sovits-rs crate) it follows.  Layout is the
 * reference's own: activations [B, C, T] row-major (Candle contiguous NCL).
 *
 * Parity pin: the reference's own tests pin only closed-form known-answer
 * cases (leaky_relu values, padded-ConvT crop, im2col conv); those cases are
 * re-created under tests/golden with expected values computed by PyTorch CPU
 * (an independent implementation of the same conv semantics).  Whole-decoder
 * results are unpinned by the reference's suite (it ships no weights or
 * dumps), so whole-decoder fixtures are cross-checked against an independent
 * float64 PyTorch restatement instead.
 *
 * Accumulation: acc64=1 accumulates every dot product in double (the checker
 * mode); acc64=0 accumulates in float like the reference's MKL sgemm path
 * (src/utils/weights.rs:106-111) and is the mode timed as the CPU baseline.
 */
#include "gsv_oracle.h"

#include <math.h>
#include <omp.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static __thread char g_err[512];

const char* gsvo_last_error(void) { return g_err; }

static int fail(const char* msg, const char* key) {
  snprintf(g_err, sizeof g_err, "%s%s%s", msg, key ? ": " : "", key ? key : "");
  return -1;
}

/* LeakyReLU exactly as the CPU FusedLeakyRelu op: the sign bit decides, so
 * -0.0 maps to -0.0 * slope (src/models/sovits_decoder.rs:46-53, 76-86). */
void gsvo_leaky_relu(float* x, int64_t n, float slope) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    float v = x[i];
    x[i] = signbit(v) ? v * slope : v;
  }
}

/* Weight-norm fold w = g * v / ||v||, the norm taken over dims (1, 2) of each
 * dim-0 slice (src/utils/weights.rs:589-614).  v is [O, I, K], g is [O]. */
void gsvo_weight_norm(const float* v, const float* g, int O, int I, int K, float* w) {
  const int64_t per = (int64_t)I * K;
  for (int o = 0; o < O; ++o) {
    double ss = 0.0;
    for (int64_t j = 0; j < per; ++j) {
      double t = v[o * per + j];
      ss += t * t;
    }
    const float norm = (float)sqrt(ss);
    for (int64_t j = 0; j < per; ++j) w[o * per + j] = (v[o * per + j] / norm) * g[o];
  }
}

/* Conv1d, stride 1, zero padding `pad`, dilation `dil`, optional bias added
 * after the convolution (src/utils/weights.rs:78-113 conv semantics,
 * :533-550 / :646-658 bias add).  x [B, Cin, L] -> y [B, Cout, Lout] with
 * Lout = L + 2 pad - dil (K - 1). */
#define OB 8
#define TB 512
int gsvo_conv1d(const float* x, int B, int Cin, int L, const float* w, int Cout, int K,
                int pad, int dil, const float* bias, float* y, int acc64) {
  const int Lout = L + 2 * pad - dil * (K - 1);
  if (Lout <= 0) return fail("conv1d: non-positive output length", NULL);
  const int nob = (Cout + OB - 1) / OB, ntb = (Lout + TB - 1) / TB;
  const int64_t ntask = (int64_t)B * nob * ntb;
#pragma omp parallel for schedule(dynamic, 1)
  for (int64_t task = 0; task < ntask; ++task) {
    const int b = (int)(task / ((int64_t)nob * ntb));
    const int ob = (int)((task / ntb) % nob);
    const int tb = (int)(task % ntb);
    const int o0 = ob * OB, t0 = tb * TB;
    const int no = (Cout - o0) < OB ? (Cout - o0) : OB;
    const int nt = (Lout - t0) < TB ? (Lout - t0) : TB;
    const float* xb = x + (int64_t)b * Cin * L;
    if (acc64) {
      double acc[OB][TB];
      for (int o = 0; o < OB; ++o)
        for (int t = 0; t < nt; ++t) acc[o][t] = 0.0;
      for (int c = 0; c < Cin; ++c) {
        const float* xr = xb + (int64_t)c * L;
        for (int k = 0; k < K; ++k) {
          const int off = k * dil - pad; /* input index = t + off */
          int lo = -off - t0; if (lo < 0) lo = 0;
          int hi = L - off - t0; if (hi > nt) hi = nt;
          double wv[OB];
          for (int o = 0; o < OB; ++o)
            wv[o] = o < no ? w[((int64_t)(o0 + o) * Cin + c) * K + k] : 0.0;
          for (int t = lo; t < hi; ++t) {
            const double xv = xr[t0 + t + off];
            for (int o = 0; o < OB; ++o) acc[o][t] += wv[o] * xv;
          }
        }
      }
      for (int o = 0; o < no; ++o) {
        float* yr = y + ((int64_t)b * Cout + o0 + o) * Lout + t0;
        for (int t = 0; t < nt; ++t) {
          float v = (float)acc[o][t];
          if (bias) v += bias[o0 + o];
          yr[t] = v;
        }
      }
    } else {
      float acc[OB][TB];
      for (int o = 0; o < OB; ++o)
        for (int t = 0; t < nt; ++t) acc[o][t] = 0.0f;
      for (int c = 0; c < Cin; ++c) {
        const float* xr = xb + (int64_t)c * L;
        for (int k = 0; k < K; ++k) {
          const int off = k * dil - pad;
          int lo = -off - t0; if (lo < 0) lo = 0;
          int hi = L - off - t0; if (hi > nt) hi = nt;
          float wv[OB];
          for (int o = 0; o < OB; ++o)
            wv[o] = o < no ? w[((int64_t)(o0 + o) * Cin + c) * K + k] : 0.0f;
          for (int t = lo; t < hi; ++t) {
            const float xv = xr[t0 + t + off];
            for (int o = 0; o < OB; ++o) acc[o][t] += wv[o] * xv;
          }
        }
      }
      for (int o = 0; o < no; ++o) {
        float* yr = y + ((int64_t)b * Cout + o0 + o) * Lout + t0;
        for (int t = 0; t < nt; ++t) yr[t] = bias ? acc[o][t] + bias[o0 + o] : acc[o][t];
      }
    }
  }
  return 0;
}

/* ConvTranspose1d with weight [Cin, Cout, K] (PyTorch/Candle layout,
 * src/models/sovits_decoder.rs:557-561), computed the way the reference's
 * mkl CPU path does it: the zero-padding transposed conv, then `pad` samples
 * cropped from both ends (src/models/sovits_decoder.rs:88-98), then the bias
 * broadcast-add (:568-573).  Lout = (L - 1) stride + K - 2 pad. */
int gsvo_conv_transpose1d(const float* x, int B, int Cin, int L, const float* w, int Cout,
                          int K, int stride, int pad, const float* bias, float* y, int acc64) {
  const int Lfull = (L - 1) * stride + K;
  const int Lout = Lfull - 2 * pad;
  if (Lout <= 0) return fail("conv_transpose1d: non-positive output length", NULL);
#pragma omp parallel
  {
    double* accd = acc64 ? (double*)malloc(sizeof(double) * (size_t)Lfull) : NULL;
    float* accf = acc64 ? NULL : (float*)malloc(sizeof(float) * (size_t)Lfull);
#pragma omp for schedule(dynamic, 1)
    for (int64_t bo = 0; bo < (int64_t)B * Cout; ++bo) {
      const int b = (int)(bo / Cout), o = (int)(bo % Cout);
      if (acc64) memset(accd, 0, sizeof(double) * (size_t)Lfull);
      else memset(accf, 0, sizeof(float) * (size_t)Lfull);
      for (int c = 0; c < Cin; ++c) {
        const float* xr = x + ((int64_t)b * Cin + c) * L;
        const float* wr = w + ((int64_t)c * Cout + o) * K;
        for (int k = 0; k < K; ++k) {
          const float wk = wr[k];
          if (acc64)
            for (int t = 0; t < L; ++t) accd[t * stride + k] += (double)wk * xr[t];
          else
            for (int t = 0; t < L; ++t) accf[t * stride + k] += wk * xr[t];
        }
      }
      float* yr = y + ((int64_t)b * Cout + o) * Lout;
      for (int t = 0; t < Lout; ++t) {
        float v = acc64 ? (float)accd[t + pad] : accf[t + pad];
        yr[t] = bias ? v + bias[o] : v;
      }
    }
    free(accd);
    free(accf);
  }
  return 0;
}

/* ------------------------------------------------------------------------ */
/* Decoder::load rules (src/models/sovits_decoder.rs:231-293, 146-194).     */

static const gsvo_tensor* find(const gsvo_tensor* ts, int n, const char* name) {
  for (int i = 0; i < n; ++i)
    if (strcmp(ts[i].name, name) == 0) return &ts[i];
  return NULL;
}

static int64_t numel(const gsvo_tensor* t) {
  int64_t n = 1;
  for (int i = 0; i < t->ndim; ++i) n *= t->shape[i];
  return n;
}

typedef struct {
  float* w;  /* folded or plain weight, [O, I, K] (ConvT: [Cin, Cout, K]) */
  const float* b;
  int O, I, K, pad, dil, stride;
} conv_t;

static int load_plain(const gsvo_tensor* ts, int n, const char* pfx, int required, conv_t* c) {
  char key[256];
  snprintf(key, sizeof key, "%s.weight", pfx);
  const gsvo_tensor* w = find(ts, n, key);
  if (!w) return required ? fail("key not found in state dict", key) : 1;
  if (w->ndim != 3) return fail("expected a 3-d conv weight", key);
  c->O = (int)w->shape[0]; c->I = (int)w->shape[1]; c->K = (int)w->shape[2];
  c->w = (float*)malloc(sizeof(float) * (size_t)numel(w));
  memcpy(c->w, w->data, sizeof(float) * (size_t)numel(w));
  snprintf(key, sizeof key, "%s.bias", pfx);
  const gsvo_tensor* b = find(ts, n, key);
  c->b = b ? b->data : NULL;
  c->pad = (c->K - 1) / 2; /* src/models/sovits_decoder.rs:319 */
  c->dil = 1; c->stride = 1;
  return 0;
}

static int load_wn(const gsvo_tensor* ts, int n, const char* pfx, conv_t* c) {
  char key[256];
  snprintf(key, sizeof key, "%s.weight_v", pfx);
  const gsvo_tensor* v = find(ts, n, key);
  if (!v) return fail("key not found in state dict", key);
  if (v->ndim != 3) return fail("expected a 3-d weight_v", key);
  snprintf(key, sizeof key, "%s.weight_g", pfx);
  const gsvo_tensor* g = find(ts, n, key);
  if (!g) return fail("key not found in state dict", key);
  c->O = (int)v->shape[0]; c->I = (int)v->shape[1]; c->K = (int)v->shape[2];
  if (numel(g) != c->O) return fail("weight_g must hold one value per dim-0 slice", key);
  c->w = (float*)malloc(sizeof(float) * (size_t)numel(v));
  gsvo_weight_norm(v->data, g->data, c->O, c->I, c->K, c->w);
  snprintf(key, sizeof key, "%s.bias", pfx);
  const gsvo_tensor* b = find(ts, n, key);
  c->b = b ? b->data : NULL;
  c->pad = (c->K - 1) / 2; c->dil = 1; c->stride = 1;
  return 0;
}

#define MAX_UPS 10
#define MAX_RB 15

typedef struct {
  conv_t pre, post, cond;
  int has_cond;
  conv_t ups[MAX_UPS];
  int n_ups;
  conv_t rb[MAX_RB][2][3];
  int rb_n1[MAX_RB], rb_n2[MAX_RB];
  int n_rb;
} dec_t;

static void free_dec(dec_t* d) {
  free(d->pre.w); free(d->post.w); free(d->cond.w);
  for (int i = 0; i < d->n_ups; ++i) free(d->ups[i].w);
  for (int r = 0; r < d->n_rb; ++r)
    for (int j = 0; j < 3; ++j) { free(d->rb[r][0][j].w); free(d->rb[r][1][j].w); }
}

static int load_dec(const gsvo_tensor* ts, int n, dec_t* d) {
  memset(d, 0, sizeof *d);
  if (load_plain(ts, n, "dec.conv_pre", 1, &d->pre)) return -1;
  if (load_plain(ts, n, "dec.conv_post", 1, &d->post)) return -1;
  int rc = load_plain(ts, n, "dec.cond", 0, &d->cond);
  if (rc < 0) return -1;
  d->has_cond = rc == 0;
  /* Upsample strides are training config, hard-coded [10,8,2,2,2] with a
   * fallback of 2 (src/models/sovits_decoder.rs:252-270). */
  static const int rates[5] = {10, 8, 2, 2, 2};
  char key[256];
  for (int i = 0; i < MAX_UPS; ++i) {
    snprintf(key, sizeof key, "dec.ups.%d.weight_v", i);
    if (!find(ts, n, key)) continue;
    snprintf(key, sizeof key, "dec.ups.%d", i);
    conv_t* u = &d->ups[d->n_ups];
    if (load_wn(ts, n, key, u)) return -1;
    u->stride = d->n_ups < 5 ? rates[d->n_ups] : 2;
    if (u->K < u->stride) return fail("ConvTranspose kernel shorter than its stride", key);
    u->pad = (u->K - u->stride) / 2; /* src/models/sovits_decoder.rs:564 */
    d->n_ups++;
  }
  /* ResBlock1: k = [3,7,11][rb % 3]; convs1 dilation [1,3,5][i] with
   * pad d (k-1)/2; convs2 dilation 1, pad (k-1)/2 (:167-191). */
  static const int ks[3] = {3, 7, 11}, dl[3] = {1, 3, 5};
  for (int r = 0; r < MAX_RB; ++r) {
    snprintf(key, sizeof key, "dec.resblocks.%d.convs1.0.weight_v", r);
    if (!find(ts, n, key)) continue;
    int idx = d->n_rb;
    for (int s = 0; s < 2; ++s) {
      int cnt = 0;
      for (int j = 0; j < 3; ++j) {
        snprintf(key, sizeof key, "dec.resblocks.%d.convs%d.%d.weight_v", r, s + 1, j);
        if (!find(ts, n, key)) continue;
        snprintf(key, sizeof key, "dec.resblocks.%d.convs%d.%d", r, s + 1, j);
        conv_t* c = &d->rb[idx][s][cnt];
        if (load_wn(ts, n, key, c)) return -1;
        const int k = ks[r % 3];
        if (c->K != k) return fail("resblock weight kernel size disagrees with [3,7,11][rb%3]", key);
        if (s == 0) { c->dil = dl[j]; c->pad = dl[j] * (k - 1) / 2; }
        else { c->dil = 1; c->pad = (k - 1) / 2; }
        cnt++;
      }
      if (s == 0) d->rb_n1[idx] = cnt; else d->rb_n2[idx] = cnt;
    }
    if (d->rb_n1[idx] != d->rb_n2[idx]) return fail("resblock convs1/convs2 counts differ", key);
    d->n_rb++;
  }
  return 0;
}

static float* alloc_f(int64_t n) { return (float*)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1)); }

/* ResBlock1::forward (src/models/sovits_decoder.rs:196-208). */
static int resblock(const dec_t* d, int r, const float* x, int B, int C, int L, float* out,
                    float* t1, float* t2, int acc64) {
  const int64_t n = (int64_t)B * C * L;
  memcpy(out, x, sizeof(float) * (size_t)n);
  for (int i = 0; i < d->rb_n1[r]; ++i) {
    const conv_t* c1 = &d->rb[r][0][i];
    const conv_t* c2 = &d->rb[r][1][i];
    memcpy(t1, out, sizeof(float) * (size_t)n);
    gsvo_leaky_relu(t1, n, 0.1f);
    if (gsvo_conv1d(t1, B, C, L, c1->w, c1->O, c1->K, c1->pad, c1->dil, c1->b, t2, acc64)) return -1;
    gsvo_leaky_relu(t2, n, 0.1f);
    if (gsvo_conv1d(t2, B, C, L, c2->w, c2->O, c2->K, c2->pad, c2->dil, c2->b, t1, acc64)) return -1;
#pragma omp parallel for schedule(static)
    for (int64_t e = 0; e < n; ++e) out[e] = out[e] + t1[e];
  }
  return 0;
}

/* Decoder::forward (src/models/sovits_decoder.rs:386-458), with the per-layer
 * taps of forward_debug (:473-526): taps[0] conv_pre(+cond), taps[1+2i]
 * ups i, taps[2+2i] resblock average of stage i, taps[1+2 n_ups] conv_post
 * before tanh.  Any tap pointer may be NULL. */
int gsvo_decoder_forward(const gsvo_tensor* ts, int n_tensors, const float* z, const float* g,
                         int B, int T0, float* wav, float** taps, int acc64, int nthreads) {
  if (nthreads > 0) omp_set_num_threads(nthreads);
  if (B <= 0 || T0 <= 0) return fail("batch and frame count must be positive", NULL);
  dec_t d;
  if (load_dec(ts, n_tensors, &d)) { free_dec(&d); return -1; }
  int rc = -1;
  int C = d.pre.O, L = T0;
  /* Largest activation: the widest C*L over all stages. */
  int64_t maxe = (int64_t)C * L;
  {
    int c = C, l = L;
    for (int i = 0; i < d.n_ups; ++i) {
      l = (l - 1) * d.ups[i].stride + d.ups[i].K - 2 * d.ups[i].pad;
      c = d.ups[i].I;
      if ((int64_t)c * l > maxe) maxe = (int64_t)c * l;
    }
  }
  maxe *= B;
  float *x = alloc_f(maxe), *y = alloc_f(maxe), *acc = alloc_f(maxe), *t1 = alloc_f(maxe),
        *t2 = alloc_f(maxe), *rbo = alloc_f(maxe);
  if (gsvo_conv1d(z, B, d.pre.I, T0, d.pre.w, d.pre.O, d.pre.K, d.pre.pad, 1, d.pre.b, x, acc64))
    goto out;
  if (d.has_cond && g) {
    /* cond(g): Conv1d(gin -> C, k1) broadcast over time (:393-399). */
    float* gp = alloc_f((int64_t)B * d.cond.O);
    if (gsvo_conv1d(g, B, d.cond.I, 1, d.cond.w, d.cond.O, d.cond.K, d.cond.pad, 1, d.cond.b, gp,
                    acc64)) { free(gp); goto out; }
    for (int b = 0; b < B; ++b)
      for (int c = 0; c < C; ++c)
        for (int t = 0; t < L; ++t) x[((int64_t)b * C + c) * L + t] += gp[(int64_t)b * C + c];
    free(gp);
  }
  if (taps && taps[0]) memcpy(taps[0], x, sizeof(float) * (size_t)B * C * L);
  for (int i = 0; i < d.n_ups; ++i) {
    const conv_t* u = &d.ups[i];
    gsvo_leaky_relu(x, (int64_t)B * C * L, 0.1f);
    /* ConvT weight is [Cin, Cout, K]: its dim 0 (O above) is Cin, dim 1 is Cout. */
    if (u->O != C) { fail("upsample channel mismatch", NULL); goto out; }
    {
      const int Cout = u->I;
      const int Lout = (L - 1) * u->stride + u->K - 2 * u->pad;
      if (gsvo_conv_transpose1d(x, B, C, L, u->w, Cout, u->K, u->stride, u->pad, u->b, y, acc64))
        goto out;
      C = Cout; L = Lout;
    }
    { float* s = x; x = y; y = s; }
    if (taps && taps[1 + 2 * i]) memcpy(taps[1 + 2 * i], x, sizeof(float) * (size_t)B * C * L);
    const int r0 = 3 * i, r1 = (r0 + 3) < d.n_rb ? r0 + 3 : d.n_rb;
    if (r0 < d.n_rb) {
      const int64_t n = (int64_t)B * C * L;
      for (int r = r0; r < r1; ++r) {
        if (d.rb[r][0][0].O != C) { fail("resblock width mismatch", NULL); goto out; }
        if (resblock(&d, r, x, B, C, L, r == r0 ? acc : rbo, t1, t2, acc64)) goto out;
        if (r > r0) {
#pragma omp parallel for schedule(static)
          for (int64_t e = 0; e < n; ++e) acc[e] = acc[e] + rbo[e];
        }
      }
      const float div = (float)(r1 - r0); /* true division (:434-440) */
#pragma omp parallel for schedule(static)
      for (int64_t e = 0; e < n; ++e) x[e] = acc[e] / div;
      if (taps && taps[2 + 2 * i]) memcpy(taps[2 + 2 * i], x, sizeof(float) * (size_t)n);
    }
  }
  /* leaky_relu(0.01) -> conv_post -> tanh (:447-455). */
  gsvo_leaky_relu(x, (int64_t)B * C * L, 0.01f);
  if (d.post.I != C) { fail("conv_post width mismatch", NULL); goto out; }
  if (gsvo_conv1d(x, B, C, L, d.post.w, d.post.O, d.post.K, d.post.pad, 1, d.post.b, y, acc64))
    goto out;
  {
    const int64_t n = (int64_t)B * d.post.O * L;
    if (taps && taps[1 + 2 * d.n_ups]) memcpy(taps[1 + 2 * d.n_ups], y, sizeof(float) * (size_t)n);
    for (int64_t e = 0; e < n; ++e) wav[e] = tanhf(y[e]);
  }
  rc = 0;
out:
  free(x); free(y); free(acc); free(t1); free(t2); free(rbo);
  free_dec(&d);
  return rc;
}

/* ------------------------------------------------------------------------ */
/* Flow inverse: ResidualCouplingBlock::forward(reverse = true)             */
/* (src/models/sovits_flow.rs:341-415) over ResidualCouplingLayer           */
/* (:186-335) and WN (:10-168), then z * y_mask (src/models/sovits.rs:394). */

#define MAX_FLOWS 8
#define MAX_WN 16

typedef struct {
  conv_t pre, post, cond;
  conv_t in[MAX_WN], rs[MAX_WN];
  int n_wn, has_cond, half;
} couple_t;

typedef struct {
  couple_t L[MAX_FLOWS];
  int n;
} flow_t;

static void free_flow(flow_t* f) {
  for (int l = 0; l < f->n; ++l) {
    couple_t* c = &f->L[l];
    free(c->pre.w); free(c->post.w); free(c->cond.w);
    for (int i = 0; i < c->n_wn; ++i) { free(c->in[i].w); free(c->rs[i].w); }
  }
}

/* ResidualCouplingLayer::load_conv (:225-279): weight-norm pair if present,
 * else the plain weight (whose g = ||w|| makes the fold the identity up to
 * rounding; the plain weight is used as is). */
static int load_pre_post(const gsvo_tensor* ts, int n, const char* pfx, conv_t* c) {
  char key[256];
  snprintf(key, sizeof key, "%s.weight_v", pfx);
  if (find(ts, n, key)) return load_wn(ts, n, pfx, c);
  return load_plain(ts, n, pfx, 1, c);
}

/* ResidualCouplingBlock::load (:346-368): layers at indices 0..7 that carry a
 * pre.weight (the flips between them hold no weights). */
static int load_flow(const gsvo_tensor* ts, int n, const char* prefix, flow_t* f) {
  memset(f, 0, sizeof *f);
  char key[200], pfx[200];
  for (int i = 0; i < MAX_FLOWS; ++i) {
    snprintf(key, sizeof key, "%s.%d.pre.weight", prefix, i);
    if (!find(ts, n, key)) continue;
    couple_t* c = &f->L[f->n];
    memset(c, 0, sizeof *c);
    f->n++;
    snprintf(pfx, sizeof pfx, "%s.%d.pre", prefix, i);
    if (load_pre_post(ts, n, pfx, &c->pre)) return -1;
    snprintf(pfx, sizeof pfx, "%s.%d.post", prefix, i);
    if (load_pre_post(ts, n, pfx, &c->post)) return -1;
    c->half = c->pre.I; /* half_channels = pre.weight_v.dims()[1] (:211-213) */
    for (int j = 0; j < MAX_WN; ++j) {
      snprintf(key, sizeof key, "%s.%d.enc.in_layers.%d.weight_v", prefix, i, j);
      if (!find(ts, n, key)) break;
      snprintf(pfx, sizeof pfx, "%s.%d.enc.in_layers.%d", prefix, i, j);
      if (load_wn(ts, n, pfx, &c->in[j])) return -1;
      c->n_wn++;
    }
    for (int j = 0; j < c->n_wn; ++j) {
      snprintf(pfx, sizeof pfx, "%s.%d.enc.res_skip_layers.%d", prefix, i, j);
      if (load_wn(ts, n, pfx, &c->rs[j])) return -1;
    }
    snprintf(key, sizeof key, "%s.%d.enc.cond_layer.weight_v", prefix, i);
    if (find(ts, n, key)) {
      snprintf(pfx, sizeof pfx, "%s.%d.enc.cond_layer", prefix, i);
      if (load_wn(ts, n, pfx, &c->cond)) return -1;
      c->has_cond = 1;
    }
    if (c->n_wn == 0) return fail("coupling layer without WN in_layers", pfx);
  }
  if (f->n == 0) return fail("no flow coupling layers under the prefix", prefix);
  return 0;
}

static double sigm(double v) { return 1.0 / (1.0 + exp(-v)); }

/* WN::forward (:119-168) on h [B, hid, T] (already masked), mask [B, T]. */
static int wn_forward(const couple_t* c, const float* h_in, const float* mask, const float* gproj,
                      int B, int T, float* out, float* xw, float* xin, float* acts, float* rsb,
                      int acc64) {
  const int hid = c->in[0].I;
  const int64_t nh = (int64_t)B * hid * T;
  memcpy(xw, h_in, sizeof(float) * (size_t)nh);
  memset(out, 0, sizeof(float) * (size_t)nh);
  for (int i = 0; i < c->n_wn; ++i) {
    const conv_t* in = &c->in[i];
    const conv_t* rs = &c->rs[i];
    /* x_masked = x * mask; x_in = in_layer(x_masked) */
#pragma omp parallel for schedule(static)
    for (int64_t e = 0; e < nh; ++e) acts[e] = xw[e] * mask[(e / ((int64_t)hid * T)) * T + e % T];
    if (gsvo_conv1d(acts, B, hid, T, in->w, in->O, in->K, in->pad, 1, in->b, xin, acc64)) return -1;
    /* fused_add_tanh_sigmoid_multiply (:171-184): tanh(a + g_a) * sigmoid(b + g_b) */
#pragma omp parallel for schedule(static)
    for (int64_t e = 0; e < nh; ++e) {
      const int64_t b = e / ((int64_t)hid * T), ch = (e / T) % hid, t = e % T;
      const float* xi = xin + (int64_t)b * 2 * hid * T;
      double a = xi[ch * T + t], s = xi[(hid + ch) * T + t];
      if (gproj) {
        const float* gl = gproj + (int64_t)b * c->cond.O + (int64_t)i * 2 * hid;
        a = (double)(float)(a + gl[ch]);
        s = (double)(float)(s + gl[hid + ch]);
      }
      acts[e] = acc64 ? (float)(tanh(a) * sigm(s)) : tanhf((float)a) * (1.0f / (1.0f + expf(-(float)s)));
    }
    if (gsvo_conv1d(acts, B, hid, T, rs->w, rs->O, rs->K, rs->pad, 1, rs->b, rsb, acc64)) return -1;
    if (i < c->n_wn - 1) {
      /* x = (x + res) * mask; output += skip */
#pragma omp parallel for schedule(static)
      for (int64_t e = 0; e < nh; ++e) {
        const int64_t b = e / ((int64_t)hid * T), ch = (e / T) % hid, t = e % T;
        const float* r = rsb + (int64_t)b * rs->O * T;
        xw[e] = (xw[e] + r[ch * T + t]) * mask[b * T + t];
        out[e] = out[e] + r[(hid + ch) * T + t];
      }
    } else {
#pragma omp parallel for schedule(static)
      for (int64_t e = 0; e < nh; ++e) {
        const int64_t b = e / ((int64_t)hid * T), ch = (e / T) % hid, t = e % T;
        out[e] = out[e] + rsb[(int64_t)b * rs->O * T + ch * T + t];
      }
    }
  }
#pragma omp parallel for schedule(static)
  for (int64_t e = 0; e < nh; ++e) out[e] = out[e] * mask[(e / ((int64_t)hid * T)) * T + e % T];
  return 0;
}

/* z = flow^-1(z_p) * y_mask.  z_p and z are [B, C, T0] (C = 2 * half);
 * g [B, gin, 1] or NULL; lengths [B] or NULL (all T0). */
int gsvo_flow_inverse(const gsvo_tensor* ts, int n_tensors, const char* prefix, const float* z_p,
                      const float* g, const int* lengths, int B, int T0, float* z, int acc64,
                      int nthreads) {
  if (nthreads > 0) omp_set_num_threads(nthreads);
  if (B <= 0 || T0 <= 0) return fail("batch and frame count must be positive", NULL);
  flow_t f;
  if (load_flow(ts, n_tensors, prefix, &f)) { free_flow(&f); return -1; }
  int rc = -1;
  const int half = f.L[0].half, C = 2 * half, T = T0;
  int hid = f.L[0].in[0].I, maxo = 0;
  for (int l = 0; l < f.n; ++l) {
    if (f.L[l].half != half || f.L[l].in[0].I != hid) { fail("flow layer shapes differ", NULL); free_flow(&f); return -1; }
    for (int i = 0; i < f.L[l].n_wn; ++i) {
      if (f.L[l].in[i].O > maxo) maxo = f.L[l].in[i].O;
      if (f.L[l].rs[i].O > maxo) maxo = f.L[l].rs[i].O;
    }
    if (f.L[l].post.O > maxo) maxo = f.L[l].post.O;
  }
  const int64_t nx = (int64_t)B * C * T, nh = (int64_t)B * hid * T, nw = (int64_t)B * maxo * T;
  float *x = alloc_f(nx), *xf = alloc_f(nx), *mask = alloc_f((int64_t)B * T), *h = alloc_f(nh),
        *out = alloc_f(nh), *xw = alloc_f(nh), *xin = alloc_f(nw), *acts = alloc_f(nh),
        *rsb = alloc_f(nw), *x0 = alloc_f((int64_t)B * half * T), *gp = NULL;
  for (int b = 0; b < B; ++b) {
    const int len = lengths ? lengths[b] : T;
    for (int t = 0; t < T; ++t) mask[(int64_t)b * T + t] = t < len ? 1.0f : 0.0f;
  }
  memcpy(x, z_p, sizeof(float) * (size_t)nx);
  for (int l = f.n - 1; l >= 0; --l) {
    const couple_t* c = &f.L[l];
    /* flip along channels (:408-414) */
    for (int b = 0; b < B; ++b)
      for (int ch = 0; ch < C; ++ch)
        memcpy(xf + ((int64_t)b * C + ch) * T, x + ((int64_t)b * C + (C - 1 - ch)) * T, sizeof(float) * (size_t)T);
    { float* s = x; x = xf; xf = s; }
    /* h = pre(x0) * mask */
    for (int b = 0; b < B; ++b)
      memcpy(x0 + (int64_t)b * half * T, x + (int64_t)b * C * T, sizeof(float) * (size_t)half * T);
    if (gsvo_conv1d(x0, B, half, T, c->pre.w, c->pre.O, c->pre.K, c->pre.pad, 1, c->pre.b, h, acc64)) goto out;
    for (int64_t e = 0; e < nh; ++e) h[e] *= mask[(e / ((int64_t)hid * T)) * T + e % T];
    free(gp); gp = NULL;
    if (c->has_cond && g) {
      gp = alloc_f((int64_t)B * c->cond.O);
      if (gsvo_conv1d(g, B, c->cond.I, 1, c->cond.w, c->cond.O, c->cond.K, c->cond.pad, 1, c->cond.b, gp, acc64)) goto out;
    }
    if (wn_forward(c, h, mask, gp, B, T, out, xw, xin, acts, rsb, acc64)) goto out;
    /* stats = post(h) * mask; mean-only when post has half_channels outputs (:298-318) */
    if (gsvo_conv1d(out, B, hid, T, c->post.w, c->post.O, c->post.K, c->post.pad, 1, c->post.b, rsb, acc64)) goto out;
    {
      const int so = c->post.O;
      const int has_logs = so >= 2 * half;
      for (int b = 0; b < B; ++b)
        for (int ch = 0; ch < half; ++ch)
          for (int t = 0; t < T; ++t) {
            const float mk = mask[(int64_t)b * T + t];
            const float m = rsb[((int64_t)b * so + ch) * T + t] * mk;
            const float lg = has_logs ? rsb[((int64_t)b * so + half + ch) * T + t] * mk : 0.0f;
            float* x1 = x + ((int64_t)b * C + half + ch) * T + t;
            /* inverse: x1 = (x1 - m) * exp(-logs) (:327-333) */
            *x1 = (*x1 - m) * expf(-lg);
          }
    }
  }
  for (int b = 0; b < B; ++b)
    for (int ch = 0; ch < C; ++ch)
      for (int t = 0; t < T; ++t)
        z[((int64_t)b * C + ch) * T + t] = x[((int64_t)b * C + ch) * T + t] * mask[(int64_t)b * T + t];
  rc = 0;
out:
  free(x); free(xf); free(mask); free(h); free(out); free(xw); free(xin); free(acts); free(rsb);
  free(x0); free(gp);
  free_flow(&f);
  return rc;
}

/* ---- EncP elementwise chains -------------------------------------------- */

/* LayerNorm over the channel axis of [B, C, T] (src/utils/weights.rs:461-502,
 * the middle-dimension branch): per (b, t) mean over c, biased variance of
 * the centred values, (v - mean) / sqrt(var + eps) * gamma + beta.  The input
 * is x + y when y is given (the post-norm residual add of EncoderLayer::forward,
 * src/models/sovits_encp.rs:102, :107), added in f32 as the reference does;
 * statistics accumulate in double.  With lengths, frames t >= lengths[b] are
 * multiplied by 0.0f (x.broadcast_mul(x_mask), :109). */
int gsvo_layer_norm(const float* x, const float* y, const float* gamma, const float* beta, int B, int C,
                    int T, float eps, const int* lengths, float* out) {
  if (B <= 0 || C <= 0 || T <= 0) return fail("layer_norm: empty shape", NULL);
#pragma omp parallel for schedule(static)
  for (int64_t bt = 0; bt < (int64_t)B * T; ++bt) {
    const int b = (int)(bt / T), t = (int)(bt % T);
    const int64_t base = (int64_t)b * C * T + t;
    double sum = 0.0;
    for (int c = 0; c < C; ++c) {
      float v = x[base + (int64_t)c * T];
      if (y) v = v + y[base + (int64_t)c * T];
      sum += v;
    }
    const double mean = sum / C;
    double sq = 0.0;
    for (int c = 0; c < C; ++c) {
      float v = x[base + (int64_t)c * T];
      if (y) v = v + y[base + (int64_t)c * T];
      sq += (v - mean) * (v - mean);
    }
    const double sd = sqrt(sq / C + (double)eps);
    const float mk = (lengths && t >= lengths[b]) ? 0.0f : 1.0f;
    for (int c = 0; c < C; ++c) {
      float v = x[base + (int64_t)c * T];
      if (y) v = v + y[base + (int64_t)c * T];
      const float o = (float)((v - mean) / sd * gamma[c] + beta[c]);
      out[base + (int64_t)c * T] = o * mk;
    }
  }
  return 0;
}

/* The FFN half of EncoderLayer::forward (src/models/sovits_encp.rs:104-109):
 * out = LayerNorm2(x + conv_2(relu(conv_1(x)))) * x_mask, FeedForward::forward
 * (:371-375) with both convs padded (k - 1) / 2 (load_conv1d :378-410) and no
 * mask between them.  x, out [B, C, T]; w1 [F, C, k1]; w2 [C, F, k2]. */
int gsvo_encp_ffn(const float* x, int B, int C, int T, const float* w1, const float* b1, int F, int k1,
                  const float* w2, const float* b2, int k2, const float* gamma, const float* beta,
                  const int* lengths, float* out, int acc64) {
  float* h = (float*)malloc(sizeof(float) * (size_t)B * F * T);
  float* y = (float*)malloc(sizeof(float) * (size_t)B * C * T);
  int rc = (h && y) ? 0 : fail("encp_ffn: out of memory", NULL);
  if (!rc) rc = gsvo_conv1d(x, B, C, T, w1, F, k1, (k1 - 1) / 2, 1, b1, h, acc64);
  if (!rc) {
    for (int64_t i = 0; i < (int64_t)B * F * T; ++i) h[i] = h[i] > 0.0f ? h[i] : 0.0f;
    rc = gsvo_conv1d(h, B, F, T, w2, C, k2, (k2 - 1) / 2, 1, b2, y, acc64);
  }
  if (!rc) rc = gsvo_layer_norm(x, y, gamma, beta, B, C, T, 1e-5f, lengths, out);
  free(h);
  free(y);
  return rc;
}

/* linear_interpolate_last_dim (src/models/sovits_encp.rs:10-40): for each
 * output index i, source = max((i + 0.5) * (T / T_out) - 0.5, 0), low =
 * min(floor(source), T - 1), up = min(low + 1, T - 1), wu = source - low,
 * wl = wu * -1 + 1 (the affine), out = x[low] * wl + x[up] * wu, every step
 * rounded in f32 (the Makefile builds with -ffp-contract=off, so no step is
 * fused into an FMA).  T_out == T copies. */
int gsvo_interpolate(const float* x, int64_t rows, int T, int T_out, float* out) {
  if (T <= 0 || T_out <= 0) return fail("interpolation length must be positive", NULL);
  if (T_out == T) {
    memcpy(out, x, sizeof(float) * (size_t)rows * T);
    return 0;
  }
  const float scale = (float)T / (float)T_out;
  for (int i = 0; i < T_out; ++i) {
    float a = (float)i + 0.5f;
    float bsc = a * scale;
    float src = bsc - 0.5f;
    if (src < 0.0f) src = 0.0f;
    int low = (int)floorf(src);
    if (low > T - 1) low = T - 1;
    const int up = low + 1 < T - 1 ? low + 1 : T - 1;
    float wu = src - (float)low;
    float neg = wu * -1.0f;
    const float wl = neg + 1.0f;
    for (int64_t r = 0; r < rows; ++r) {
      float p = x[r * T + low] * wl;
      float q = x[r * T + up] * wu;
      out[r * T_out + i] = p + q;
    }
  }
  return 0;
}

/* EncP output projection and prior sample: stats = proj(y) * y_mask (a 1x1
 * conv, pad 0), m = stats[:, :Co], logs = clamp(stats[:, Co:], -5, 2)
 * (src/models/sovits_encp.rs:871-879), z_p = m + (noise * exp(logs)) *
 * noise_scale (src/models/sovits.rs:378-385).  w [2 Co, C, 1].  m, logs, z_p
 * may be NULL; z_p needs noise. */
int gsvo_encp_project(const float* y, int B, int C, int T, const float* w, const float* bias, int Co2,
                      const int* lengths, const float* noise, float noise_scale, float* m, float* logs,
                      float* z_p, int acc64) {
  if (Co2 % 2) return fail("encp_project: odd projection width", NULL);
  const int Co = Co2 / 2;
  float* st = (float*)malloc(sizeof(float) * (size_t)B * Co2 * T);
  if (!st) return fail("encp_project: out of memory", NULL);
  int rc = gsvo_conv1d(y, B, C, T, w, Co2, 1, 0, 1, bias, st, acc64);
  if (!rc) {
    for (int b = 0; b < B; ++b)
      for (int c = 0; c < Co; ++c)
        for (int t = 0; t < T; ++t) {
          const float mk = (lengths && t >= lengths[b]) ? 0.0f : 1.0f;
          const float mv = st[((int64_t)b * Co2 + c) * T + t] * mk;
          float lv = st[((int64_t)b * Co2 + Co + c) * T + t] * mk;
          lv = lv < -5.0f ? -5.0f : lv;
          lv = lv > 2.0f ? 2.0f : lv;
          const int64_t o = ((int64_t)b * Co + c) * T + t;
          if (m) m[o] = mv;
          if (logs) logs[o] = lv;
          if (z_p) {
            float e = noise[o] * expf(lv);
            float s = e * noise_scale;
            z_p[o] = mv + s;
          }
        }
  }
  free(st);
  return rc;
}
