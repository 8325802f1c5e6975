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
  char key[160];
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
  char key[160];
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
  char key[160];
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
