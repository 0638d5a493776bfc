/*
 * cutetts_oracle.c -- CPU restatement of RCuteTTS's per-frame decode path.
 *
 * TEST INFRASTRUCTURE ONLY (the checker and the timed CPU baseline); the
 * shipped library never calls it.  Compile with -ffp-contract=off: every
 * fused multiply-add below is an explicit fmaf() where the reference Rust
 * kernels use FMA (simd.rs gemv8_fma / micro_8x8_fma), and every other sum
 * is the plain sequential `acc += a*b` the Rust loops compute.
 *
 * Each function cites the reference file:line it restates.  Paths are
 * relative to the RCuteTTS project root.
 */
#include "cutetts_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static int g_nth = 1;

void orc_set_threads(int nth) { g_nth = nth < 1 ? 1 : nth; }
int orc_get_threads(void) { return g_nth; }

/* ------------------------------------------------------------ primitives */

/* rust-codec/src/simd.rs:359-368 (gemv8_fma) and simd.rs:256-270
 * (micro_8x8_fma): accumulator starts at the bias, then one FMA per k in
 * ascending order.  Threads split output rows like qwen.rs:177-208
 * (disjoint rows => bitwise identical for any thread count). */
/* Many rows: x transposed to [I][S padded to 16] once, then each output
 * runs 16 rows side by side (one vector FMA per k); every output still
 * starts at its bias and takes one fmaf per k in ascending order, so the
 * result is bitwise the one of the row-by-row loop below. */
#define ORC_ROWS 16
static void linear_many_rows(const float* x, int S, int I, const float* W, const float* b, int O,
                             float* y, int nth) {
  const int Sp = (S + ORC_ROWS - 1) / ORC_ROWS * ORC_ROWS;
  float* xt = calloc((size_t)I * Sp, sizeof(float));
  for (int s = 0; s < S; s++)
    for (int i = 0; i < I; i++) xt[(size_t)i * Sp + s] = x[(size_t)s * I + i];
#pragma omp parallel for schedule(static) num_threads(nth) collapse(2)
  for (int o = 0; o < O; o++) {
    for (int s0 = 0; s0 < Sp; s0 += ORC_ROWS) {
      const float* wr = W + (size_t)o * I;
      const float bias = b ? b[o] : 0.0f;
      float acc[ORC_ROWS];
      for (int j = 0; j < ORC_ROWS; j++) acc[j] = bias;
      for (int i = 0; i < I; i++) {
        const float wv = wr[i];
        const float* xr = xt + (size_t)i * Sp + s0;
        for (int j = 0; j < ORC_ROWS; j++) acc[j] = fmaf(wv, xr[j], acc[j]);
      }
      const int ns = S - s0 < ORC_ROWS ? S - s0 : ORC_ROWS;
      for (int j = 0; j < ns; j++) y[(size_t)(s0 + j) * O + o] = acc[j];
    }
  }
  free(xt);
}

void orc_linear(const float* x, int S, int I, const float* W, const float* b, int O,
                float* y) {
  long ops = (long)S * I * O;
  int nth = ops >= 1000000 ? g_nth : 1;
  if (S >= ORC_ROWS) {
    linear_many_rows(x, S, I, W, b, O, y, nth);
    return;
  }
  const int nblk = (O + 7) / 8;
  /* eight output rows per task, each with its own sequential FMA chain
   * (the gemv8 panel shape); per-output arithmetic is unchanged. */
#pragma omp parallel for schedule(static) num_threads(nth)
  for (int blk = 0; blk < nblk; blk++) {
    const int o0 = blk * 8, nr = O - o0 < 8 ? O - o0 : 8;
    const float* wr[8];
    for (int r = 0; r < 8; r++) wr[r] = W + (size_t)(o0 + (r < nr ? r : 0)) * I;
    for (int s = 0; s < S; s++) {
      const float* xr = x + (size_t)s * I;
      float acc[8];
      for (int r = 0; r < 8; r++) acc[r] = (b && r < nr) ? b[o0 + r] : 0.0f;
      for (int i = 0; i < I; i++) {
        const float xv = xr[i];
        acc[0] = fmaf(wr[0][i], xv, acc[0]);
        acc[1] = fmaf(wr[1][i], xv, acc[1]);
        acc[2] = fmaf(wr[2][i], xv, acc[2]);
        acc[3] = fmaf(wr[3][i], xv, acc[3]);
        acc[4] = fmaf(wr[4][i], xv, acc[4]);
        acc[5] = fmaf(wr[5][i], xv, acc[5]);
        acc[6] = fmaf(wr[6][i], xv, acc[6]);
        acc[7] = fmaf(wr[7][i], xv, acc[7]);
      }
      for (int r = 0; r < nr; r++) y[(size_t)s * O + o0 + r] = acc[r];
    }
  }
}

/* rust-codec/src/dit.rs:247-255 */
void orc_rms_norm_row(const float* x, const float* w, int n, float eps, float* out) {
  float s = 0.0f;
  for (int i = 0; i < n; i++) s += x[i] * x[i];
  float inv = 1.0f / sqrtf(s / (float)n + eps);
  for (int i = 0; i < n; i++) out[i] = x[i] * inv * w[i];
}

/* rust-codec/src/qwen.rs:152-174 (inv[i] = theta^(-2i/d), angle = pos*inv[i]);
 * the DiT tables (dit.rs:277-306) compute the same rotate-half form. */
void orc_rope(const float* v, int d, int pos, float theta, float* out) {
  int h = d / 2;
  for (int i = 0; i < h; i++) {
    float inv = powf(theta, -((float)(2 * i)) / (float)d);
    float ang = (float)pos * inv;
    float s = sinf(ang), c = cosf(ang);
    float a = v[i], bb = v[h + i];
    out[i] = a * c - bb * s;
    out[h + i] = a * s + bb * c;
  }
}

/* rust-codec/src/dit.rs:308-319 */
void orc_softmax_row(float* x, int n) {
  float m = -INFINITY;
  for (int i = 0; i < n; i++) m = x[i] > m ? x[i] : m;
  float s = 0.0f;
  for (int i = 0; i < n; i++) {
    x[i] = expf(x[i] - m);
    s += x[i];
  }
  float inv = 1.0f / s;
  for (int i = 0; i < n; i++) x[i] *= inv;
}

static inline float silu(float g) { return g / (1.0f + expf(-g)); }

/* rust-codec/src/qwen.rs:304 / 370 */
void orc_swiglu(const float* g, const float* u, int n, float* out) {
  for (int i = 0; i < n; i++) out[i] = silu(g[i]) * u[i];
}

/* rust-codec/src/qwen.rs:409-417 */
int orc_embed_lookup(const float* table, int vocab, int hidden, const int64_t* ids,
                     int n, float* out) {
  for (int s = 0; s < n; s++) {
    if (ids[s] < 0 || ids[s] >= vocab) return -1;
    memcpy(out + (size_t)s * hidden, table + (size_t)ids[s] * hidden,
           sizeof(float) * hidden);
  }
  return 0;
}

/* ------------------------------------------------------------- LM (Qwen3) */

/* rust-codec/src/qwen.rs:229-310 (prefill) and 312-376 (decode).  The
 * prefill in the reference only attends to the tokens of the same call
 * (empty cache); decode attends to the whole cache.  Both are the special
 * cases of "token i sees cache rows [0, len+i]" restated here. */
void orc_lm_layer(const orc_lm_dims* d, const orc_lm_layer_w* w, const float* h, int T,
                  int pos0, float* kc, float* vc, int len, float* out) {
  const int H = d->hidden, hd = d->head_dim, nq = d->n_heads, nkv = d->n_kv;
  const int qdim = nq * hd, kvdim = nkv * hd, F = d->ffn;
  const float scale = 1.0f / sqrtf((float)hd);
  if (T <= 0) return;
  float* normed = malloc(sizeof(float) * (size_t)T * H);
  float* q = malloc(sizeof(float) * (size_t)T * qdim);
  float* k = malloc(sizeof(float) * (size_t)T * kvdim);
  float* v = malloc(sizeof(float) * (size_t)T * kvdim);
  float* att = malloc(sizeof(float) * (size_t)T * qdim);
  float* proj = malloc(sizeof(float) * (size_t)T * H);
  float* g = malloc(sizeof(float) * (size_t)T * F);
  float* u = malloc(sizeof(float) * (size_t)T * F);
  float* tmp = malloc(sizeof(float) * hd);
  float* tmp2 = malloc(sizeof(float) * hd);

  for (int s = 0; s < T; s++)
    orc_rms_norm_row(h + (size_t)s * H, w->norm1, H, d->eps, normed + (size_t)s * H);
  orc_linear(normed, T, H, w->wq, NULL, qdim, q);
  orc_linear(normed, T, H, w->wk, NULL, kvdim, k);
  orc_linear(normed, T, H, w->wv, NULL, kvdim, v);
  for (int s = 0; s < T; s++) {
    for (int hh = 0; hh < nq; hh++) {
      float* qh = q + (size_t)s * qdim + hh * hd;
      if (d->qk_norm) {
        orc_rms_norm_row(qh, w->qn, hd, d->eps, tmp2);
        orc_rope(tmp2, hd, pos0 + s, d->rope_theta, tmp);
      } else {
        orc_rope(qh, hd, pos0 + s, d->rope_theta, tmp);
      }
      memcpy(qh, tmp, sizeof(float) * hd);
    }
    float* krow = kc + (size_t)(len + s) * kvdim;
    float* vrow = vc + (size_t)(len + s) * kvdim;
    for (int kh = 0; kh < nkv; kh++) {
      float* kh_ = k + (size_t)s * kvdim + kh * hd;
      if (d->qk_norm) {
        orc_rms_norm_row(kh_, w->kn, hd, d->eps, tmp2);
        orc_rope(tmp2, hd, pos0 + s, d->rope_theta, krow + kh * hd);
      } else {
        orc_rope(kh_, hd, pos0 + s, d->rope_theta, krow + kh * hd);
      }
    }
    memcpy(vrow, v + (size_t)s * kvdim, sizeof(float) * kvdim);
  }
  /* attention: qwen.rs:341-362 */
  const int group = nq / nkv;
  int ncache = len + T;
  int nth = (long)ncache * T * nq * hd >= 200000 ? g_nth : 1;
  /* Every score is sum_dd q*k in dd order and every output sum_j p*v in j
   * order, as in qwen.rs:341-362; the loops run many keys (scores, keys
   * transposed once per call) or many dims (outputs) side by side. */
  float* kt = malloc(sizeof(float) * (size_t)nkv * hd * ncache);
  for (int kh = 0; kh < nkv; kh++)
    for (int j = 0; j < ncache; j++)
      for (int dd = 0; dd < hd; dd++)
        kt[((size_t)kh * hd + dd) * ncache + j] = kc[(size_t)j * kvdim + kh * hd + dd];
#pragma omp parallel num_threads(nth)
  {
    float* scores = malloc(sizeof(float) * ncache);
    float* acc = malloc(sizeof(float) * hd);
#pragma omp for schedule(static) collapse(2)
    for (int hh = 0; hh < nq; hh++) {
      for (int i = 0; i < T; i++) {
        int kh = hh / group;
        int n = len + i + 1;
        const float* qi = q + (size_t)i * qdim + hh * hd;
        for (int j = 0; j < n; j++) scores[j] = 0.0f;
        for (int dd = 0; dd < hd; dd++) {
          const float qv = qi[dd];
          const float* kr = kt + ((size_t)kh * hd + dd) * ncache;
          for (int j = 0; j < n; j++) scores[j] += qv * kr[j];
        }
        for (int j = 0; j < n; j++) scores[j] *= scale;
        orc_softmax_row(scores, n);
        for (int dd = 0; dd < hd; dd++) acc[dd] = 0.0f;
        for (int j = 0; j < n; j++) {
          const float p = scores[j];
          const float* vr = vc + (size_t)j * kvdim + kh * hd;
          for (int dd = 0; dd < hd; dd++) acc[dd] += p * vr[dd];
        }
        for (int dd = 0; dd < hd; dd++) att[(size_t)i * qdim + hh * hd + dd] = acc[dd];
      }
    }
    free(scores);
    free(acc);
  }
  free(kt);
  orc_linear(att, T, qdim, w->wo, NULL, H, proj);
  float* h2 = out;
  for (size_t i = 0; i < (size_t)T * H; i++) h2[i] = h[i] + proj[i];
  for (int s = 0; s < T; s++)
    orc_rms_norm_row(h2 + (size_t)s * H, w->norm2, H, d->eps, normed + (size_t)s * H);
  orc_linear(normed, T, H, w->wg, NULL, F, g);
  orc_linear(normed, T, H, w->wu, NULL, F, u);
  orc_swiglu(g, u, T * F, g);
  orc_linear(g, T, F, w->wd, NULL, H, proj);
  for (size_t i = 0; i < (size_t)T * H; i++) h2[i] += proj[i];

  free(normed); free(q); free(k); free(v); free(att); free(proj);
  free(g); free(u); free(tmp); free(tmp2);
}

/* rust-codec/src/qwen.rs:379-406 */
void orc_lm_forward(const orc_lm_dims* d, int n_layers, const orc_lm_layer_w* layers,
                    const float* final_norm, const float* x, int T, int pos0, float** kc,
                    float** vc, int len, float* out) {
  const int H = d->hidden;
  float* a = malloc(sizeof(float) * (size_t)T * H);
  float* b = malloc(sizeof(float) * (size_t)T * H);
  memcpy(a, x, sizeof(float) * (size_t)T * H);
  for (int l = 0; l < n_layers; l++) {
    orc_lm_layer(d, &layers[l], a, T, pos0, kc[l], vc[l], len, b);
    float* t = a; a = b; b = t;
  }
  for (int s = 0; s < T; s++)
    orc_rms_norm_row(a + (size_t)s * H, final_norm, H, d->eps, out + (size_t)s * H);
  free(a);
  free(b);
}

/* ------------------------------------------------------------- DiT head */

/* diffusion_head.py:306-320 (dit.rs:262-273): half = dim/2,
 * e = ln(10000)/(half-1), v_i = (1000*x) * exp(-e*i), [sin(v), cos(v)]. */
void orc_sin_emb(float x, int dim, float* out) {
  int half = dim / 2;
  float e = (float)(log(10000.0) / (double)(half - 1));
  for (int i = 0; i < half; i++) {
    float f = expf((float)i * -e);
    float v = (1000.0f * x) * f;
    out[i] = sinf(v);
    out[half + i] = cosf(v);
  }
}

/* rust-codec/src/dit.rs:846-854 */
void orc_sway_timesteps(int steps, float coeff, float* out) {
  for (int s = 0; s <= steps; s++) {
    float u = (float)s / (float)steps;
    out[s] = u + coeff * (cosf(0.5f * (float)M_PI * u) - 1.0f + u);
  }
}

/* TimestepEmbedding: Linear -> SiLU -> Linear (diffusion_head.py:323-331,
 * dit.rs:651-656). */
static void time_mlp(const float* x, int H, const float* w1, const float* b1,
                     const float* w2, const float* b2, float* out) {
  float* hbuf = malloc(sizeof(float) * H);
  orc_linear(x, 1, H, w1, b1, H, hbuf);
  for (int i = 0; i < H; i++) hbuf[i] = silu(hbuf[i]);
  orc_linear(hbuf, 1, H, w2, b2, H, out);
  free(hbuf);
}

/* One LocalTransformerLayer on seq rows (diffusion_head.py:198-264,
 * dit.rs:323-435).  ad: [6*H] adaln chunks (shift/scale/gate attn, shift/
 * scale/gate mlp) or NULL for the plain residual path. */
static void dit_layer(const orc_dit_dims* d, const orc_dit_layer_w* lw, float* hs, int seq,
                      const float* ad) {
  const int H = d->hidden, hd = d->head_dim, nq = d->n_heads, nkv = d->n_kv, F = d->ffn;
  const int kvdim = nkv * hd, group = nq / nkv;
  const float scale = 1.0f / sqrtf((float)hd);
  float* normed = malloc(sizeof(float) * seq * H);
  float* q = malloc(sizeof(float) * seq * H);
  float* k = malloc(sizeof(float) * seq * kvdim);
  float* v = malloc(sizeof(float) * seq * kvdim);
  float* att = malloc(sizeof(float) * seq * H);
  float* proj = malloc(sizeof(float) * seq * H);
  float* g = malloc(sizeof(float) * seq * F);
  float* u = malloc(sizeof(float) * seq * F);
  float* qr = malloc(sizeof(float) * seq * hd);
  float* kr = malloc(sizeof(float) * seq * hd);
  float* scores = malloc(sizeof(float) * seq * seq);

  for (int s = 0; s < seq; s++) {
    float* nr = normed + s * H;
    orc_rms_norm_row(hs + s * H, lw->norm1, H, d->eps, nr);
    if (ad)
      for (int i = 0; i < H; i++) nr[i] = nr[i] * (1.0f + ad[H + i]) + ad[i];
  }
  orc_linear(normed, seq, H, lw->wq, NULL, H, q);
  orc_linear(normed, seq, H, lw->wk, NULL, kvdim, k);
  orc_linear(normed, seq, H, lw->wv, NULL, kvdim, v);
  for (int hh = 0; hh < nq; hh++) {
    int kh = hh / group;
    for (int s = 0; s < seq; s++) {
      orc_rope(q + s * H + hh * hd, hd, s, d->rope_theta, qr + s * hd);
      orc_rope(k + s * kvdim + kh * hd, hd, s, d->rope_theta, kr + s * hd);
    }
    for (int i = 0; i < seq; i++) {
      for (int j = 0; j < seq; j++) {
        float acc = 0.0f;
        for (int dd = 0; dd < hd; dd++) acc += qr[i * hd + dd] * kr[j * hd + dd];
        scores[i * seq + j] = acc * scale;
      }
      orc_softmax_row(scores + i * seq, seq);
    }
    for (int i = 0; i < seq; i++) {
      for (int dd = 0; dd < hd; dd++) {
        float acc = 0.0f;
        for (int j = 0; j < seq; j++) acc += scores[i * seq + j] * v[j * kvdim + kh * hd + dd];
        att[i * H + hh * hd + dd] = acc;
      }
    }
  }
  orc_linear(att, seq, H, lw->wo, NULL, H, proj);
  for (int s = 0; s < seq; s++)
    for (int i = 0; i < H; i++)
      hs[s * H + i] += (ad ? 1.0f + ad[2 * H + i] : 1.0f) * proj[s * H + i];

  for (int s = 0; s < seq; s++) {
    float* nr = normed + s * H;
    orc_rms_norm_row(hs + s * H, lw->norm2, H, d->eps, nr);
    if (ad)
      for (int i = 0; i < H; i++) nr[i] = nr[i] * (1.0f + ad[4 * H + i]) + ad[3 * H + i];
  }
  orc_linear(normed, seq, H, lw->wg, NULL, F, g);
  orc_linear(normed, seq, H, lw->wu, NULL, F, u);
  orc_swiglu(g, u, seq * F, g);
  orc_linear(g, seq, F, lw->wd, NULL, H, proj);
  for (int s = 0; s < seq; s++)
    for (int i = 0; i < H; i++)
      hs[s * H + i] += (ad ? 1.0f + ad[5 * H + i] : 1.0f) * proj[s * H + i];

  free(normed); free(q); free(k); free(v); free(att); free(proj);
  free(g); free(u); free(qr); free(kr); free(scores);
}

/* locenc_embed (locenc.rs:222-255): per item the sequence [CLS, in_proj of
 * the patch frames], plain LocalTransformer layers, final RMSNorm of the CLS
 * row, then locenc_to_lm_proj (model.py:128-130). */
void orc_locenc_embed(const orc_dit_dims* d, const orc_locenc_w* w, const float* x, int n, float* out) {
  const int H = d->hidden, P = d->patch, S = 1 + P, L = d->latent;
  float* hs = malloc(sizeof(float) * S * H);
  float* cls = malloc(sizeof(float) * H);
  for (int it = 0; it < n; it++) {
    memcpy(hs, w->special, sizeof(float) * H);
    orc_linear(x + (size_t)it * P * L, P, L, w->in_w, w->in_b, H, hs + H);
    for (int l = 0; l < d->n_layers; l++) dit_layer(d, &w->layers[l], hs, S, NULL);
    orc_rms_norm_row(hs, w->final_norm, H, d->eps, cls);
    orc_linear(cls, 1, H, w->proj_w, w->proj_b, w->out_dim, out + (size_t)it * w->out_dim);
  }
  free(hs);
  free(cls);
}

/* Per-sample constants (dit.rs:756-772 sample_prologue): dt_emb, the
 * mu token without t_emb (mu_proj(z) + cfg + step), per-layer adaln. */
typedef struct {
  float* mu;   /* [H] */
  float* dt_emb;
  float* ad;   /* [n_layers][6H] or NULL */
} prologue_t;

static void prologue(const orc_dit_dims* d, const orc_dit_w* w, const float* z,
                     const float* spk, float dt, float cfg_w, prologue_t* p) {
  const int H = d->hidden;
  float* se = malloc(sizeof(float) * H);
  float* tmp = malloc(sizeof(float) * H);
  p->mu = malloc(sizeof(float) * H);
  p->dt_emb = malloc(sizeof(float) * H);
  /* mu = mu_proj(z) (+ cfg_strength + step_size) : diffusion_head.py:601-627 */
  if (w->mu_w)
    orc_linear(z, 1, d->cond_dim, w->mu_w, w->mu_b, H, p->mu);
  else
    memcpy(p->mu, z, sizeof(float) * H);
  if (w->cfg0_w && w->cfg2_w) {
    float wn = cfg_w / 5.0f;
    float* hh = malloc(sizeof(float) * H);
    orc_linear(&wn, 1, 1, w->cfg0_w, NULL, H, hh);
    for (int i = 0; i < H; i++) hh[i] = silu(hh[i]);
    orc_linear(hh, 1, H, w->cfg2_w, NULL, H, tmp);
    for (int i = 0; i < H; i++) p->mu[i] += tmp[i];
    free(hh);
  }
  if (w->st1_w) {
    orc_sin_emb(dt, H, se);
    time_mlp(se, H, w->st1_w, w->st1_b, w->st2_w, w->st2_b, tmp);
    for (int i = 0; i < H; i++) p->mu[i] += tmp[i];
  }
  orc_sin_emb(0.0f, H, se);
  time_mlp(se, H, w->dt1_w, w->dt1_b, w->dt2_w, w->dt2_b, p->dt_emb);
  p->ad = NULL;
  if (spk) {
    p->ad = malloc(sizeof(float) * (size_t)d->n_layers * 6 * H);
    for (int l = 0; l < d->n_layers; l++) {
      if (w->layers[l].adaln)
        orc_linear(spk, 1, d->spk_dim, w->layers[l].adaln, NULL, 6 * H, p->ad + (size_t)l * 6 * H);
      else
        memset(p->ad + (size_t)l * 6 * H, 0, sizeof(float) * 6 * H);
    }
  }
  free(se);
  free(tmp);
}

static void prologue_free(prologue_t* p) {
  free(p->mu);
  free(p->dt_emb);
  free(p->ad);
}

/* _predict with cached conditions (dit.rs:775-814, diffusion_head.py:544-635):
 * seq = [mu + t_emb + dt_emb, cond_proj(cond), in_proj(x)] -> layers ->
 * final norm -> out_proj(last `patch` rows). */
static void predict_cached(const orc_dit_dims* d, const orc_dit_w* w, const float* x,
                           float t, const float* cond, const prologue_t* p, float* v) {
  const int H = d->hidden, P = d->patch, L = d->latent;
  const int seq = 1 + 2 * P;
  float* hs = malloc(sizeof(float) * seq * H);
  float* se = malloc(sizeof(float) * H);
  float* temb = malloc(sizeof(float) * H);
  float* nrm = malloc(sizeof(float) * P * H);
  orc_linear(cond, P, L, w->cond_w, w->cond_b, H, hs + H);
  orc_linear(x, P, L, w->in_w, w->in_b, H, hs + (1 + P) * H);
  orc_sin_emb(t, H, se);
  time_mlp(se, H, w->t1_w, w->t1_b, w->t2_w, w->t2_b, temb);
  for (int i = 0; i < H; i++) hs[i] = (p->mu[i] + temb[i]) + p->dt_emb[i];
  for (int l = 0; l < d->n_layers; l++)
    dit_layer(d, &w->layers[l], hs, seq, p->ad ? p->ad + (size_t)l * 6 * H : NULL);
  for (int s = 0; s < P; s++)
    orc_rms_norm_row(hs + (1 + P + s) * H, w->final_norm, H, d->eps, nrm + s * H);
  orc_linear(nrm, P, H, w->out_w, w->out_b, L, v);
  free(hs); free(se); free(temb); free(nrm);
}

void orc_dit_predict(const orc_dit_dims* d, const orc_dit_w* w, const float* x, float t,
                     const float* z, const float* cond, float dt, const float* spk,
                     float cfg_w, float* v) {
  prologue_t p;
  prologue(d, w, z, spk, dt, cfg_w, &p);
  predict_cached(d, w, x, t, cond, &p, v);
  prologue_free(&p);
}

/* rust-codec/src/dit.rs:819-842 (diffusion_head.py:637-697 at cfg=0):
 * t_s = s*dt, x += v*dt. */
void orc_dit_euler_sample(const orc_dit_dims* d, const orc_dit_w* w, const float* x0,
                          const float* z, const float* cond, const float* spk, int steps,
                          float cfg_w, float* x_out) {
  const int n = d->patch * d->latent;
  float dt = 1.0f / (float)steps;
  prologue_t p;
  prologue(d, w, z, spk, dt, cfg_w, &p);
  float* v = malloc(sizeof(float) * n);
  memcpy(x_out, x0, sizeof(float) * n);
  for (int s = 0; s < steps; s++) {
    float t = (float)s * dt;
    predict_cached(d, w, x_out, t, cond, &p, v);
    for (int i = 0; i < n; i++) x_out[i] += v[i] * dt;
  }
  free(v);
  prologue_free(&p);
}

/* rust-codec/src/dit.rs:862-900: sway grid, two branches, the uncond branch
 * feeds a zero speaker row through AdaLN (exact zeros), v = vc + cfg*(vc-vu). */
void orc_dit_euler_sample_cfg(const orc_dit_dims* d, const orc_dit_w* w, const float* x0,
                              const float* z_c, const float* z_u, const float* cond,
                              const float* uncond, const float* spk, int steps,
                              float coeff, float cfg, float* x_out) {
  const int n = d->patch * d->latent, H = d->hidden;
  prologue_t pc, pu;
  prologue(d, w, z_c, spk, 1.0f / (float)steps, cfg, &pc);
  prologue(d, w, z_u, spk, 1.0f / (float)steps, cfg, &pu);
  if (pu.ad) memset(pu.ad, 0, sizeof(float) * (size_t)d->n_layers * 6 * H);
  float* times = malloc(sizeof(float) * (steps + 1));
  orc_sway_timesteps(steps, coeff, times);
  float* vc = malloc(sizeof(float) * n);
  float* vu = malloc(sizeof(float) * n);
  memcpy(x_out, x0, sizeof(float) * n);
  for (int s = 0; s < steps; s++) {
    float t = times[s], dt = times[s + 1] - times[s];
    predict_cached(d, w, x_out, t, cond, &pc, vc);
    predict_cached(d, w, x_out, t, uncond, &pu, vu);
    for (int i = 0; i < n; i++) x_out[i] += (vc[i] + cfg * (vc[i] - vu[i])) * dt;
  }
  free(times); free(vc); free(vu);
  prologue_free(&pc);
  prologue_free(&pu);
}

/* ----------------------------------------------------------- VAE decoder */

/* rust-codec/src/snake.rs:26-36: x += (1/(a+1e-9)) * sin(a*x)^2 */
void orc_snake(float* x, int C, int T, const float* alpha) {
  int nth = (long)C * T >= 200000 ? g_nth : 1;
#pragma omp parallel for schedule(static) num_threads(nth)
  for (int c = 0; c < C; c++) {
    float a = alpha[c];
    float inv = 1.0f / (a + 1e-9f);
    float* row = x + (size_t)c * T;
    for (int t = 0; t < T; t++) {
      float s = sinf(row[t] * a);
      row[t] += inv * s * s;
    }
  }
}

/* rust-codec/src/conv.rs:12-30: w = g * v / ||v|| per out channel, in f64 */
void orc_fuse_weight_norm(const float* g, const float* v, int O, int IK, float* w) {
  for (int o = 0; o < O; o++) {
    double s = 0.0;
    for (int i = 0; i < IK; i++) {
      double x = v[(size_t)o * IK + i];
      s += x * x;
    }
    double nrm = sqrt(s);
    double scale = (double)g[o] / (nrm > 1e-12 ? nrm : 1e-12);
    for (int i = 0; i < IK; i++) w[(size_t)o * IK + i] = (float)((double)v[(size_t)o * IK + i] * scale);
  }
}

/* rust-codec/src/conv.rs:36-115: left pad 2*pad, bias first, then channels
 * ascending, taps ascending; k=1 rows use the SAXPY order (channel-outer). */
void orc_causal_conv1d(const float* x, int c_in, int T, const float* w, const float* b,
                       int c_out, int k, int dil, int groups, int pad, float* out) {
  const int cig = c_in / groups, cog = c_out / groups, left = 2 * pad;
  long ops = (long)c_out * T * cig * k;
  int nth = ops >= 200000 ? g_nth : 1;
#pragma omp parallel for schedule(static) num_threads(nth)
  for (int o = 0; o < c_out; o++) {
    int grp = o / cog, c0 = grp * cig;
    float* orow = out + (size_t)o * T;
    if (k == 1 && dil == 1 && pad == 0) {
      for (int t = 0; t < T; t++) orow[t] = b[o];
      for (int ci = 0; ci < cig; ci++) {
        float s = w[(size_t)o * cig + ci];
        const float* xr = x + (size_t)(c0 + ci) * T;
        for (int t = 0; t < T; t++) orow[t] += xr[t] * s;
      }
      continue;
    }
    /* Each output sample is bias, then + x*w over channels ascending and
     * taps ascending (taps before the signal start skipped), one rounding
     * per product and per add.  The loop runs that sequence for a block of
     * samples at once (time innermost, vectorised); the per-sample order is
     * the one of conv.rs:53-115. */
    enum { TB = 2048 };
    for (int t0 = 0; t0 < T; t0 += TB) {
      const int t1 = t0 + TB < T ? t0 + TB : T;
      for (int t = t0; t < t1; t++) orow[t] = b[o];
      for (int ci = 0; ci < cig; ci++) {
        const float* xr = x + (size_t)(c0 + ci) * T;
        const float* wr = w + ((size_t)o * cig + ci) * k;
        for (int kk = 0; kk < k; kk++) {
          const int off = kk * dil - left;
          const int ts = t0 > -off ? t0 : -off;
          const float wv = wr[kk];
          for (int t = ts; t < t1; t++) orow[t] += xr[t + off] * wv;
        }
      }
    }
  }
}

/* rust-codec/src/conv.rs:153-210: full transpose conv (padding 0) then the
 * right trim of 2*pad - out_pad samples, bias added last. */
void orc_causal_transpose_conv1d(const float* x, int c_in, int T, const float* w,
                                 const float* b, int c_out, int k, int stride, int groups,
                                 int pad, int out_pad, float* out) {
  const int cog = c_out / groups, cig = c_in / groups;
  const int full_t = (T - 1) * stride + k;
  const int out_t = full_t - (2 * pad - out_pad);
  long ops = (long)c_out * T * cig * k;
  int nth = ops >= 200000 ? g_nth : 1;
#pragma omp parallel num_threads(nth)
  {
    float* frow = malloc(sizeof(float) * full_t);
#pragma omp for schedule(static)
    for (int o = 0; o < c_out; o++) {
      int grp = o / cog, og = o % cog;
      memset(frow, 0, sizeof(float) * full_t);
      for (int cg = 0; cg < cig; cg++) {
        int c = grp * cig + cg;
        const float* xi = x + (size_t)c * T;
        const float* wr = w + ((size_t)c * cog + og) * k;
        for (int i = 0; i < T; i++) {
          float xv = xi[i];
          if (xv == 0.0f) continue;
          float* fb = frow + (size_t)i * stride;
          for (int kk = 0; kk < k; kk++) fb[kk] += xv * wr[kk];
        }
      }
      for (int t = 0; t < out_t; t++) out[(size_t)o * out_t + t] = frow[t] + b[o];
    }
    free(frow);
  }
}

/* CausalResidualUnit (audio_vae.py:98-123): x + conv1(snake(conv7(snake(x)))) */
static void res_unit(float* h, int C, int T, int dil, const orc_res_w* r, int groups) {
  size_t n = (size_t)C * T;
  float* a = malloc(sizeof(float) * n);
  float* bb = malloc(sizeof(float) * n);
  memcpy(a, h, sizeof(float) * n);
  orc_snake(a, C, T, r->a0);
  orc_causal_conv1d(a, C, T, r->w0, r->b0, C, 7, dil, groups, (6 * dil) / 2, bb);
  orc_snake(bb, C, T, r->a1);
  orc_causal_conv1d(bb, C, T, r->w1, r->b1, C, 1, 1, 1, 0, a);
  for (size_t i = 0; i < n; i++) h[i] += a[i];
  free(a);
  free(bb);
}

/* CausalDecoder.forward (audio_vae.py:243-292; decode.rs:94-136) */
void orc_vae_decode(const orc_vae_w* w, const float* latent, int T, float* wav) {
  int ch = w->channels;
  float* h = malloc(sizeof(float) * (size_t)ch * T);
  if (w->depthwise) {
    float* t0 = malloc(sizeof(float) * (size_t)w->latent * T);
    orc_causal_conv1d(latent, w->latent, T, w->front_w, w->front_b, w->latent, 7, 1, w->latent, 3, t0);
    orc_causal_conv1d(t0, w->latent, T, w->front_pw_w, w->front_pw_b, ch, 1, 1, 1, 0, h);
    free(t0);
  } else {
    orc_causal_conv1d(latent, w->latent, T, w->front_w, w->front_b, ch, 7, 1, 1, 3, h);
  }
  int t = T;
  for (int si = 0; si < w->n_stages; si++) {
    int s = w->strides[si];
    int cin = w->channels >> si, cout = w->channels >> (si + 1);
    const orc_stage_w* st = &w->stages[si];
    orc_snake(h, cin, t, st->alpha);
    int pad = (s + 1) / 2, opad = s % 2;
    int out_t = (t - 1) * s + 2 * s - (2 * pad - opad);
    float* h2 = malloc(sizeof(float) * (size_t)cout * out_t);
    orc_causal_transpose_conv1d(h, cin, t, st->tw, st->tb, cout, 2 * s, s, 1, pad, opad, h2);
    free(h);
    h = h2;
    t = out_t;
    int groups = w->depthwise ? cout : 1;
    static const int dils[3] = {1, 3, 9};
    for (int r = 0; r < 3; r++) res_unit(h, cout, t, dils[r], &st->res[r], groups);
    ch = cout;
  }
  orc_snake(h, ch, t, w->final_alpha);
  orc_causal_conv1d(h, ch, t, w->final_w, w->final_b, 1, 7, 1, 1, 3, wav);
  for (int i = 0; i < t; i++) wav[i] = tanhf(wav[i]);
  free(h);
}

/* rust-codec/src/e2e.rs:83-92 (bias first, sequential non-fused sum) */
void orc_stop_logits(const float* w, const float* b, int H, const float* h, float* out2) {
  for (int r = 0; r < 2; r++) {
    float acc = b[r];
    for (int i = 0; i < H; i++) acc += w[(size_t)r * H + i] * h[i];
    out2[r] = acc;
  }
}
