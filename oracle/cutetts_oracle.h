/*
 * cutetts_oracle.h -- CPU restatement of RCuteTTS's per-frame decode path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker the parity tests,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg compare the CUDA
 * path against.  The product (rcutetts_b200) never links or calls it.
 *
 * Every routine restates the arithmetic of the reference Rust crate
 * (rust-codec/src/{qwen,dit,conv,snake,decode,e2e}.rs) at generic shapes:
 * same op order (bias first, then K ascending with a fused multiply-add for
 * the linears, sequential non-fused sums for norms / attention), same
 * formulas for RMSNorm, NeoX RoPE, softmax, SwiGLU, AdaLN-Zero, the Euler
 * flow update, the causal (transpose) convolutions and Snake.  Where the
 * Rust port lacks a module that the upstream torch model has (the DiT's
 * mu_proj Linear, diffusion_head.py:421,601) it follows the torch module.
 *
 * Layouts: activations row-major [rows, features]; Linear weights [out, in]
 * row-major (torch nn.Linear layout, not the Rust MR=8 packed panels -- the
 * packing only changes memory order, not arithmetic); conv activations
 * channel-first [C, T]; conv weights [out, in/groups, k]; transpose-conv
 * weights [in, out/groups, k] (torch ConvTranspose1d layout).
 */
#ifndef CUTETTS_ORACLE_H
#define CUTETTS_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------ primitives */
void orc_set_threads(int nth);
int orc_get_threads(void);

/* y[s,o] = b[o] + sum_i W[o,i] x[s,i]  (gemm.rs:230-291 / simd.rs:359-368 order) */
void orc_linear(const float* x, int S, int I, const float* W, const float* b, int O,
                float* y);
/* rms_norm_row (dit.rs:247-255) */
void orc_rms_norm_row(const float* x, const float* w, int n, float eps, float* out);
/* NeoX rotate-half RoPE of one head vector at absolute position (qwen.rs:152-174) */
void orc_rope(const float* v, int d, int pos, float theta, float* out);
/* max-subtracted softmax (dit.rs:308-319) */
void orc_softmax_row(float* x, int n);
/* silu(g)*u elementwise (qwen.rs:304,370) */
void orc_swiglu(const float* g, const float* u, int n, float* out);
/* embedding row gather (qwen.rs:409-417); returns -1 on an out-of-range id */
int orc_embed_lookup(const float* table, int vocab, int hidden, const int64_t* ids,
                     int n, float* out);

/* ------------------------------------------------------------- LM (Qwen3) */
typedef struct {
  int hidden, n_heads, n_kv, head_dim, ffn;
  float eps, rope_theta;
  int qk_norm; /* 1: per-head RMSNorm on q and k before RoPE (Qwen3) */
} orc_lm_dims;

typedef struct {
  const float *norm1, *norm2, *wq, *wk, *wv, *wo, *qn, *kn, *wg, *wu, *wd;
} orc_lm_layer_w;

/* One decoder layer over T new tokens at positions pos0.. (qwen.rs:229-376).
 * kc/vc hold this layer's cache, row = n_kv*head_dim floats, rows [0,len)
 * valid; the T new post-RoPE K rows / V rows are appended at [len, len+T).
 * Token i attends cache rows [0, len+i]. */
void orc_lm_layer(const orc_lm_dims* d, const orc_lm_layer_w* w, const float* h, int T,
                  int pos0, float* kc, float* vc, int len, float* out);

/* All layers + final RMSNorm (prefill qwen.rs:379-391 / decode_step 394-406).
 * kc[l], vc[l]: per-layer caches. */
void orc_lm_forward(const orc_lm_dims* d, int n_layers, const orc_lm_layer_w* layers,
                    const float* final_norm, const float* x, int T, int pos0, float** kc,
                    float** vc, int len, float* out);

/* ------------------------------------------------------------- DiT head */
typedef struct {
  int latent, hidden, n_heads, n_kv, head_dim, ffn, n_layers, patch, cond_dim, spk_dim;
  float eps, rope_theta;
} orc_dit_dims;

typedef struct {
  const float *norm1, *norm2, *wq, *wk, *wv, *wo, *wg, *wu, *wd;
  const float* adaln; /* [6*hidden, spk_dim] or NULL */
} orc_dit_layer_w;

typedef struct {
  const float *in_w, *in_b, *cond_w, *cond_b;
  const float *mu_w, *mu_b; /* NULL => identity (cond_dim == hidden) */
  const float *out_w, *out_b;
  const float *t1_w, *t1_b, *t2_w, *t2_b;   /* time_mlp */
  const float *dt1_w, *dt1_b, *dt2_w, *dt2_b; /* delta_time_mlp */
  const float *st1_w, *st1_b, *st2_w, *st2_b; /* step_size_embedding or NULL */
  const float *cfg0_w, *cfg2_w;               /* cfg_strength_embedding or NULL */
  const float* final_norm;
  const orc_dit_layer_w* layers;
} orc_dit_w;

/* LocEnc + locenc_to_lm_proj (locenc.rs:222-255 locenc_embed,
 * diffusion_head.py:334-378 AudioLocEnc, model.py:128-130): dims use
 * latent (input), hidden, n_heads, n_kv, head_dim, ffn, n_layers, patch,
 * eps, rope_theta of orc_dit_dims; layers are plain (adaln NULL). */
typedef struct {
  const float *in_w, *in_b, *special, *final_norm, *proj_w, *proj_b;
  const orc_dit_layer_w* layers;
  int out_dim;
} orc_locenc_w;
/* x [n][patch][latent] -> out [n][out_dim] */
void orc_locenc_embed(const orc_dit_dims* d, const orc_locenc_w* w, const float* x, int n, float* out);

/* SinusoidalPosEmb (diffusion_head.py:306-320, dit.rs:262-273) */
void orc_sin_emb(float x, int dim, float* out);
/* sway_timesteps (dit.rs:846-854) -> steps+1 floats */
void orc_sway_timesteps(int steps, float coeff, float* out);
/* _predict (diffusion_head.py:544-635 / dit.rs:681-737) for one utterance:
 * x,cond [patch*latent], z [cond_dim], spk [spk_dim] or NULL -> v [patch*latent] */
void orc_dit_predict(const orc_dit_dims* d, const orc_dit_w* w, const float* x, float t,
                     const float* z, const float* cond, float dt, const float* spk,
                     float cfg_w, float* v);
/* euler_sample (dit.rs:819-842, uniform grid t_s = s/steps) */
void orc_dit_euler_sample(const orc_dit_dims* d, const orc_dit_w* w, const float* x0,
                          const float* z, const float* cond, const float* spk, int steps,
                          float cfg_w, float* x_out);
/* euler_sample_cfg (dit.rs:862-900): sway grid + v = vc + cfg*(vc - vu) */
void orc_dit_euler_sample_cfg(const orc_dit_dims* d, const orc_dit_w* w, const float* x0,
                              const float* z_c, const float* z_u, const float* cond,
                              const float* uncond, const float* spk, int steps,
                              float coeff, float cfg, float* x_out);

/* ----------------------------------------------------------- VAE decoder */
void orc_snake(float* x, int C, int T, const float* alpha);
void orc_fuse_weight_norm(const float* g, const float* v, int O, int IK, float* w);
void orc_causal_conv1d(const float* x, int c_in, int T, const float* w, const float* b,
                       int c_out, int k, int dil, int groups, int pad, float* out);
/* out_t = (T-1)*stride + k - (2*pad - out_pad) */
void orc_causal_transpose_conv1d(const float* x, int c_in, int T, const float* w,
                                 const float* b, int c_out, int k, int stride, int groups,
                                 int pad, int out_pad, float* out);

typedef struct {
  const float *a0, *w0, *b0, *a1, *w1, *b1; /* Snake, conv k7 dil, Snake, conv k1 */
} orc_res_w;

typedef struct {
  const float *alpha, *tw, *tb; /* Snake + ConvTranspose1d(k=2s) */
  orc_res_w res[3];
} orc_stage_w;

typedef struct {
  int latent, channels, n_stages, depthwise;
  int strides[8];
  const float *front_w, *front_b;       /* dense [ch,latent,7]; depthwise [latent,1,7] */
  const float *front_pw_w, *front_pw_b; /* depthwise only: [ch,latent,1] */
  const orc_stage_w* stages;
  const float *final_alpha, *final_w, *final_b;
} orc_vae_w;

/* CausalDecoder.forward (audio_vae.py:243-292, decode.rs:94-136):
 * latent [latent, T] -> wav [T*prod(strides)] */
void orc_vae_decode(const orc_vae_w* w, const float* latent, int T, float* wav);

/* --------------------------------------------------- per-frame AR loop */
/* Stop head Linear(H,2) (e2e.rs:83-92). */
void orc_stop_logits(const float* w, const float* b, int H, const float* h, float* out2);

#ifdef __cplusplus
}
#endif
#endif
