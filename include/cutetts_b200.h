/*
 * cutetts_b200.h -- C ABI of the B200 (sm_100a) per-frame decode path.
 *
 * The reference crate (RCuteTTS rust-codec) exposes its hot path as Rust
 * functions (qwen.rs, dit.rs, decode.rs, e2e.rs) plus a three-function C ABI
 * for the VAE (ffi.rs).  This header is the boundary a Rust (or any FFI)
 * host binds instead: every entry point names the reference function it
 * replaces.  Plain pointers and sizes only; no C++ or torch types.
 *
 * Conventions
 *  - Every function returns an int status: CTTS_OK (0) or a negative code.
 *    ctts_last_error() gives a one-line message for the calling thread.
 *  - Handles bind one device.  Entry points named *_dev take device
 *    pointers and a cudaStream_t passed as void* (NULL = the handle's own
 *    stream) and are asynchronous; the others take host pointers, copy in
 *    and out, and synchronize before returning.
 *  - Activations are float32, row-major [rows, features].  Linear weights
 *    are [out, in] (torch nn.Linear layout) and are given in float32; a
 *    handle created with weight_dtype = CTTS_BF16 stores them as bf16
 *    (round to nearest even) and accumulates in float32.
 *  - `nth` thread-count arguments of the reference are not present: the
 *    device decides its own parallelism.
 */
#ifndef CUTETTS_B200_H
#define CUTETTS_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define CTTS_API __attribute__((visibility("default")))
#else
#define CTTS_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------- status */
#define CTTS_OK 0
#define CTTS_ERR_ARG (-1)     /* bad handle, pointer, shape or name */
#define CTTS_ERR_CUDA (-2)    /* a CUDA runtime call failed */
#define CTTS_ERR_TIMEOUT (-3) /* a bounded device-side wait gave up */
#define CTTS_ERR_STATE (-4)   /* call not valid in the handle's state */
#define CTTS_ERR_IO (-5)      /* file could not be read / parsed */
#define CTTS_ERR_NOMEM (-6)   /* device or host allocation failed */
#define CTTS_ERR_RANGE (-7)   /* index out of range (token id, cache full) */

#define CTTS_F32 0
#define CTTS_BF16 1

/* One line describing the last error on this thread ("" if none). */
CTTS_API const char* ctts_last_error(void);
/* Error-path testing of the bounded device waits.  The reference's
 * analogue is the panic -> -1 contract of rust-codec/src/ffi.rs:51-64 (no
 * direct counterpart).  While `skip` is non-zero, launches of the
 * small-batch fp32 DiT grid loop enqueued afterwards run with CTA 0 leaving
 * its QKV outputs unwritten, so the attention phase polls exchange words no
 * producer writes; every poll gives up after `spin_limit` tries (0 = the
 * default, about four million).  The kernel records the timeout and runs to
 * its end; the host call that reads the DiT error word returns
 * CTTS_ERR_TIMEOUT and clears it, and the device stays usable.
 * Process-wide, off by default; frames already captured in a CUDA graph
 * keep the setting they were captured with. */
CTTS_API int ctts_debug_inject_wait_fault(int skip, unsigned spin_limit);
/* Library version string. */
CTTS_API const char* ctts_version(void);

/* ------------------------------------------------------- LM (Qwen3 stack)
 * Replaces rust-codec/src/qwen.rs: QwenW (26-44), load_qwen_weights (75-120),
 * QwenCache (139-149), prefill (379-391), decode_step (394-406),
 * embed_lookup (409-417).  Shape-generic (qwen.rs:17-24 are constants). */
typedef struct {
  int hidden, n_layers, n_heads, n_kv_heads, head_dim, ffn, vocab;
  float rms_eps, rope_theta;
  int qk_norm;      /* 1: per-head RMSNorm of q and k before RoPE (Qwen3) */
  int weight_dtype; /* CTTS_F32 or CTTS_BF16 */
} ctts_lm_config;

typedef struct ctts_lm ctts_lm;
typedef struct ctts_kv ctts_kv;

CTTS_API int ctts_lm_create(const ctts_lm_config* cfg, int device, ctts_lm** out);
/* Upload one tensor by its checkpoint name (without the "qwen_backbone."
 * prefix), e.g. "layers.3.self_attn.q_proj.weight", "embed_tokens.weight",
 * "norm.weight".  `host` holds float32 (dtype CTTS_F32) or bf16 bit
 * patterns (CTTS_BF16) of exactly the shape the config implies. */
CTTS_API int ctts_lm_set_tensor(ctts_lm* lm, const char* name, const void* host, int dtype,
                       const int64_t* shape, int ndim);
/* load_qwen_weights (qwen.rs:75-120): read every "<prefix>..." tensor of a
 * .safetensors file (F32 or BF16). */
CTTS_API int ctts_lm_load(ctts_lm* lm, const char* safetensors_path, const char* prefix);
/* Number of tensors still missing before the model can run (0 = ready). */
CTTS_API int ctts_lm_missing(const ctts_lm* lm);
CTTS_API void ctts_lm_free(ctts_lm* lm);

/* QwenCache::empty (qwen.rs:146), batched: `batch` independent utterances,
 * each with room for `capacity` positions per layer.  K is stored post-RoPE
 * (qwen.rs:338-340) in the model's weight dtype. */
CTTS_API int ctts_kv_alloc(const ctts_lm* lm, int batch, int capacity, ctts_kv** out);
CTTS_API int ctts_kv_reset(ctts_kv* kv);                 /* every length back to 0 */
CTTS_API int ctts_kv_len(const ctts_kv* kv, int b);      /* QwenCache.len (>=0) or <0 */
CTTS_API int ctts_kv_set_len(ctts_kv* kv, int b, int len);
CTTS_API void ctts_kv_free(ctts_kv* kv);

/* prefill (qwen.rs:379-391) of utterance b: x [T, hidden] at positions
 * len..len+T-1; writes the final-normed hidden states [T, hidden]. */
CTTS_API int ctts_lm_prefill(ctts_lm* lm, ctts_kv* kv, int b, const float* x, int T, float* out);
CTTS_API int ctts_lm_prefill_dev(ctts_lm* lm, ctts_kv* kv, int b, const float* x_dev, int T,
                        float* out_dev, void* stream);
/* decode_step (qwen.rs:394-406) for all `batch` utterances at once:
 * x [batch, hidden], each at position len[b]; out [batch, hidden].
 * Lengths advance by one (host-side bookkeeping, no device sync in _dev). */
CTTS_API int ctts_lm_decode_step(ctts_lm* lm, ctts_kv* kv, const float* x, float* out);
CTTS_API int ctts_lm_decode_step_dev(ctts_lm* lm, ctts_kv* kv, const float* x_dev, float* out_dev,
                            void* stream);
/* embed_lookup (qwen.rs:409-417): ids [n] -> [n, hidden]; CTTS_ERR_RANGE on
 * an id outside [0, vocab). */
CTTS_API int ctts_lm_embed_lookup(ctts_lm* lm, const int64_t* ids, int n, float* out);

/* --------------------------------------------------------- DiT flow head
 * Replaces rust-codec/src/dit.rs: DitW/load_dit_weights (27-159), predict
 * (681-737), sample_prologue (756-772), euler_sample (819-842),
 * sway_timesteps (846-854), euler_sample_cfg (862-900); mu_proj follows
 * diffusion_head.py:421,601 (absent from the Rust port). */
typedef struct {
  int latent, hidden, n_heads, n_kv_heads, head_dim, ffn, n_layers, patch;
  int cond_dim, spk_dim;
  float rms_eps, rope_theta;
  int adaln, step_emb, cfg_emb; /* which optional modules exist */
  int weight_dtype;
} ctts_dit_config;

typedef struct ctts_dit ctts_dit;

CTTS_API int ctts_dit_create(const ctts_dit_config* cfg, int device, ctts_dit** out);
/* names without the "head." prefix, e.g. "decoder.layers.0.speaker_adaln.weight" */
CTTS_API int ctts_dit_set_tensor(ctts_dit* dit, const char* name, const void* host, int dtype,
                        const int64_t* shape, int ndim);
CTTS_API int ctts_dit_load(ctts_dit* dit, const char* safetensors_path, const char* prefix);
CTTS_API int ctts_dit_missing(const ctts_dit* dit);
CTTS_API void ctts_dit_free(ctts_dit* dit);

/* predict for `batch` utterances: x, cond [batch, patch*latent], z
 * [batch, cond_dim], spk [batch, spk_dim] or NULL, t / dt / cfg_w scalars
 * shared by the batch -> v [batch, patch*latent]. */
CTTS_API int ctts_dit_predict(ctts_dit* dit, int batch, const float* x, float t, const float* z,
                     const float* cond, float dt, const float* spk, float cfg_w, float* v);
/* euler_sample, batched: uniform grid t_s = s/steps, x += v/steps. */
CTTS_API int ctts_dit_euler_sample(ctts_dit* dit, int batch, const float* x0, const float* z,
                          const float* cond, const float* spk, int steps, float cfg_w,
                          float* x_out);
CTTS_API int ctts_dit_euler_sample_dev(ctts_dit* dit, int batch, const float* x0_dev,
                              const float* z_dev, const float* cond_dev,
                              const float* spk_dev, int steps, float cfg_w,
                              float* x_out_dev, void* stream);
/* euler_sample_cfg: sway grid (coeff), v = vc + cfg*(vc - vu), both
 * branches run as one 2*batch pass over shared weights
 * (the sgemm_bias_dual fusion, gemm.rs:299-595). */
CTTS_API int ctts_dit_euler_sample_cfg(ctts_dit* dit, int batch, const float* x0, const float* z_c,
                              const float* z_u, const float* cond, const float* uncond,
                              const float* spk, int steps, float coeff, float cfg,
                              float* x_out);
/* sway_timesteps (host arithmetic, steps+1 floats). */
CTTS_API int ctts_sway_timesteps(int steps, float coeff, float* out);

/* ---------------------------------------------------- per-frame engine
 * The AR loop body of bin/cutetts.rs:429-523 (generation.py:931-1087):
 * stop logits (e2e.rs:83-92) -> DiT Euler sample from supplied noise ->
 * latent out (pred/scale - bias) -> feedback Linear(latent->hidden)
 * (stands in for locenc_embed, locenc.rs:222-255) -> LM decode_step.
 * One frame for all utterances is one CUDA-graph replay. */
typedef struct ctts_engine ctts_engine;

typedef struct {
  int batch;         /* utterances advanced together */
  int capacity;      /* KV positions per utterance */
  int euler_steps;
  float latent_scale, latent_bias; /* scaled = raw/scale - bias */
  int use_graph;     /* 1: capture the frame step as a CUDA graph */
  int groups;        /* sub-batches run as parallel graph branches (divides batch; <=0 -> 1) */
  float cfg_strength; /* > 0: base-variant classifier-free guidance (bin/cutetts.rs:440-456,
                         503-509): a second, unconditional LM branch per utterance (its own KV
                         cache, prefilled with ctts_engine_prefill_uncond) fed the same latent,
                         and the CFG Euler sampler v = vc + s*(vc - vu) on the sway grid */
  float sway_coeff;   /* sway_timesteps coefficient of the CFG grid (dit.rs:846-854) */
} ctts_engine_config;

CTTS_API int ctts_engine_create(ctts_lm* lm, ctts_dit* dit, const ctts_engine_config* cfg,
                       ctts_engine** out);
/* Stop head and feedback projection weights (float32 host):
 * stop_w [2, hidden], stop_b [2], proj_w [hidden, latent*patch], proj_b [hidden]. */
CTTS_API int ctts_engine_set_heads(ctts_engine* e, const float* stop_w, const float* stop_b,
                          const float* proj_w, const float* proj_b);
/* Prefill utterance b with rows x [T, hidden] (text embeddings and
 * projected prompt latents) and set its first DiT cond (previous raw
 * latent patch, [patch*latent]). */
CTTS_API int ctts_engine_prefill(ctts_engine* e, int b, const float* x, int T, const float* cond0);
/* AdaLN speaker embedding of utterance b (spk [spk_dim] host floats;
 * bin/cutetts.rs passes the speaker encoder's vector to every euler_sample).
 * Required for every utterance when the DiT's spk_dim differs from the LM
 * hidden width (the shipped model: 256); otherwise the LM state conditions
 * AdaLN unless speakers are set (the first call before the first step). */
CTTS_API int ctts_engine_set_speaker(ctts_engine* e, int b, const float* spk);
/* CFG mode: prefill utterance b's unconditional branch (x [T, hidden]) and
 * its initial uncond latent condition. */
CTTS_API int ctts_engine_prefill_uncond(ctts_engine* e, int b, const float* x, int T, const float* cond0);
/* One frame for every utterance: noise [batch, patch*latent] (host) ->
 * latents_out [batch, patch*latent] (scaled), stop_out [batch, 2] or NULL. */
CTTS_API int ctts_engine_step(ctts_engine* e, const float* noise, float* latents_out, float* stop_out);
/* Device-pointer variant (noise_dev / out_dev on the engine's device). */
CTTS_API int ctts_engine_step_dev(ctts_engine* e, const float* noise_dev, float* latents_dev,
                         float* stop_dev, void* stream);
/* Kernel launches issued by one frame step (for measurement reporting). */
CTTS_API int ctts_engine_launches_per_step(const ctts_engine* e);
/* Per-frame phase timers (the --profile-steps instrument of
 * rust-codec/src/bin/cutetts.rs:328-350,466-478): while on, every frame runs
 * eagerly with CUDA events between its phases -- 0 stop head, 1 DiT sample,
 * 2 feedback projection, 3 LM step -- and the step synchronizes its stream.
 * Switching on or off clears the collected times.  Single sub-batch group
 * only (CTTS_ERR_STATE otherwise). */
CTTS_API int ctts_engine_set_profile(ctts_engine* e, int on);
/* mean, p50, p99 (ms) of one phase over the profiled frames; *n = frames. */
CTTS_API int ctts_engine_profile_stats(const ctts_engine* e, int phase, float* mean_p50_p99, int* n);
/* "name: n=N mean=Xms p50=Yms p99=Zms" per phase (profile_report,
 * bin/cutetts.rs:338-350) into buf; returns the bytes written. */
CTTS_API int ctts_engine_profile_report(const ctts_engine* e, char* buf, int len);
/* The engine's stream (cudaStream_t as void*). */
CTTS_API void* ctts_engine_stream(const ctts_engine* e);
CTTS_API void ctts_engine_free(ctts_engine* e);

/* ------------------------------------------------------ VAE decoder
 * Replaces rust-codec/src/decode.rs:decode_nth (94-136), weights.rs
 * load_decoder_weights (98-186) at generic shapes, dense (depthwise = 0,
 * audio_vae.py CausalDecoder(depthwise=False)) or the shipped depthwise
 * topology (depthwise = 1: depthwise k7 + pointwise front, depthwise
 * dilated k7 in every residual unit; decode.rs:97-128). */
typedef struct {
  int latent, channels, n_stages, depthwise;
  int strides[8];
  int weight_dtype;
} ctts_vae_config;

typedef struct ctts_vae ctts_vae;

CTTS_API int ctts_vae_create(const ctts_vae_config* cfg, int device, ctts_vae** out);
/* names without "decoder." prefix, fused weights ("model.0.weight") or the
 * weight-norm pair ("...weight_g" + "...weight_v", fused when both are set,
 * conv.rs:12-30). */
CTTS_API int ctts_vae_set_tensor(ctts_vae* v, const char* name, const void* host, int dtype,
                        const int64_t* shape, int ndim);
CTTS_API int ctts_vae_load_file(ctts_vae* v, const char* safetensors_path, const char* prefix);
CTTS_API int ctts_vae_missing(const ctts_vae* v);
CTTS_API void ctts_vae_free(ctts_vae* v);
/* latent [batch, latent, T] -> wav [batch, T*hop] */
CTTS_API int ctts_vae_decode_batch(ctts_vae* v, int batch, const float* latent, int T, float* wav);
CTTS_API int ctts_vae_decode_batch_dev(ctts_vae* v, int batch, const float* latent_dev, int T,
                              float* wav_dev, void* stream);

/* Streaming decoder (replaces rust-codec/src/stream.rs:62 StreamingDecoder::new,
 * :82 reset, :96 decode_chunk): per-conv left histories carried across
 * chunks, so decoding an utterance chunk by chunk gives exactly the samples
 * of the offline decode.  latent [batch, latent, frames] -> wav
 * [batch, frames*hop]; histories start (and reset) at zero. */
typedef struct ctts_vae_stream ctts_vae_stream;
CTTS_API int ctts_vae_stream_create(ctts_vae* v, int batch, ctts_vae_stream** out);
CTTS_API int ctts_vae_stream_reset(ctts_vae_stream* s);
CTTS_API int ctts_vae_stream_decode_chunk(ctts_vae_stream* s, const float* latent, int frames, float* wav);
CTTS_API int ctts_vae_stream_decode_chunk_dev(ctts_vae_stream* s, const float* latent_dev, int frames,
                              float* wav_dev, void* stream);
CTTS_API void ctts_vae_stream_free(ctts_vae_stream* s);

/* ------------------------------------------------------- LocEnc feedback
 * AudioLocEnc + locenc_to_lm_proj (replaces rust-codec/src/locenc.rs:222
 * locenc_embed and load_locenc_weights :88; diffusion_head.py:334-378,
 * model.py:128-130): x [n, patch, latent] (n items = utterance-steps) ->
 * LM input rows [n, out_dim].  Tensor names are the module's own
 * (special_token, in_proj.*, encoder.layers.{i}.*, encoder.norm.weight)
 * plus locenc_to_lm_proj.*; ctts_locenc_load reads a full checkpoint with
 * prefix "locenc.". */
typedef struct {
  int latent, hidden, n_heads, n_kv_heads, head_dim, ffn, n_layers, patch, out_dim;
  float rms_eps, rope_theta;
  int weight_dtype;
} ctts_locenc_config;
typedef struct ctts_locenc ctts_locenc;
CTTS_API int ctts_locenc_create(const ctts_locenc_config* cfg, int device, ctts_locenc** out);
CTTS_API int ctts_locenc_set_tensor(ctts_locenc* l, const char* name, const void* host, int dtype,
                           const int64_t* shape, int ndim);
CTTS_API int ctts_locenc_load(ctts_locenc* l, const char* safetensors_path, const char* prefix);
CTTS_API int ctts_locenc_missing(const ctts_locenc* l);
CTTS_API void ctts_locenc_free(ctts_locenc* l);
CTTS_API int ctts_locenc_embed(ctts_locenc* l, const float* x, int n, float* out);
CTTS_API int ctts_locenc_embed_dev(ctts_locenc* l, const float* x_dev, int n, float* out_dev, void* stream);

/* Exact signatures of rust-codec/src/ffi.rs:19-65 (used by
 * src/cutetts/modeling/rust_vae.py through ctypes).  The handle decodes
 * the shipped topology read from the file (latent 64, rates read from the
 * tensors' shapes).  wav_out holds frames*hop floats; 0 ok, -1 error. */
CTTS_API void* cutetts_vae_load(const char* safetensors_path);
CTTS_API void cutetts_vae_free(void* handle);
CTTS_API int cutetts_vae_decode(void* handle, const float* latent64xT, unsigned long frames,
                       float* wav_out);

/* ------------------------------------------------- op-level entry points
 * The fused layer kernels on their own (BASELINE op sweep).  All device
 * pointers, asynchronous on `stream`. */
/* y[M,N] = RMSNorm(x[M,K]; norm_w, eps) . W[N,K]^T (+ res[M,N]).
 * norm_w NULL: no norm.  w_dtype CTTS_F32 (float*) or CTTS_BF16 (uint16
 * bf16 bits). */
CTTS_API int ctts_op_linear(const float* x, int M, int K, const void* w, int w_dtype, int N,
                   const float* norm_w, float eps, const float* res, float* y, void* stream);
/* ctts_op_linear without any device allocation.  No counterpart in the
 * reference (whose CPU kernels allocate host vectors freely): for callers
 * that cannot call cudaMalloc -- a process whose device heap is owned by
 * its own pool, or a serving loop that must not allocate after set-up
 * because it cannot afford cudaMalloc's implicit device-wide
 * synchronization.  Same arguments and results as ctts_op_linear.
 * The bf16 tensor-core path (w_dtype CTTS_BF16, M >= 16, K % 64 == 0) keeps
 * its bf16 activation operand in a static device array of 2^20 elements
 * (2 MiB, held by every GPU that loads this library until exit) instead of
 * an allocated buffer; M*K above 2^20 returns CTTS_ERR_RANGE.  The first call
 * on a device looks the array's device address up (cudaGetSymbolAddress),
 * so make it before any stream capture.  All calls share the array: calls
 * that overlap on the GPU (different streams, or threads on one device)
 * race on it, so serialize them.  Asynchronous like ctts_op_linear: a
 * bounded device-side wait that gives up ends the kernel early without a
 * hang but is not reported in the return code. */
CTTS_API int ctts_op_linear_noalloc(const float* x, int M, int K, const void* w, int w_dtype, int N,
                                    const float* norm_w, float eps, const float* res, float* y,
                                    void* stream);
/* NeoX RoPE in place on x [M, heads, head_dim] at positions pos[M]. */
CTTS_API int ctts_op_rope(float* x, int M, int heads, int head_dim, const int* pos, float theta,
                 void* stream);
/* out[M,F] = silu(gu[M, 0:F]) * gu[M, F:2F] */
CTTS_API int ctts_op_swiglu(const float* gu, int M, int F, float* out, void* stream);
/* Causal Conv1d, stride 1 (rust-codec/src/conv.rs:36-51 causal_conv1d):
 * x [batch, c_in, T] -> y [batch, c_out, T], w [c_out, c_in/groups, k]
 * (weight norm already fused), bias [c_out] or NULL, left pad 2*pad
 * (the module's padding argument, audio_vae.py CausalConv1d).  groups is 1
 * (dense) or c_in == c_out (depthwise); other groupings return CTTS_ERR_ARG. */
CTTS_API int ctts_op_causal_conv1d(const float* x, int batch, int c_in, int T, const void* w, int w_dtype,
                                   const float* bias, int c_out, int k, int dilation, int groups, int pad,
                                   float* y, void* stream);
/* out[n, H] = table[ids[n], :]; ids validated on device, *bad_count (device
 * int, may be NULL) receives the number of out-of-range ids (rows zeroed). */
CTTS_API int ctts_op_embed_gather(const float* table, int vocab, int H, const int64_t* ids, int n,
                         float* out, int* bad_count, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* CUTETTS_B200_H */
