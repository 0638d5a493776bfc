// model.h -- the objects behind the C ABI handles.
#pragma once

#include <algorithm>
#include <vector>

#include "api_common.h"
#include "dit_cluster.cuh"
#include "dit_grid.cuh"
#include "lm_grid.cuh"

// LM stack (replaces QwenW, qwen.rs:26-44).  Weights of a layer are fused
// into wide matrices at load: [q;k;v] -> wqkv, [gate;up] -> wgu, so one
// pass over the activations feeds all of them.
struct LMLayer {
  float *norm1 = nullptr, *norm2 = nullptr, *qn = nullptr, *kn = nullptr;
  void *wqkv = nullptr, *wo = nullptr, *wgu = nullptr, *wd = nullptr;
};

struct ctts_lm {
  ctts_lm_config cfg{};
  int device = 0;
  int bf16 = 0;
  cudaStream_t stream = nullptr;
  ctts::DevArena arena;
  ctts::SlotTable slots;
  void* embed = nullptr;
  std::vector<LMLayer> layers;
  float* final_norm = nullptr;
  float* inv_freq = nullptr;
};

// Batched KV cache (replaces QwenCache, qwen.rs:139-149) plus the decode /
// prefill workspace sized for this batch.  Layout per layer:
// [batch][kv_head][capacity][head_dim] in the model weight dtype.
struct ctts_kv {
  const ctts_lm* lm = nullptr;
  int batch = 0, cap = 0, nsplit = 0, chunk = 128, ws_rows = 0;
  int* cnt = nullptr;  // decode-attention split tickets [batch][n_kv_heads]
  unsigned* gbar = nullptr;  // grid-persistent decode step barrier counters (zero at rest)
  float* gpart = nullptr;    // its attention partials
  float* ssp = nullptr;  // residual-row sum-of-squares partials [hidden/128][ws_rows]
  size_t layer_elems = 0;
  ctts::DevArena arena;
  void *k = nullptr, *v = nullptr;
  int* pos = nullptr;  // device positions (= cache lengths)
  int* err = nullptr;
  std::vector<int> pos_host;
  float *h = nullptr, *qkv = nullptr, *qrot = nullptr, *att = nullptr, *act = nullptr,
        *part = nullptr, *xin = nullptr, *xout = nullptr;
  // tensor-core path (bf16 models, >= 16 rows): bf16 operands + split-K scratch
  uint16_t *xb = nullptr, *attb = nullptr, *actb = nullptr;
  ctts::TcScratch tc;
};

// DiT head (replaces DitW, dit.rs:27-68).
struct DitLayer {
  float *norm1 = nullptr, *norm2 = nullptr;
  void *wqkv = nullptr, *wo = nullptr, *wgu = nullptr, *wd = nullptr;
};

struct DitWs {  // workspace for `rows` utterance-branches
  int rows = 0, steps = 0;
  ctts::DevArena arena;
  float *seq = nullptr, *qkv = nullptr, *att = nullptr, *act = nullptr, *mu = nullptr,
        *ad = nullptr, *condh = nullptr, *temb = nullptr, *dtemb = nullptr, *tmp = nullptr,
        *se = nullptr, *tv = nullptr, *x = nullptr, *v = nullptr, *z = nullptr,
        *cond = nullptr, *spk = nullptr, *hbuf = nullptr, *stemb = nullptr;
  uint16_t *xb = nullptr, *attb = nullptr, *actb = nullptr;
  ctts::TcScratch tc;
  int* err = nullptr;
  unsigned* gbar = nullptr;  // grid-persistent Euler loop: launch generation, exit count
  unsigned long long* gll = nullptr;  // its flag-tagged exchange words (zero at allocation)
};

struct ctts_dit {
  ctts_dit_config cfg{};
  int device = 0;
  int bf16 = 0;
  cudaStream_t stream = nullptr;
  ctts::DevArena arena;
  ctts::SlotTable slots;
  void *in_w = nullptr, *cond_w = nullptr, *mu_w = nullptr, *out_w = nullptr;
  void *t1_w = nullptr, *t2_w = nullptr, *dt1_w = nullptr, *dt2_w = nullptr;
  void *st1_w = nullptr, *st2_w = nullptr;
  float *in_b = nullptr, *cond_b = nullptr, *mu_b = nullptr, *out_b = nullptr;
  float *t1_b = nullptr, *t2_b = nullptr, *dt1_b = nullptr, *dt2_b = nullptr;
  float *st1_b = nullptr, *st2_b = nullptr;
  float* cfg0_w = nullptr;  // [H,1] float32 (applied on the host: scalar input)
  void* cfg2_w = nullptr;
  void* adaln = nullptr;  // [n_layers*6H, spk_dim]
  std::vector<DitLayer> layers;
  float* final_norm = nullptr;
  float* inv_freq = nullptr;
  DitWs ws;
  // cluster-resident Euler loop (dit_cluster.cu): packed weights, state
  // 0 = not tried, 1 = ready, -1 = shapes/device unsupported, disabled, or
  // off after a split-K partial left the fp16 exchange range; dirty = a
  // tensor was uploaded since the weights were packed
  ctts::DitClusterW* cl = nullptr;
  int cl_state = 0;
  bool cl_dirty = false;
};

struct EngineGroup {
  int b0 = 0, nb = 0;          // utterances [b0, b0 + nb)
  ctts_kv* kv = nullptr;       // their KV cache + LM workspace
  DitWs* ws = nullptr;         // their DiT workspace (owned)
  cudaStream_t stream = nullptr;
  cudaEvent_t done = nullptr;
  // side branch of a frame: the stop head, concurrent with the DiT
  cudaStream_t side = nullptr;
  cudaEvent_t side_fork = nullptr, side_join = nullptr;
};

struct ctts_engine {
  ctts_lm* lm = nullptr;
  ctts_dit* dit = nullptr;
  ctts_kv* kv = nullptr;  // groups[0].kv
  std::vector<EngineGroup> groups;
  cudaEvent_t fork = nullptr;
  ctts_engine_config cfg{};
  cudaStream_t stream = nullptr;
  ctts::DevArena arena;
  float *stop_w = nullptr, *stop_b = nullptr, *proj_w = nullptr, *proj_b = nullptr;
  float *z = nullptr, *x = nullptr, *cond = nullptr, *lat = nullptr, *stop = nullptr,
        *fb = nullptr, *noise = nullptr;
  float *h_noise = nullptr, *h_lat = nullptr, *h_stop = nullptr;  // pinned staging
  int* h_err = nullptr;  // pinned: each group's KV and DiT error words, read with the latents
  bool heads_set = false;
  bool cfg_on = false;  // classifier-free guidance: per-group rows [cond B | uncond B]
  std::vector<bool> prefilled, prefilled_u;
  // AdaLN conditioning: the LM state z (spk_dim == LM hidden, the benchmark
  // model) or a per-utterance speaker embedding set by ctts_engine_set_speaker
  // (required when spk_dim differs, the shipped model's 256-wide speaker
  // vector); rows laid out like z
  float* spk = nullptr;
  bool use_spk = false;
  std::vector<bool> spk_set;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  int steps_done = 0;
  int launches = 0;
  // per-phase timers (ctts_engine_set_profile): frames run eagerly with CUDA
  // events between the phases; per-frame device milliseconds per phase
  static constexpr int kPhases = 4;  // stop head, DiT sample, feedback, LM step
  bool profile = false;
  cudaEvent_t pev[kPhases + 1] = {};
  std::vector<float> ptimes[kPhases];
};

// VAE decoder (replaces DecoderW, weights.rs:34-44).
struct VaeRes {
  float *a0 = nullptr, *b0 = nullptr, *a1 = nullptr, *b1 = nullptr;
  void *w0 = nullptr, *w1 = nullptr;
  void *w0_tc = nullptr, *w1_tc = nullptr;  // bf16 tensor-core layout (repack_conv_tc) or null
};
struct VaeStage {
  int cin = 0, cout = 0, stride = 0;
  float *alpha = nullptr, *tb = nullptr;
  void* tw = nullptr;  // repacked [stride][cout][cin*2]
  void* tw_tc = nullptr;
  VaeRes res[3];
};
struct ctts_vae {
  ctts_vae_config cfg{};
  int device = 0;
  int bf16 = 0;
  cudaStream_t stream = nullptr;
  ctts::DevArena arena;
  ctts::SlotTable slots;
  void *front_w = nullptr, *front_pw_w = nullptr;
  float *front_b = nullptr, *front_pw_b = nullptr;
  std::vector<VaeStage> stages;
  float *final_alpha = nullptr, *final_b = nullptr;
  void* final_w = nullptr;
  int hop = 1;
  // bf16 weights of the dense convs in the tensor-core layout, rebuilt from
  // the uploaded weights before the first decode after any upload
  void *front_tc = nullptr, *front_pw_tc = nullptr;
  bool tc_dirty = true;
  ctts::DevArena tc_arena;
  int* err = nullptr;  // device error word of the tensor-core convs
  // workspace
  size_t ws_elems = 0;
  float *buf[3] = {nullptr, nullptr, nullptr};
  ctts::DevArena ws_arena;
  float *lat_dev = nullptr, *wav_dev = nullptr;
  size_t io_lat = 0, io_wav = 0;
};

namespace ctts {
int lm_forward_rows(ctts_lm* lm, ctts_kv* kv, int rows, int prefill_b, int pos0, float* out,
                    cudaStream_t s, int* launches);
int lm_check_ready(const ctts_lm* lm);
int lm_decode_dev(ctts_lm* lm, ctts_kv* kv, const float* x_dev, float* out_dev, cudaStream_t s,
                  int* launches);
// VAE tensor-core convs (api_vae.cu): rebuild the repacked bf16 weights
// after an upload, point a conv at them, read back the error word.
struct ConvArgs;
int vae_tc_prepare(ctts_vae* v);
void use_tc(const ctts_vae* v, ConvArgs& a, const void* w_tc);
int vae_read_err(ctts_vae* v);
}  // namespace ctts
