// api_locenc.cu -- C ABI: the LocEnc latent-feedback encoder
// (rust-codec/src/locenc.rs:147-255 loc_layer / locenc_embed;
// src/cutetts/modeling/diffusion_head.py:334-378 AudioLocEnc and
// model.py:128-130 embed_acoustic_latents = locenc_to_lm_proj(locenc(x))).
//
// Per item (one AR step of one utterance): the sequence [CLS, patch frames]
// (CLS = the learned special token, frames = in_proj of the latents) runs
// through plain LocalTransformer layers (RMSNorm -> q/k/v -> RoPE at
// positions 0..P -> bidirectional GQA attention -> o-proj + residual;
// RMSNorm -> SwiGLU -> down + residual), then the final RMSNorm of the CLS
// row and locenc_to_lm_proj.  The layers run on the DiT head's kernels
// (skinny linears with the norm fused into the operand load, the
// short-sequence RoPE attention); the final norm is fused into the
// projection's operand load and reads the CLS rows in place.
#include <string>
#include <vector>

#include "api_common.h"
#include "common.cuh"
#include "model.h"

using namespace ctts;

struct ctts_locenc {
  ctts_locenc_config cfg{};
  int device = 0;
  int bf16 = 0;
  cudaStream_t stream = nullptr;
  DevArena arena;
  SlotTable slots;
  void *in_w = nullptr, *proj_w = nullptr;
  float *in_b = nullptr, *proj_b = nullptr, *special = nullptr, *final_norm = nullptr, *inv_freq = nullptr;
  std::vector<DitLayer> layers;
  // workspace for `rows` items
  int ws_items = 0;
  DevArena ws;
  float *seq = nullptr, *qkv = nullptr, *att = nullptr, *act = nullptr, *x_dev = nullptr, *out_dev = nullptr;
};

namespace {

__global__ void cls_rows_kernel(float* seq, const float* special, int H, int S) {
  grid_dep_enter();
  float* row = seq + (size_t)blockIdx.x * S * H;
  for (int i = threadIdx.x; i < H; i += blockDim.x) row[i] = special[i];
}

int ws_ensure(ctts_locenc* l, int n) {
  if (n <= l->ws_items) return CTTS_OK;
  const ctts_locenc_config& c = l->cfg;
  const int S = 1 + c.patch, H = c.hidden;
  const int qkvw = (c.n_heads + 2 * c.n_kv_heads) * c.head_dim, qd = c.n_heads * c.head_dim;
  cudaDeviceSynchronize();
  l->ws.~DevArena();
  new (&l->ws) DevArena();
  const size_t rows = (size_t)n * S;
  l->seq = l->ws.alloc<float>(rows * H);
  l->qkv = l->ws.alloc<float>(rows * qkvw);
  l->att = l->ws.alloc<float>(rows * qd);
  l->act = l->ws.alloc<float>(rows * c.ffn);
  l->x_dev = l->ws.alloc<float>((size_t)n * c.patch * c.latent);
  l->out_dev = l->ws.alloc<float>((size_t)n * c.out_dim);
  if (!l->seq || !l->qkv || !l->att || !l->act || !l->x_dev || !l->out_dev) {
    l->ws_items = 0;
    return set_error(CTTS_ERR_NOMEM, "LocEnc workspace");
  }
  l->ws_items = n;
  return CTTS_OK;
}

int enqueue(ctts_locenc* l, const float* x, int n, float* out, cudaStream_t s) {
  const ctts_locenc_config& c = l->cfg;
  const int P = c.patch, S = 1 + P, H = c.hidden, F = c.ffn, hd = c.head_dim;
  const int qd = c.n_heads * hd, qkvw = qd + 2 * c.n_kv_heads * hd, R = n * S;
  auto lin = [&](LinearArgs a) -> int {
    a.w_bf16 = l->bf16;
    cudaError_t e = launch_linear(a, s);
    if (e != cudaSuccess) {
      (void)cudaGetLastError();
      return set_error(CTTS_ERR_CUDA, std::string("linear: ") + cudaGetErrorString(e));
    }
    return CTTS_OK;
  };
  int rc;
  // [CLS, in_proj(frames)] per item (locenc.rs:222-240)
  CTTS_CK(launch_k(cls_rows_kernel, dim3(n), dim3(128), 0, s, l->seq, (const float*)l->special, H, S));
  {
    LinearArgs a; a.x = x; a.x_ld = c.latent; a.M = n * P; a.K = c.latent; a.N = H; a.w = l->in_w;
    a.bias = l->in_b; a.y = l->seq + H; a.y_ld = H; a.y_div = P; a.y_ld_outer = (long)S * H;
    if ((rc = lin(a))) return rc;
  }
  for (const DitLayer& Ly : l->layers) {  // loc_layer (locenc.rs:147-219)
    LinearArgs q; q.x = l->seq; q.x_ld = H; q.M = R; q.K = H; q.N = qkvw; q.w = Ly.wqkv;
    q.y = l->qkv; q.y_ld = qkvw; q.norm_w = Ly.norm1; q.eps = c.rms_eps;
    if ((rc = lin(q))) return rc;
    CTTS_CK(launch_dit_attn(l->qkv, n, S, c.n_heads, c.n_kv_heads, hd, l->inv_freq, l->att, nullptr, s));
    LinearArgs o; o.x = l->att; o.x_ld = qd; o.M = R; o.K = qd; o.N = H; o.w = Ly.wo;
    o.y = l->seq; o.y_ld = H; o.res = l->seq;
    if ((rc = lin(o))) return rc;
    LinearArgs g; g.x = l->seq; g.x_ld = H; g.M = R; g.K = H; g.N = F; g.w = Ly.wgu;
    g.y = l->act; g.y_ld = F; g.act = 2; g.norm_w = Ly.norm2; g.eps = c.rms_eps;
    if ((rc = lin(g))) return rc;
    LinearArgs dn; dn.x = l->act; dn.x_ld = F; dn.M = R; dn.K = F; dn.N = H; dn.w = Ly.wd;
    dn.y = l->seq; dn.y_ld = H; dn.res = l->seq;
    if ((rc = lin(dn))) return rc;
  }
  // final norm of the CLS rows fused into locenc_to_lm_proj (model.py:128-130)
  LinearArgs p; p.x = l->seq; p.x_ld = (long)S * H; p.M = n; p.K = H; p.N = c.out_dim; p.w = l->proj_w;
  p.bias = l->proj_b; p.y = out; p.y_ld = c.out_dim; p.norm_w = l->final_norm; p.eps = c.rms_eps;
  return lin(p);
}

}  // namespace

extern "C" int ctts_locenc_create(const ctts_locenc_config* cfg, int device, ctts_locenc** out) {
  CTTS_REQ(cfg && out, CTTS_ERR_ARG, "null argument");
  const ctts_locenc_config& c = *cfg;
  CTTS_REQ(c.latent > 0 && c.hidden > 0 && c.n_heads > 0 && c.n_kv_heads > 0 && c.head_dim > 0 && c.ffn > 0 &&
               c.n_layers > 0 && c.patch > 0 && c.out_dim > 0,
           CTTS_ERR_ARG, "non-positive dimension");
  CTTS_REQ(1 + c.patch <= 5, CTTS_ERR_ARG, "patch must be 1..4");
  CTTS_REQ(c.n_heads % c.n_kv_heads == 0, CTTS_ERR_ARG, "n_heads % n_kv_heads != 0");
  CTTS_REQ(c.head_dim % 64 == 0 && c.head_dim <= 128, CTTS_ERR_ARG, "head_dim must be 64 or 128");
  CTTS_REQ(c.hidden % 64 == 0 && c.ffn % 64 == 0 && c.latent % 8 == 0 && c.out_dim % 8 == 0, CTTS_ERR_ARG,
           "hidden/ffn must be multiples of 64, latent/out_dim of 8");
  CTTS_REQ(c.weight_dtype == CTTS_F32 || c.weight_dtype == CTTS_BF16, CTTS_ERR_ARG, "bad weight dtype");
  CTTS_CK(cudaSetDevice(device));
  auto* l = new ctts_locenc();
  l->cfg = c;
  l->device = device;
  l->bf16 = c.weight_dtype == CTTS_BF16;
  l->slots.model_bf16 = l->bf16;
  cudaStreamCreateWithFlags(&l->stream, cudaStreamNonBlocking);
  const int H = c.hidden, F = c.ffn, hd = c.head_dim, qd = c.n_heads * hd, kvd = c.n_kv_heads * hd;
  const size_t es = l->bf16 ? 2 : 4;
  DevArena& A = l->arena;
  auto W = [&](size_t n) -> void* { return A.alloc<uint8_t>(n * es); };
  l->in_w = W((size_t)H * c.latent);
  l->in_b = A.alloc<float>(H);
  l->slots.add("in_proj.weight", l->in_w, {H, c.latent}, true);
  l->slots.add("in_proj.bias", l->in_b, {H}, false);
  l->special = A.alloc<float>(H);
  l->slots.add("special_token", l->special, {1, 1, 1, H}, false);
  l->layers.resize(c.n_layers);
  for (int i = 0; i < c.n_layers; i++) {
    DitLayer& Ly = l->layers[i];
    const std::string p = "encoder.layers." + std::to_string(i) + ".";
    Ly.norm1 = A.alloc<float>(H);
    Ly.norm2 = A.alloc<float>(H);
    Ly.wqkv = W((size_t)(qd + 2 * kvd) * H);
    Ly.wo = W((size_t)H * qd);
    Ly.wgu = W((size_t)2 * F * H);
    Ly.wd = W((size_t)H * F);
    char* qkv = reinterpret_cast<char*>(Ly.wqkv);
    char* gu = reinterpret_cast<char*>(Ly.wgu);
    l->slots.add(p + "input_layernorm.weight", Ly.norm1, {H}, false);
    l->slots.add(p + "post_attention_layernorm.weight", Ly.norm2, {H}, false);
    l->slots.add(p + "self_attn.q_proj.weight", qkv, {qd, H}, true);
    l->slots.add(p + "self_attn.k_proj.weight", qkv + (size_t)qd * H * es, {kvd, H}, true);
    l->slots.add(p + "self_attn.v_proj.weight", qkv + (size_t)(qd + kvd) * H * es, {kvd, H}, true);
    l->slots.add(p + "self_attn.o_proj.weight", Ly.wo, {H, qd}, true);
    l->slots.add(p + "mlp.gate_proj.weight", gu, {F, H}, true);
    l->slots.add(p + "mlp.up_proj.weight", gu + (size_t)64 * H * es, {F, H}, true);
    for (const char* nm : {"mlp.gate_proj.weight", "mlp.up_proj.weight"}) {
      Slot& sl = l->slots.slots[p + nm];
      sl.transform = kXformRowInterleave;  // 64-row gate/up tiles (SwiGLU epilogue)
      sl.t_b = H;
    }
    l->slots.add(p + "mlp.down_proj.weight", Ly.wd, {H, F}, true);
  }
  l->final_norm = A.alloc<float>(H);
  l->slots.add("encoder.norm.weight", l->final_norm, {H}, false);
  l->proj_w = W((size_t)c.out_dim * H);
  l->proj_b = A.alloc<float>(c.out_dim);
  l->slots.add("locenc_to_lm_proj.weight", l->proj_w, {c.out_dim, H}, true);
  l->slots.add("locenc_to_lm_proj.bias", l->proj_b, {c.out_dim}, false);
  std::vector<float> inv = rope_inv_freq(hd, c.rope_theta);
  l->inv_freq = A.alloc<float>(hd / 2);
  if (!l->final_norm || !l->inv_freq || !l->proj_b ||
      cudaMemcpy(l->inv_freq, inv.data(), inv.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess) {
    delete l;
    return set_error(CTTS_ERR_NOMEM, "device allocation failed");
  }
  *out = l;
  return CTTS_OK;
}

extern "C" int ctts_locenc_set_tensor(ctts_locenc* l, const char* name, const void* host, int dtype,
                                      const int64_t* shape, int ndim) {
  CTTS_REQ(l, CTTS_ERR_ARG, "null handle");
  CTTS_CK(cudaSetDevice(l->device));
  return slot_set(l->slots, name, host, dtype, shape, ndim);
}

extern "C" int ctts_locenc_load(ctts_locenc* l, const char* path, const char* prefix) {
  CTTS_REQ(l, CTTS_ERR_ARG, "null handle");
  auto set = [&](const char* n, const void* p, int dt, const int64_t* s, int nd) {
    return ctts_locenc_set_tensor(l, n, p, dt, s, nd);
  };
  int rc = load_safetensors(path, prefix, set);
  if (rc) return rc;
  // locenc_to_lm_proj sits beside the encoder's module in a full checkpoint
  if (!l->slots.slots["locenc_to_lm_proj.weight"].set) {
    rc = load_safetensors(path, "", set);
    if (rc && rc != CTTS_ERR_IO) return rc;
  }
  return CTTS_OK;
}

extern "C" int ctts_locenc_missing(const ctts_locenc* l) { return l ? l->slots.missing() : -1; }

extern "C" void ctts_locenc_free(ctts_locenc* l) {
  if (!l) return;
  cudaSetDevice(l->device);
  cudaDeviceSynchronize();
  if (l->stream) cudaStreamDestroy(l->stream);
  delete l;
}

extern "C" int ctts_locenc_embed_dev(ctts_locenc* l, const float* x_dev, int n, float* out_dev, void* stream) {
  CTTS_REQ(l && x_dev && out_dev && n > 0, CTTS_ERR_ARG, "bad argument");
  if (l->slots.missing()) return set_error(CTTS_ERR_STATE, "LocEnc weights missing: " + l->slots.first_missing());
  CTTS_CK(cudaSetDevice(l->device));
  int rc = ws_ensure(l, n);
  if (rc) return rc;
  return enqueue(l, x_dev, n, out_dev, as_stream(stream, l->stream));
}

extern "C" int ctts_locenc_embed(ctts_locenc* l, const float* x, int n, float* out) {
  CTTS_REQ(l && x && out && n > 0, CTTS_ERR_ARG, "bad argument");
  if (l->slots.missing()) return set_error(CTTS_ERR_STATE, "LocEnc weights missing: " + l->slots.first_missing());
  CTTS_CK(cudaSetDevice(l->device));
  int rc = ws_ensure(l, n);
  if (rc) return rc;
  const ctts_locenc_config& c = l->cfg;
  CTTS_CK(cudaMemcpyAsync(l->x_dev, x, sizeof(float) * n * c.patch * c.latent, cudaMemcpyHostToDevice, l->stream));
  rc = enqueue(l, l->x_dev, n, l->out_dev, l->stream);
  if (rc) return rc;
  CTTS_CK(cudaMemcpyAsync(out, l->out_dev, sizeof(float) * n * c.out_dim, cudaMemcpyDeviceToHost, l->stream));
  CTTS_CK(cudaStreamSynchronize(l->stream));
  return CTTS_OK;
}
