// api_lm.cu -- C ABI: errors, the LM stack (qwen.rs), its KV cache and the
// op-level entry points.
#include <cstdio>

#include "api_common.h"
#include "model.h"

namespace ctts {

static thread_local std::string g_err;

int set_error(int code, const std::string& msg) {
  g_err = msg;
  return code;
}

std::string shape_str(const std::vector<int64_t>& s) {
  std::string r = "[";
  for (size_t i = 0; i < s.size(); i++) r += (i ? "," : "") + std::to_string(s[i]);
  return r + "]";
}

int slot_set(SlotTable& t, const char* name, const void* host, int dtype, const int64_t* shape,
             int ndim) {
  CTTS_REQ(name && host && (ndim == 0 || shape), CTTS_ERR_ARG, "null argument");
  CTTS_REQ(dtype == CTTS_F32 || dtype == CTTS_BF16, CTTS_ERR_ARG, "bad dtype");
  auto it = t.slots.find(name);
  CTTS_REQ(it != t.slots.end(), CTTS_ERR_ARG, std::string("unknown tensor ") + name);
  Slot& s = it->second;
  std::vector<int64_t> got(shape, shape + ndim);
  CTTS_REQ(got == s.shape, CTTS_ERR_ARG,
           std::string("shape for ") + name + ": got " + shape_str(got) + ", want " + shape_str(s.shape));
  size_t n = shape_numel(got);
  std::vector<float> f;
  host_to_f32(host, dtype, n, &f);
  int rc = upload_f32(s, f.data(), n, t.model_bf16);
  if (rc == CTTS_OK) s.set = true;
  return rc;
}

}  // namespace ctts

using namespace ctts;

extern "C" const char* ctts_last_error(void) { return g_err.c_str(); }
extern "C" const char* ctts_version(void) { return "cutetts_b200 0.1 (sm_100a)"; }

// ---------------------------------------------------------------------- LM

extern "C" int ctts_lm_create(const ctts_lm_config* cfg, int device, ctts_lm** out) {
  CTTS_REQ(cfg && out, CTTS_ERR_ARG, "null argument");
  const ctts_lm_config& c = *cfg;
  CTTS_REQ(c.hidden > 0 && c.n_layers > 0 && c.n_heads > 0 && c.n_kv_heads > 0 && c.head_dim > 0 &&
               c.ffn > 0 && c.vocab > 0,
           CTTS_ERR_ARG, "non-positive dimension");
  CTTS_REQ(c.n_heads % c.n_kv_heads == 0 && c.n_heads / c.n_kv_heads <= 8, CTTS_ERR_ARG,
           "n_heads must be a multiple of n_kv_heads (group <= 8)");
  CTTS_REQ(c.head_dim % 64 == 0 && c.head_dim <= 128, CTTS_ERR_ARG, "head_dim must be 64 or 128");
  CTTS_REQ(c.hidden % 64 == 0 && c.ffn % 64 == 0, CTTS_ERR_ARG, "hidden and ffn must be multiples of 64");
  CTTS_REQ(c.weight_dtype == CTTS_F32 || c.weight_dtype == CTTS_BF16, CTTS_ERR_ARG, "bad weight dtype");
  CTTS_CK(cudaSetDevice(device));
  auto* lm = new ctts_lm();
  lm->cfg = c;
  lm->device = device;
  lm->bf16 = c.weight_dtype == CTTS_BF16;
  lm->slots.model_bf16 = lm->bf16;
  if (cudaStreamCreateWithFlags(&lm->stream, cudaStreamNonBlocking) != cudaSuccess) {
    delete lm;
    return set_error(CTTS_ERR_CUDA, "stream create failed");
  }
  const int H = c.hidden, hd = c.head_dim, qd = c.n_heads * hd, kvd = c.n_kv_heads * hd, F = c.ffn;
  const int qkvw = qd + 2 * kvd;
  const size_t es = lm->bf16 ? 2 : 4;
  auto W = [&](size_t n) -> void* { return lm->arena.alloc<uint8_t>(n * es); };
  lm->embed = W((size_t)c.vocab * H);
  lm->slots.add("embed_tokens.weight", lm->embed, {c.vocab, H}, true, /*optional=*/true);
  lm->final_norm = lm->arena.alloc<float>(H);
  lm->slots.add("norm.weight", lm->final_norm, {H}, false);
  lm->layers.resize(c.n_layers);
  for (int i = 0; i < c.n_layers; i++) {
    LMLayer& L = lm->layers[i];
    std::string p = "layers." + std::to_string(i) + ".";
    L.norm1 = lm->arena.alloc<float>(H);
    L.norm2 = lm->arena.alloc<float>(H);
    L.qn = lm->arena.alloc<float>(hd);
    L.kn = lm->arena.alloc<float>(hd);
    L.wqkv = W((size_t)qkvw * H);
    L.wo = W((size_t)H * qd);
    L.wgu = W((size_t)2 * F * H);
    L.wd = W((size_t)H * F);
    char* qkv = reinterpret_cast<char*>(L.wqkv);
    char* gu = reinterpret_cast<char*>(L.wgu);
    lm->slots.add(p + "input_layernorm.weight", L.norm1, {H}, false);
    lm->slots.add(p + "post_attention_layernorm.weight", L.norm2, {H}, false);
    lm->slots.add(p + "self_attn.q_norm.weight", L.qn, {hd}, false, !c.qk_norm);
    lm->slots.add(p + "self_attn.k_norm.weight", L.kn, {hd}, false, !c.qk_norm);
    lm->slots.add(p + "self_attn.q_proj.weight", qkv, {qd, H}, true);
    lm->slots.add(p + "self_attn.k_proj.weight", qkv + (size_t)qd * H * es, {kvd, H}, true);
    lm->slots.add(p + "self_attn.v_proj.weight", qkv + (size_t)(qd + kvd) * H * es, {kvd, H}, true);
    lm->slots.add(p + "self_attn.o_proj.weight", L.wo, {H, qd}, true);
    lm->slots.add(p + "mlp.gate_proj.weight", gu, {F, H}, true);
    lm->slots.add(p + "mlp.up_proj.weight", gu + (size_t)64 * H * es, {F, H}, true);
    for (const char* nm : {"mlp.gate_proj.weight", "mlp.up_proj.weight"}) {
      Slot& sl = lm->slots.slots[p + nm];
      sl.transform = kXformRowInterleave;
      sl.t_b = H;
    }
    lm->slots.add(p + "mlp.down_proj.weight", L.wd, {H, F}, true);
  }
  std::vector<float> inv = rope_inv_freq(hd, c.rope_theta);
  lm->inv_freq = lm->arena.alloc<float>(hd / 2);
  if (!lm->embed || !lm->final_norm || !lm->inv_freq ||
      cudaMemcpy(lm->inv_freq, inv.data(), inv.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaStreamSynchronize(cudaStreamLegacy) != cudaSuccess) {
    delete lm;
    return set_error(CTTS_ERR_NOMEM, "device allocation failed");
  }
  *out = lm;
  return CTTS_OK;
}

extern "C" int ctts_lm_set_tensor(ctts_lm* lm, const char* name, const void* host, int dtype,
                                  const int64_t* shape, int ndim) {
  CTTS_REQ(lm, CTTS_ERR_ARG, "null handle");
  CTTS_CK(cudaSetDevice(lm->device));
  return slot_set(lm->slots, name, host, dtype, shape, ndim);
}

extern "C" int ctts_lm_load(ctts_lm* lm, const char* path, const char* prefix) {
  CTTS_REQ(lm, CTTS_ERR_ARG, "null handle");
  return load_safetensors(path, prefix, [&](const char* n, const void* d, int dt, const int64_t* s, int nd) {
    return ctts_lm_set_tensor(lm, n, d, dt, s, nd);
  });
}

extern "C" int ctts_lm_missing(const ctts_lm* lm) { return lm ? lm->slots.missing() : -1; }

extern "C" void ctts_lm_free(ctts_lm* lm) {
  if (!lm) return;
  cudaSetDevice(lm->device);
  cudaStreamSynchronize(lm->stream);
  cudaStreamDestroy(lm->stream);
  delete lm;
}

// ---------------------------------------------------------------------- KV

extern "C" int ctts_kv_alloc(const ctts_lm* lm, int batch, int capacity, ctts_kv** out) {
  CTTS_REQ(lm && out, CTTS_ERR_ARG, "null argument");
  CTTS_REQ(batch > 0 && capacity > 0, CTTS_ERR_ARG, "batch and capacity must be positive");
  CTTS_REQ(capacity <= 12000, CTTS_ERR_ARG, "capacity above 12000 positions");
  CTTS_CK(cudaSetDevice(lm->device));
  const ctts_lm_config& c = lm->cfg;
  auto* kv = new ctts_kv();
  kv->lm = lm;
  kv->batch = batch;
  kv->cap = capacity;
  const size_t es = lm->bf16 ? 2 : 4;
  kv->layer_elems = (size_t)batch * c.n_kv_heads * capacity * c.head_dim;
  kv->k = kv->arena.alloc<uint8_t>(kv->layer_elems * c.n_layers * es);
  kv->v = kv->arena.alloc<uint8_t>(kv->layer_elems * c.n_layers * es);
  kv->pos = kv->arena.alloc<int>(batch);
  kv->err = kv->arena.alloc<int>(1);
  kv->pos_host.assign(batch, 0);
  const int rows = std::max(batch, capacity);
  const int H = c.hidden, qd = c.n_heads * c.head_dim, kvd = c.n_kv_heads * c.head_dim;
  // keys per attention split: small batches use short splits so the
  // decode attention still spreads over many SMs
  kv->chunk = batch >= 16 ? 128 : 32;
  kv->nsplit = (capacity + kv->chunk - 1) / kv->chunk;
  kv->ws_rows = rows;
  kv->h = kv->arena.alloc<float>((size_t)rows * H);
  kv->qkv = kv->arena.alloc<float>((size_t)rows * (qd + 2 * kvd));
  kv->qrot = kv->arena.alloc<float>((size_t)rows * qd);
  kv->att = kv->arena.alloc<float>((size_t)rows * qd);
  kv->act = kv->arena.alloc<float>((size_t)rows * c.ffn);
  kv->part = kv->arena.alloc<float>((size_t)batch * c.n_heads * kv->nsplit * (c.head_dim + 2));
  kv->cnt = kv->arena.alloc<int>((size_t)batch * c.n_kv_heads);
  kv->gbar = kv->arena.alloc<unsigned>((size_t)ctts::lm_grid_counters(c.n_layers));
  kv->gpart = kv->arena.alloc<float>(ctts::lm_grid_part_floats(c.head_dim));
  kv->xin = kv->arena.alloc<float>((size_t)rows * H);
  kv->xout = kv->arena.alloc<float>((size_t)rows * H);
  if (!kv->k || !kv->v || !kv->pos || !kv->h || !kv->qkv || !kv->qrot || !kv->att || !kv->act ||
      !kv->part || !kv->cnt || !kv->xin || !kv->xout || !kv->gbar || !kv->gpart) {
    delete kv;
    return set_error(CTTS_ERR_NOMEM, "KV cache allocation failed");
  }
  if (lm->bf16) {
    kv->ssp = kv->arena.alloc<float>((size_t)((H + 127) / 128) * rows);
    kv->xb = kv->arena.alloc<uint16_t>((size_t)rows * std::max(H, qd));
    kv->attb = kv->arena.alloc<uint16_t>((size_t)rows * qd);
    kv->actb = kv->arena.alloc<uint16_t>((size_t)rows * c.ffn);
    const int qkvw = qd + 2 * kvd;
    std::vector<std::array<int, 3>> shapes;
    for (int m : {batch, std::min(rows, 256)})
      for (auto nk : {std::array<int, 2>{qkvw, H}, {H, qd}, {2 * c.ffn, H}, {H, c.ffn}})
        shapes.push_back({m, nk[0], nk[1]});
    int rc = tc_alloc(kv->arena, &kv->tc, shapes, kv->err);
    if (rc != CTTS_OK || !kv->xb || !kv->attb || !kv->actb || !kv->ssp) {
      delete kv;
      return rc != CTTS_OK ? rc : set_error(CTTS_ERR_NOMEM, "KV workspace allocation failed");
    }
  }
  *out = kv;
  return CTTS_OK;
}

extern "C" int ctts_kv_reset(ctts_kv* kv) {
  CTTS_REQ(kv, CTTS_ERR_ARG, "null handle");
  CTTS_CK(cudaSetDevice(kv->lm->device));
  CTTS_CK(cudaMemsetAsync(kv->pos, 0, sizeof(int) * kv->batch, kv->lm->stream));
  CTTS_CK(cudaMemsetAsync(kv->err, 0, sizeof(int), kv->lm->stream));
  CTTS_CK(cudaStreamSynchronize(kv->lm->stream));
  std::fill(kv->pos_host.begin(), kv->pos_host.end(), 0);
  return CTTS_OK;
}

extern "C" int ctts_kv_len(const ctts_kv* kv, int b) {
  if (!kv || b < 0 || b >= kv->batch) return set_error(CTTS_ERR_ARG, "bad handle or index");
  return kv->pos_host[b];
}

extern "C" int ctts_kv_set_len(ctts_kv* kv, int b, int len) {
  CTTS_REQ(kv && b >= 0 && b < kv->batch, CTTS_ERR_ARG, "bad handle or index");
  CTTS_REQ(len >= 0 && len <= kv->cap, CTTS_ERR_RANGE, "length outside [0, capacity]");
  CTTS_CK(cudaSetDevice(kv->lm->device));
  kv->pos_host[b] = len;
  CTTS_CK(cudaMemcpyAsync(kv->pos + b, &len, sizeof(int), cudaMemcpyHostToDevice, kv->lm->stream));
  CTTS_CK(cudaStreamSynchronize(kv->lm->stream));
  return CTTS_OK;
}

extern "C" void ctts_kv_free(ctts_kv* kv) {
  if (!kv) return;
  cudaSetDevice(kv->lm->device);
  cudaDeviceSynchronize();
  delete kv;
}

// ------------------------------------------------------------- LM forward

namespace ctts {

// Runs the layer stack over `rows` rows already in kv->h.  prefill_b >= 0:
// all rows belong to utterance prefill_b at positions pos0..; else one row
// per utterance at its device position.  Final-normed output -> out.
int lm_forward_rows(ctts_lm* lm, ctts_kv* kv, int rows, int prefill_b, int pos0, float* out,
                    cudaStream_t s, int* launches) {
  const ctts_lm_config& c = lm->cfg;
  const int H = c.hidden, hd = c.head_dim, qd = c.n_heads * hd, kvd = c.n_kv_heads * hd;
  const int qkvw = qd + 2 * kvd, F = c.ffn;
  const size_t es = lm->bf16 ? 2 : 4;
  int nl = 0;
  // bf16 weights with >= 16 rows: the tensor-core linears (tc_linear.cu);
  // otherwise the CUDA-core skinny linears (linear.cu).
  const bool tc = lm->bf16 && rows >= 16;
  // Tensor-core path: each residual-writing GEMM (o-proj, down) also writes
  // the next RMSNorm's operand bf16(h * gain) and per-tile row sums of
  // squares; the consuming GEMM (QKV, gate/up) applies 1/rms to its
  // accumulator rows, so only layer 0 needs a separate norm pass.
  const int nt = (H + 127) / 128;
  auto fold_in = [&](TcArgs& e) {
    e.rs_ssp = kv->ssp; e.rs_ld = kv->ws_rows; e.rs_nt = nt; e.rs_k = (float)H; e.rs_eps = c.rms_eps;
  };
  auto fold_out = [&](TcArgs& e, const float* gain) {
    e.yb2 = kv->xb; e.g2 = gain; e.ssp = kv->ssp; e.ssp_ld = kv->ws_rows;
  };
  // Small decode batches with fp32 weights: the whole step (every layer,
  // the final norm and the position advance) as one grid-persistent launch
  // (lm_grid.cu) unless CTTS_LM_GRID=0.
  const char* grid_e = getenv("CTTS_LM_GRID");
  if (prefill_b < 0 && !lm->bf16 && rows == kv->batch && (!grid_e || atoi(grid_e) != 0) &&
      ctts::lm_grid_supported(rows, c.n_layers, H, c.n_heads, c.n_kv_heads, hd, F)) {
    ctts::LmGridArgs g;
    g.R = rows; g.NL = c.n_layers; g.H = H; g.nq = c.n_heads; g.nkv = c.n_kv_heads; g.hd = hd; g.F = F;
    g.cap = kv->cap; g.eps = c.rms_eps;
    g.h = kv->h; g.qkv = kv->qkv; g.part = kv->gpart; g.act = kv->act; g.out = out;
    g.final_norm = lm->final_norm; g.pos = kv->pos; g.inv_freq = lm->inv_freq;
    g.kcache = static_cast<float*>(kv->k); g.vcache = static_cast<float*>(kv->v); g.layer_elems = kv->layer_elems;
    for (int l = 0; l < c.n_layers; l++) {
      const LMLayer& L = lm->layers[l];
      g.wqkv[l] = static_cast<const float*>(L.wqkv); g.wo[l] = static_cast<const float*>(L.wo);
      g.wgu[l] = static_cast<const float*>(L.wgu); g.wd[l] = static_cast<const float*>(L.wd);
      g.norm1[l] = L.norm1; g.norm2[l] = L.norm2;
      g.qn[l] = c.qk_norm ? L.qn : nullptr; g.kn[l] = c.qk_norm ? L.kn : nullptr;
    }
    g.bar = kv->gbar; g.err = kv->err;
    CTTS_CK(ctts::launch_lm_grid(g, s)); nl++;
    if (launches) *launches += nl;
    return CTTS_OK;
  }
  for (int l = 0; l < c.n_layers; l++) {
    const LMLayer& L = lm->layers[l];
    if (tc) {
      TcArgs e; e.y = kv->qkv; e.y_ld = qkvw;
      if (l == 0) {
        PrepArgs pa;
        pa.x = kv->h; pa.x_ld = H; pa.y = kv->xb; pa.y_ld = H; pa.M = rows; pa.K = H;
        pa.norm_w = L.norm1; pa.eps = c.rms_eps;
        CTTS_CK(launch_prep_bf16(pa, s)); nl++;
      } else {
        fold_in(e);
      }
      int rc = tc_run(kv->tc, kv->xb, rows, H, L.wqkv, qkvw, e, s, &nl);
      if (rc) return rc;
    } else {
      LinearArgs q;
      q.x = kv->h; q.x_ld = H; q.M = rows; q.K = H; q.N = qkvw;
      q.w = L.wqkv; q.w_bf16 = lm->bf16; q.y = kv->qkv; q.y_ld = qkvw;
      q.norm_w = L.norm1; q.eps = c.rms_eps;
      CTTS_CK(launch_linear(q, s)); nl++;
    }

    AttnArgs a;
    a.qkv = kv->qkv; a.rows = rows; a.prefill_b = prefill_b; a.pos0 = pos0; a.pos = kv->pos;
    a.nq = c.n_heads; a.nkv = c.n_kv_heads; a.hd = hd;
    a.qn = c.qk_norm ? L.qn : nullptr; a.kn = c.qk_norm ? L.kn : nullptr; a.eps = c.rms_eps;
    a.inv_freq = lm->inv_freq;
    a.kcache = reinterpret_cast<uint8_t*>(kv->k) + (size_t)l * kv->layer_elems * es;
    a.vcache = reinterpret_cast<uint8_t*>(kv->v) + (size_t)l * kv->layer_elems * es;
    a.kv_bf16 = lm->bf16; a.cap = kv->cap; a.batch = kv->batch;
    a.qrot = kv->qrot; a.out = kv->att; a.part = kv->part; a.nsplit = kv->nsplit; a.chunk = kv->chunk;
    a.cnt = kv->cnt; a.err = kv->err;
    if (tc) a.out_b = kv->attb;
    if (prefill_b >= 0) {
      CTTS_CK(launch_qk_rope_append(a, s)); nl++;
      CTTS_CK(launch_attn_prefill(a, s)); nl++;
    } else {  // norm/RoPE, KV append, attention and split merge in one launch
      CTTS_CK(launch_attn_decode(a, s)); nl++;
    }

    if (tc) {
      TcArgs e; e.y = kv->h; e.y_ld = H; e.res = kv->h;
      fold_out(e, L.norm2);
      int rc = tc_run(kv->tc, kv->attb, rows, qd, L.wo, H, e, s, &nl);
      if (rc) return rc;
      TcArgs g; g.act = 2; g.yb = kv->actb; g.y_ld = F;
      fold_in(g);
      rc = tc_run(kv->tc, kv->xb, rows, H, L.wgu, 2 * F, g, s, &nl);
      if (rc) return rc;
      TcArgs d; d.y = kv->h; d.y_ld = H; d.res = kv->h;
      if (l + 1 < c.n_layers) fold_out(d, lm->layers[l + 1].norm1);
      rc = tc_run(kv->tc, kv->actb, rows, F, L.wd, H, d, s, &nl);
      if (rc) return rc;
      continue;
    }

    LinearArgs o;
    o.x = kv->att; o.x_ld = qd; o.M = rows; o.K = qd; o.N = H;
    o.w = L.wo; o.w_bf16 = lm->bf16; o.y = kv->h; o.y_ld = H; o.res = kv->h;
    CTTS_CK(launch_linear(o, s)); nl++;

    LinearArgs g;
    g.x = kv->h; g.x_ld = H; g.M = rows; g.K = H; g.N = F;
    g.w = L.wgu; g.w_bf16 = lm->bf16; g.y = kv->act; g.y_ld = F; g.act = 2;
    g.norm_w = L.norm2; g.eps = c.rms_eps;
    CTTS_CK(launch_linear(g, s)); nl++;

    LinearArgs d;
    d.x = kv->act; d.x_ld = F; d.M = rows; d.K = F; d.N = H;
    d.w = L.wd; d.w_bf16 = lm->bf16; d.y = kv->h; d.y_ld = H; d.res = kv->h;
    CTTS_CK(launch_linear(d, s)); nl++;
  }
  CTTS_CK(launch_rmsnorm_rows(kv->h, rows, H, lm->final_norm, c.rms_eps, out, s)); nl++;
  if (prefill_b < 0) {
    CTTS_CK(launch_advance_pos(kv->pos, kv->batch, s));
    nl++;
  }
  if (launches) *launches += nl;
  return CTTS_OK;
}

int lm_check_ready(const ctts_lm* lm) {
  if (lm->slots.missing())
    return set_error(CTTS_ERR_STATE, "LM weights missing: " + lm->slots.first_missing());
  return CTTS_OK;
}

int lm_decode_dev(ctts_lm* lm, ctts_kv* kv, const float* x_dev, float* out_dev, cudaStream_t s,
                  int* launches) {
  for (int b = 0; b < kv->batch; b++)
    CTTS_REQ(kv->pos_host[b] < kv->cap, CTTS_ERR_RANGE, "KV cache full");
  const int H = lm->cfg.hidden;
  if (x_dev != kv->h)
    CTTS_CK(cudaMemcpyAsync(kv->h, x_dev, sizeof(float) * kv->batch * H, cudaMemcpyDeviceToDevice, s));
  int rc = lm_forward_rows(lm, kv, kv->batch, -1, 0, out_dev, s, launches);
  if (rc != CTTS_OK) return rc;
  for (int b = 0; b < kv->batch; b++) kv->pos_host[b]++;
  return CTTS_OK;
}

}  // namespace ctts

extern "C" int ctts_lm_prefill_dev(ctts_lm* lm, ctts_kv* kv, int b, const float* x_dev, int T,
                                   float* out_dev, void* stream) {
  CTTS_REQ(lm && kv && kv->lm == lm && x_dev && out_dev, CTTS_ERR_ARG, "null or mismatched argument");
  CTTS_REQ(b >= 0 && b < kv->batch && T > 0, CTTS_ERR_ARG, "bad utterance index or length");
  CTTS_REQ(lm_check_ready(lm) == CTTS_OK, CTTS_ERR_STATE, ctts_last_error());
  const int pos0 = kv->pos_host[b];
  CTTS_REQ(pos0 + T <= kv->cap && T <= kv->ws_rows, CTTS_ERR_RANGE, "prefill exceeds KV capacity");
  CTTS_CK(cudaSetDevice(lm->device));
  cudaStream_t s = as_stream(stream, lm->stream);
  const int H = lm->cfg.hidden;
  CTTS_CK(cudaMemcpyAsync(kv->h, x_dev, sizeof(float) * T * H, cudaMemcpyDeviceToDevice, s));
  int rc = lm_forward_rows(lm, kv, T, b, pos0, out_dev, s, nullptr);
  if (rc != CTTS_OK) return rc;
  kv->pos_host[b] = pos0 + T;
  int np = pos0 + T;
  CTTS_CK(cudaMemcpyAsync(kv->pos + b, &np, sizeof(int), cudaMemcpyHostToDevice, s));
  CTTS_CK(cudaStreamSynchronize(s));  // &np is a stack value
  return CTTS_OK;
}

extern "C" int ctts_lm_prefill(ctts_lm* lm, ctts_kv* kv, int b, const float* x, int T, float* out) {
  CTTS_REQ(lm && kv && x && out, CTTS_ERR_ARG, "null argument");
  CTTS_REQ(T > 0 && T <= kv->ws_rows, CTTS_ERR_RANGE, "prefill length outside workspace");
  CTTS_CK(cudaSetDevice(lm->device));
  const size_t n = (size_t)T * lm->cfg.hidden;
  // stream-ordered with the kernels that consume it
  CTTS_CK(cudaMemcpyAsync(kv->xin, x, n * 4, cudaMemcpyHostToDevice, lm->stream));
  int rc = ctts_lm_prefill_dev(lm, kv, b, kv->xin, T, kv->xout, nullptr);
  if (rc != CTTS_OK) return rc;
  CTTS_CK(cudaMemcpy(out, kv->xout, n * 4, cudaMemcpyDeviceToHost));
  return CTTS_OK;
}

extern "C" int ctts_lm_decode_step_dev(ctts_lm* lm, ctts_kv* kv, const float* x_dev, float* out_dev,
                                       void* stream) {
  CTTS_REQ(lm && kv && kv->lm == lm && x_dev && out_dev, CTTS_ERR_ARG, "null or mismatched argument");
  CTTS_REQ(lm_check_ready(lm) == CTTS_OK, CTTS_ERR_STATE, ctts_last_error());
  CTTS_CK(cudaSetDevice(lm->device));
  return lm_decode_dev(lm, kv, x_dev, out_dev, as_stream(stream, lm->stream), nullptr);
}

extern "C" int ctts_lm_decode_step(ctts_lm* lm, ctts_kv* kv, const float* x, float* out) {
  CTTS_REQ(lm && kv && x && out, CTTS_ERR_ARG, "null argument");
  CTTS_CK(cudaSetDevice(lm->device));
  const size_t n = (size_t)kv->batch * lm->cfg.hidden;
  CTTS_CK(cudaMemcpyAsync(kv->xin, x, n * 4, cudaMemcpyHostToDevice, lm->stream));
  int rc = ctts_lm_decode_step_dev(lm, kv, kv->xin, kv->xout, nullptr);
  if (rc != CTTS_OK) return rc;
  CTTS_CK(cudaStreamSynchronize(lm->stream));
  int err = 0;
  CTTS_CK(cudaMemcpy(&err, kv->err, sizeof(int), cudaMemcpyDeviceToHost));
  CTTS_REQ(err != 1, CTTS_ERR_RANGE, "device reported a KV position outside capacity");
  CTTS_REQ(err == 0, CTTS_ERR_TIMEOUT, "a tensor-core linear gave up waiting on its pipeline");
  CTTS_CK(cudaMemcpy(out, kv->xout, n * 4, cudaMemcpyDeviceToHost));
  return CTTS_OK;
}

extern "C" int ctts_lm_embed_lookup(ctts_lm* lm, const int64_t* ids, int n, float* out) {
  CTTS_REQ(lm && ids && out && n >= 0, CTTS_ERR_ARG, "null argument");
  CTTS_REQ(lm->slots.slots["embed_tokens.weight"].set, CTTS_ERR_STATE, "embedding table not loaded");
  for (int i = 0; i < n; i++)
    CTTS_REQ(ids[i] >= 0 && ids[i] < lm->cfg.vocab, CTTS_ERR_RANGE,
             "token id " + std::to_string(ids[i]) + " out of range");
  if (n == 0) return CTTS_OK;
  CTTS_CK(cudaSetDevice(lm->device));
  const int H = lm->cfg.hidden;
  int64_t* d_ids = nullptr;
  float* d_out = nullptr;
  CTTS_CK(cudaMalloc(&d_ids, n * 8));
  if (cudaMalloc(&d_out, (size_t)n * H * 4) != cudaSuccess) {
    cudaFree(d_ids);
    return set_error(CTTS_ERR_NOMEM, "embed scratch");
  }
  cudaError_t e = cudaMemcpyAsync(d_ids, ids, n * 8, cudaMemcpyHostToDevice, lm->stream);
  if (e == cudaSuccess) e = launch_embed_gather(lm->embed, lm->bf16, lm->cfg.vocab, H, d_ids, n, d_out, nullptr, lm->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(lm->stream);
  if (e == cudaSuccess) e = cudaMemcpy(out, d_out, (size_t)n * H * 4, cudaMemcpyDeviceToHost);
  cudaFree(d_ids);
  cudaFree(d_out);
  CTTS_CK(e);
  return CTTS_OK;
}

// -------------------------------------------------------------- op level

namespace {

// Per-device workspace of the op-level tensor-core linear (bf16 operand +
// split-K scratch), grown on demand.
struct OpTcWs {
  size_t xb_elems = 0, part = 0;
  int counters = 0;
  DevArena* arena = nullptr;
  uint16_t* xb = nullptr;
  TcScratch tc;
  int* err = nullptr;
};

int op_tc_ws(int M, int N, int K, OpTcWs** out) {
  static thread_local std::unordered_map<int, OpTcWs> wss;
  int dev = 0;
  CTTS_CK(cudaGetDevice(&dev));
  OpTcWs& w = wss[dev];
  int cnt = 0;
  size_t need = tc_scratch_need({{M, N, K}}, 64, &cnt);
  if (!w.arena || (size_t)M * K > w.xb_elems || need > w.part || cnt > w.counters) {
    CTTS_CK(cudaDeviceSynchronize());
    delete w.arena;
    w.arena = new DevArena();
    w.xb_elems = std::max((size_t)M * K, w.xb_elems);
    w.part = std::max(need, w.part);
    w.counters = std::max(cnt, w.counters);
    w.xb = w.arena->alloc<uint16_t>(w.xb_elems);
    w.err = w.arena->alloc<int>(1);
    w.tc.part = w.arena->alloc<float>(std::max<size_t>(w.part, 1));
    w.tc.part_floats = w.part;
    w.tc.counters = w.arena->alloc<int>(std::max(w.counters, 1));
    w.tc.ncounters = w.counters;
    w.tc.err = w.err;
    if (!w.xb || !w.tc.part || !w.tc.counters) return set_error(CTTS_ERR_NOMEM, "op workspace");
  }
  *out = &w;
  return CTTS_OK;
}

}  // namespace

extern "C" int ctts_op_linear(const float* x, int M, int K, const void* w, int w_dtype, int N,
                              const float* norm_w, float eps, const float* res, float* y,
                              void* stream) {
  CTTS_REQ(x && w && y && M >= 0 && K > 0 && N > 0, CTTS_ERR_ARG, "bad argument");
  CTTS_REQ(K % (w_dtype == CTTS_BF16 ? 8 : 4) == 0, CTTS_ERR_ARG, "K must be a multiple of 4 (f32) / 8 (bf16)");
  cudaStream_t s = as_stream(stream, 0);
  if (w_dtype == CTTS_BF16 && M >= 16 && K % 64 == 0) {
    // bf16 weights and a batch of rows: tcgen05 tensor cores, the activation
    // is normalized and rounded to bf16 first
    OpTcWs* ws = nullptr;
    int rc = op_tc_ws(M, N, K, &ws);
    if (rc) return rc;
    PrepArgs pa;
    pa.x = x; pa.x_ld = K; pa.y = ws->xb; pa.y_ld = K; pa.M = M; pa.K = K; pa.norm_w = norm_w; pa.eps = eps;
    CTTS_CK(launch_prep_bf16(pa, s));
    TcArgs e; e.y = y; e.y_ld = N; e.res = res;
    return tc_run(ws->tc, ws->xb, M, K, w, N, e, s, nullptr);
  }
  LinearArgs a;
  a.x = x; a.x_ld = K; a.M = M; a.K = K; a.N = N; a.w = w; a.w_bf16 = w_dtype == CTTS_BF16;
  a.y = y; a.y_ld = N; a.norm_w = norm_w; a.eps = eps; a.res = res;
  CTTS_CK(launch_linear(a, s));
  return CTTS_OK;
}

extern "C" int ctts_op_rope(float* x, int M, int heads, int head_dim, const int* pos, float theta,
                            void* stream) {
  CTTS_REQ(x && pos && M >= 0 && heads > 0 && head_dim > 0 && head_dim % 2 == 0, CTTS_ERR_ARG,
           "bad argument");
  // inverse frequencies: small per-call device table (cached per (hd, theta))
  static thread_local std::unordered_map<std::string, float*> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  std::string key = std::to_string(dev) + ":" + std::to_string(head_dim) + ":" + std::to_string(theta);
  float*& inv = cache[key];
  if (!inv) {
    std::vector<float> h = rope_inv_freq(head_dim, theta);
    CTTS_CK(cudaMalloc(&inv, h.size() * 4));
    CTTS_CK(cudaMemcpy(inv, h.data(), h.size() * 4, cudaMemcpyHostToDevice));
    CTTS_CK(cudaStreamSynchronize(cudaStreamLegacy));
  }
  CTTS_CK(launch_rope_inplace(x, M, heads, head_dim, pos, inv, as_stream(stream, 0)));
  return CTTS_OK;
}

extern "C" int ctts_op_swiglu(const float* gu, int M, int F, float* out, void* stream) {
  CTTS_REQ(gu && out && M >= 0 && F > 0, CTTS_ERR_ARG, "bad argument");
  CTTS_CK(launch_swiglu(gu, M, F, out, as_stream(stream, 0)));
  return CTTS_OK;
}

extern "C" int ctts_op_embed_gather(const float* table, int vocab, int H, const int64_t* ids, int n,
                                    float* out, int* bad_count, void* stream) {
  CTTS_REQ(table && ids && out && vocab > 0 && H > 0 && n >= 0, CTTS_ERR_ARG, "bad argument");
  CTTS_CK(launch_embed_gather(table, 0, vocab, H, ids, n, out, bad_count, as_stream(stream, 0)));
  return CTTS_OK;
}
