// api_vae.cu -- C ABI: the causal VAE decoder (decode.rs / weights.rs /
// ffi.rs, audio_vae.py:243-292) at generic topology.
#include <cstdio>
#include <cstdlib>

#include "api_common.h"
#include "model.h"

using namespace ctts;

namespace {

constexpr int kTransposeRepack = 1;

// weight-norm fuse w = g * v / ||v|| per output channel, in double
// (conv.rs:12-30).
void fuse_wn(const std::vector<float>& g, const std::vector<float>& v, size_t O, std::vector<float>* w) {
  size_t ik = v.size() / O;
  w->resize(v.size());
  for (size_t o = 0; o < O; o++) {
    double s = 0.0;
    for (size_t i = 0; i < ik; i++) {
      double x = v[o * ik + i];
      s += x * x;
    }
    double n = std::sqrt(s);
    double scale = (double)g[o] / (n > 1e-12 ? n : 1e-12);
    for (size_t i = 0; i < ik; i++) (*w)[o * ik + i] = (float)((double)v[o * ik + i] * scale);
  }
}

// ConvTranspose1d weight [cin, cout, 2s] -> per-phase conv weights
// [s][cout][cin*2]: tap 0 multiplies x[i-1] (W[c,o,s+j]), tap 1 x[i]
// (W[c,o,j]); output sample i*s + j (decode.rs:39-80, weights.rs:133-147).
void repack_transpose(const float* w, int cin, int cout, int s, std::vector<float>* out) {
  out->assign((size_t)s * cout * cin * 2, 0.0f);
  for (int j = 0; j < s; j++)
    for (int o = 0; o < cout; o++)
      for (int c = 0; c < cin; c++) {
        (*out)[(((size_t)j * cout + o) * cin + c) * 2 + 0] = w[((size_t)c * cout + o) * 2 * s + s + j];
        (*out)[(((size_t)j * cout + o) * cin + c) * 2 + 1] = w[((size_t)c * cout + o) * 2 * s + j];
      }
}

int vae_store(ctts_vae* v, Slot& s, const std::vector<float>& w) {
  if (s.transform == kTransposeRepack) {
    std::vector<float> rp;
    repack_transpose(w.data(), s.t_a, s.t_b, s.t_c, &rp);
    return upload_f32(s, rp.data(), rp.size(), v->bf16);
  }
  return upload_f32(s, w.data(), w.size(), v->bf16);
}

}  // namespace

extern "C" int ctts_vae_create(const ctts_vae_config* cfg, int device, ctts_vae** out) {
  CTTS_REQ(cfg && out, CTTS_ERR_ARG, "null argument");
  const ctts_vae_config& c = *cfg;
  CTTS_REQ(c.latent > 0 && c.channels > 0 && c.n_stages > 0 && c.n_stages <= 8, CTTS_ERR_ARG, "bad dims");
  CTTS_REQ(c.weight_dtype == CTTS_F32 || c.weight_dtype == CTTS_BF16, CTTS_ERR_ARG, "bad weight dtype");
  for (int i = 0; i < c.n_stages; i++) CTTS_REQ(c.strides[i] > 0, CTTS_ERR_ARG, "bad stride");
  CTTS_REQ((c.channels >> c.n_stages) > 0 && ((c.channels >> c.n_stages) << c.n_stages) == c.channels,
           CTTS_ERR_ARG, "channels must halve cleanly per stage");
  CTTS_CK(cudaSetDevice(device));
  auto* v = new ctts_vae();
  v->cfg = c;
  v->device = device;
  v->bf16 = c.weight_dtype == CTTS_BF16;
  v->slots.model_bf16 = v->bf16;
  cudaStreamCreateWithFlags(&v->stream, cudaStreamNonBlocking);
  const size_t es = v->bf16 ? 2 : 4;
  DevArena& A = v->arena;
  auto W = [&](size_t n) -> void* { return A.alloc<uint8_t>(n * es); };
  auto conv = [&](const std::string& p, void** w, float** b, int o, int i, int k) {
    *w = W((size_t)o * i * k);
    *b = A.alloc<float>(o);
    v->slots.add(p + ".weight", *w, {o, i, k}, true);
    v->slots.add(p + ".bias", *b, {o}, false);
  };
  const int C = c.channels, L = c.latent;
  // dense: model.0 = Conv(latent -> channels, k7); depthwise (the shipped
  // topology, audio_vae.py:255-266): model.0 = depthwise k7 on the latent,
  // model.1 = pointwise latent -> channels (weights.rs:115-121)
  int idx = 1;
  if (c.depthwise) {
    conv("model.0", &v->front_w, &v->front_b, L, 1, 7);
    conv("model.1", &v->front_pw_w, &v->front_pw_b, C, L, 1);
    idx = 2;
  } else {
    conv("model.0", &v->front_w, &v->front_b, C, L, 7);
  }
  v->hop = 1;
  v->stages.resize(c.n_stages);
  for (int si = 0; si < c.n_stages; si++) {
    VaeStage& st = v->stages[si];
    st.cin = C >> si;
    st.cout = C >> (si + 1);
    st.stride = c.strides[si];
    v->hop *= st.stride;
    std::string b = "model." + std::to_string(idx + si) + ".block.";
    st.alpha = A.alloc<float>(st.cin);
    v->slots.add(b + "0.alpha", st.alpha, {1, st.cin, 1}, false);
    st.tw = W((size_t)st.stride * st.cout * st.cin * 2);
    st.tb = A.alloc<float>(st.cout);
    v->slots.add(b + "1.weight", st.tw, {st.cin, st.cout, 2 * st.stride}, true);
    Slot& ts = v->slots.slots[b + "1.weight"];
    ts.transform = kTransposeRepack;
    ts.t_a = st.cin;
    ts.t_b = st.cout;
    ts.t_c = st.stride;
    v->slots.add(b + "1.bias", st.tb, {st.cout}, false);
    for (int r = 0; r < 3; r++) {
      std::string rb = b + std::to_string(2 + r) + ".block.";
      VaeRes& R = st.res[r];
      R.a0 = A.alloc<float>(st.cout);
      R.a1 = A.alloc<float>(st.cout);
      v->slots.add(rb + "0.alpha", R.a0, {1, st.cout, 1}, false);
      v->slots.add(rb + "2.alpha", R.a1, {1, st.cout, 1}, false);
      conv(rb + "1", &R.w0, &R.b0, st.cout, c.depthwise ? 1 : st.cout, 7);  // depthwise: [C, 1, 7]
      conv(rb + "3", &R.w1, &R.b1, st.cout, st.cout, 1);
    }
  }
  const int fi = idx + c.n_stages, ch = C >> c.n_stages;
  v->final_alpha = A.alloc<float>(ch);
  v->slots.add("model." + std::to_string(fi) + ".alpha", v->final_alpha, {1, ch, 1}, false);
  conv("model." + std::to_string(fi + 1), &v->final_w, &v->final_b, 1, ch, 7);
  v->err = A.alloc<int>(1);
  if (!v->final_b || !v->err) {
    delete v;
    return set_error(CTTS_ERR_NOMEM, "device allocation failed");
  }
  *out = v;
  return CTTS_OK;
}

extern "C" int ctts_vae_set_tensor(ctts_vae* v, const char* name, const void* host, int dtype,
                                   const int64_t* shape, int ndim) {
  CTTS_REQ(v && name && host && (ndim == 0 || shape), CTTS_ERR_ARG, "null argument");
  CTTS_REQ(dtype == CTTS_F32 || dtype == CTTS_BF16, CTTS_ERR_ARG, "bad dtype");
  CTTS_CK(cudaSetDevice(v->device));
  std::string n = name;
  std::vector<int64_t> got(shape, shape + ndim);
  std::vector<float> f;
  host_to_f32(host, dtype, shape_numel(got), &f);
  // weight-norm halves: "<p>.weight_g" [O,1,1] and "<p>.weight_v" [O,I,K]
  auto ends = [&](const char* suf) {
    size_t l = strlen(suf);
    return n.size() > l && n.compare(n.size() - l, l, suf) == 0;
  };
  if (ends(".weight_g") || ends(".weight_v")) {
    std::string base = n.substr(0, n.size() - 2);  // "...weight"
    auto it = v->slots.slots.find(base);
    CTTS_REQ(it != v->slots.slots.end(), CTTS_ERR_ARG, "unknown tensor " + n);
    Slot& s = it->second;
    const int64_t O = s.transform == kTransposeRepack ? s.shape[0] : s.shape[0];
    if (ends(".weight_g")) {
      CTTS_REQ(got.size() == 3 && got[0] == O && got[1] == 1 && got[2] == 1, CTTS_ERR_ARG,
               "shape for " + n + ": " + shape_str(got));
      s.wn_g = f;
    } else {
      CTTS_REQ(got == s.shape, CTTS_ERR_ARG, "shape for " + n + ": " + shape_str(got));
      s.wn_v = f;
    }
    if (!s.wn_g.empty() && !s.wn_v.empty()) {
      std::vector<float> w;
      fuse_wn(s.wn_g, s.wn_v, (size_t)O, &w);
      int rc = vae_store(v, s, w);
      if (rc) return rc;
      s.set = true;
      v->tc_dirty = true;
      s.wn_g.clear();
      s.wn_v.clear();
    }
    return CTTS_OK;
  }
  auto it = v->slots.slots.find(n);
  CTTS_REQ(it != v->slots.slots.end(), CTTS_ERR_ARG, "unknown tensor " + n);
  Slot& s = it->second;
  CTTS_REQ(got == s.shape, CTTS_ERR_ARG,
           "shape for " + n + ": got " + shape_str(got) + ", want " + shape_str(s.shape));
  int rc = vae_store(v, s, f);
  if (rc) return rc;
  s.set = true;
  v->tc_dirty = true;
  return CTTS_OK;
}

extern "C" int ctts_vae_load_file(ctts_vae* v, const char* path, const char* prefix) {
  CTTS_REQ(v, CTTS_ERR_ARG, "null handle");
  return load_safetensors(path, prefix, [&](const char* n, const void* d, int dt, const int64_t* s, int nd) {
    return ctts_vae_set_tensor(v, n, d, dt, s, nd);
  });
}

extern "C" int ctts_vae_missing(const ctts_vae* v) { return v ? v->slots.missing() : -1; }

extern "C" void ctts_vae_free(ctts_vae* v) {
  if (!v) return;
  cudaSetDevice(v->device);
  cudaStreamSynchronize(v->stream);
  cudaStreamDestroy(v->stream);
  delete v;
}

namespace {

int vae_ws_ensure(ctts_vae* v, int B, int T) {
  size_t need = 0;
  int t = T;
  need = std::max(need, (size_t)std::max(v->cfg.channels, v->cfg.latent) * t);
  for (auto& st : v->stages) {
    t *= st.stride;
    need = std::max(need, (size_t)st.cout * t);
  }
  need *= (size_t)B;
  if (need <= v->ws_elems) return CTTS_OK;
  cudaDeviceSynchronize();
  v->ws_arena.~DevArena();
  new (&v->ws_arena) DevArena();
  for (int i = 0; i < 3; i++) {
    v->buf[i] = v->ws_arena.alloc<float>(need);
    if (!v->buf[i]) {
      v->ws_elems = 0;
      return set_error(CTTS_ERR_NOMEM, "VAE workspace (" + std::to_string(need * 4 >> 20) + " MiB x3)");
    }
  }
  v->ws_elems = need;
  return CTTS_OK;
}

}  // namespace

namespace ctts {

int cout_pad128(int c) { return (c + 127) / 128 * 128; }

// Rebuilds the tensor-core copies of the bf16 dense conv weights after an
// upload (synchronous; outside any stream capture).
int vae_tc_prepare(ctts_vae* v) {
  if (!v->bf16 || !v->tc_dirty) return CTTS_OK;
  CTTS_CK(cudaDeviceSynchronize());
  v->tc_arena.~DevArena();
  new (&v->tc_arena) DevArena();
  auto make = [&](const void* w, int nphase, int cout, int cin, int k, void** out) -> int {
    *out = nullptr;
    ConvArgs probe;
    probe.w_bf16 = 1; probe.w_tc = w; probe.cout_pad = cout_pad128(cout); probe.Cin = cin; probe.Cout = cout;
    probe.k = k; probe.dil = 1;
    if (!conv_tc_supported(probe)) return CTTS_OK;  // stays on the CUDA-core kernel
    uint16_t* d = v->tc_arena.alloc<uint16_t>((size_t)nphase * k * cin * cout_pad128(cout));
    if (!d) return set_error(CTTS_ERR_NOMEM, "VAE tensor-core weights");
    CTTS_CK(repack_conv_tc(d, static_cast<const uint16_t*>(w), nphase, cout, cin, k, cout_pad128(cout), nullptr));
    *out = d;
    return CTTS_OK;
  };
  const ctts_vae_config& c = v->cfg;
  int rc = CTTS_OK;
  if (c.depthwise) {
    rc = make(v->front_pw_w, 1, c.channels, c.latent, 1, &v->front_pw_tc);
  } else {
    rc = make(v->front_w, 1, c.channels, c.latent, 7, &v->front_tc);
  }
  for (auto& st : v->stages) {
    if (!rc) rc = make(st.tw, st.stride, st.cout, st.cin, 2, &st.tw_tc);
    for (auto& R : st.res) {
      if (!rc && !c.depthwise) rc = make(R.w0, 1, st.cout, st.cout, 7, &R.w0_tc);
      if (!rc) rc = make(R.w1, 1, st.cout, st.cout, 1, &R.w1_tc);
    }
  }
  if (rc) return rc;
  CTTS_CK(cudaDeviceSynchronize());
  v->tc_dirty = false;
  return CTTS_OK;
}

// Points a conv at its tensor-core weights (null: CUDA-core kernel).
void use_tc(const ctts_vae* v, ConvArgs& a, const void* w_tc) {
  a.w_tc = w_tc;
  a.cout_pad = cout_pad128(a.Cout);
  a.err = v->err;
}

// Reads back (and clears) the tensor-core convs' error word after a
// synchronized decode.
int vae_read_err(ctts_vae* v) {
  int err = 0;
  CTTS_CK(cudaMemcpy(&err, v->err, sizeof(int), cudaMemcpyDeviceToHost));
  if (err != 0) CTTS_CK(cudaMemset(v->err, 0, sizeof(int)));
  CTTS_REQ(err == 0, CTTS_ERR_TIMEOUT, "a VAE tensor-core conv gave up waiting on its pipeline");
  return CTTS_OK;
}

}  // namespace ctts

namespace {

// Per-stage timing of a host decode under CUTETTS_PROFILE=1 (the "[prof]"
// lines of decode.rs:12-24): CUDA events recorded between the stages,
// printed to stderr after the decode synchronizes.
struct VaeProf {
  std::vector<std::pair<std::string, cudaEvent_t>> marks;
  int mark(const std::string& name, cudaStream_t s) {
    cudaEvent_t ev = nullptr;
    CTTS_CK(cudaEventCreate(&ev));
    marks.emplace_back(name, ev);
    CTTS_CK(cudaEventRecord(ev, s));
    return CTTS_OK;
  }
  void report() {
    for (size_t i = 1; i < marks.size(); i++) {
      float ms = 0.0f;
      if (cudaEventElapsedTime(&ms, marks[i - 1].second, marks[i].second) == cudaSuccess)
        fprintf(stderr, "[prof] %-24s %8.3fms\n", marks[i].first.c_str(), ms);
    }
  }
  ~VaeProf() {
    for (auto& m : marks) cudaEventDestroy(m.second);
  }
};

bool vae_profile_env() {
  const char* e = getenv("CUTETTS_PROFILE");
  return e && e[0] == '1' && e[1] == 0;
}

int vae_enqueue(ctts_vae* v, int B, const float* lat, int T, float* wav, cudaStream_t s, VaeProf* prof = nullptr) {
  const int bf = v->bf16;
  auto mark = [&](const std::string& name) -> int { return prof ? prof->mark(name, s) : CTTS_OK; };
  if (int rc = mark("start")) return rc;
  float* h = v->buf[0];
  float* h2 = v->buf[1];
  float* r = v->buf[2];
  const int dw = v->cfg.depthwise;
  ConvArgs a;
  a.x = lat; a.w = v->front_w; a.w_bf16 = bf; a.bias = v->front_b; a.y = dw ? r : h;
  a.B = B; a.Cin = v->cfg.latent; a.Cout = dw ? v->cfg.latent : v->cfg.channels; a.Tin = T; a.Tout = T; a.k = 7;
  a.dil = 1; a.left = 6; a.groups = dw ? v->cfg.latent : 1;
  if (!dw) use_tc(v, a, v->front_tc);
  CTTS_CK(launch_conv1d(a, s));
  if (dw) {  // pointwise latent -> channels
    ConvArgs p;
    p.x = r; p.w = v->front_pw_w; p.w_bf16 = bf; p.bias = v->front_pw_b; p.y = h;
    p.B = B; p.Cin = v->cfg.latent; p.Cout = v->cfg.channels; p.Tin = T; p.Tout = T; p.k = 1; p.dil = 1; p.left = 0;
    use_tc(v, p, v->front_pw_tc);
    CTTS_CK(launch_conv1d(p, s));
  }
  if (int rc = mark("front conv")) return rc;
  int t = T;
  static const int dils[3] = {1, 3, 9};
  for (auto& st : v->stages) {
    ConvArgs tr;
    tr.x = h; tr.w = st.tw; tr.w_bf16 = bf; tr.bias = st.tb; tr.y = h2; tr.snake_alpha = st.alpha;
    tr.B = B; tr.Cin = st.cin; tr.Cout = st.cout; tr.Tin = t; tr.Tout = t * st.stride; tr.k = 2;
    tr.dil = 1; tr.left = 1; tr.stride = st.stride;
    use_tc(v, tr, st.tw_tc);
    CTTS_CK(launch_conv_transpose(tr, s));
    t *= st.stride;
    std::swap(h, h2);
    const std::string sn = "stage " + std::to_string(&st - v->stages.data()) + " ";
    if (int rc = mark(sn + "snake+transpose")) return rc;
    for (int ri = 0; ri < 3; ri++) {
      const VaeRes& R = st.res[ri];
      ConvArgs c7;
      c7.x = h; c7.w = R.w0; c7.w_bf16 = bf; c7.bias = R.b0; c7.y = r; c7.snake_alpha = R.a0;
      c7.B = B; c7.Cin = st.cout; c7.Cout = st.cout; c7.Tin = t; c7.Tout = t; c7.k = 7;
      c7.dil = dils[ri]; c7.left = 6 * dils[ri]; c7.groups = dw ? st.cout : 1;
      use_tc(v, c7, R.w0_tc);
      CTTS_CK(launch_conv1d(c7, s));
      ConvArgs c1;
      c1.x = r; c1.w = R.w1; c1.w_bf16 = bf; c1.bias = R.b1; c1.y = h; c1.res = h; c1.snake_alpha = R.a1;
      c1.B = B; c1.Cin = st.cout; c1.Cout = st.cout; c1.Tin = t; c1.Tout = t; c1.k = 1; c1.dil = 1;
      c1.left = 0;
      use_tc(v, c1, R.w1_tc);
      CTTS_CK(launch_conv1d(c1, s));
      if (int rc = mark(sn + "resunit d" + std::to_string(dils[ri]))) return rc;
    }
  }
  ConvArgs f;
  f.x = h; f.w = v->final_w; f.w_bf16 = bf; f.bias = v->final_b; f.y = wav; f.snake_alpha = v->final_alpha;
  f.B = B; f.Cin = v->cfg.channels >> v->cfg.n_stages; f.Cout = 1; f.Tin = t; f.Tout = t; f.k = 7;
  f.dil = 1; f.left = 6; f.tanh_out = 1;
  CTTS_CK(launch_conv1d(f, s));
  if (int rc = mark("final snake+conv+tanh")) return rc;
  return CTTS_OK;
}

}  // namespace

extern "C" int ctts_vae_decode_batch_dev(ctts_vae* v, int batch, const float* latent_dev, int T,
                                         float* wav_dev, void* stream) {
  CTTS_REQ(v && latent_dev && wav_dev && batch > 0 && T > 0, CTTS_ERR_ARG, "bad argument");
  if (v->slots.missing()) return set_error(CTTS_ERR_STATE, "VAE weights missing: " + v->slots.first_missing());
  CTTS_CK(cudaSetDevice(v->device));
  int rc = vae_ws_ensure(v, batch, T);
  if (rc) return rc;
  if ((rc = vae_tc_prepare(v))) return rc;
  return vae_enqueue(v, batch, latent_dev, T, wav_dev, as_stream(stream, v->stream));
}

extern "C" int ctts_vae_decode_batch(ctts_vae* v, int batch, const float* latent, int T, float* wav) {
  CTTS_REQ(v && latent && wav && batch > 0 && T > 0, CTTS_ERR_ARG, "bad argument");
  CTTS_CK(cudaSetDevice(v->device));
  const size_t nl = (size_t)batch * v->cfg.latent * T, nw = (size_t)batch * T * v->hop;
  if (nl > v->io_lat || nw > v->io_wav) {
    if (v->lat_dev) cudaFree(v->lat_dev);
    if (v->wav_dev) cudaFree(v->wav_dev);
    v->lat_dev = v->wav_dev = nullptr;
    v->io_lat = v->io_wav = 0;
    CTTS_CK(cudaMalloc(&v->lat_dev, nl * 4));
    CTTS_CK(cudaMalloc(&v->wav_dev, nw * 4));
    v->io_lat = nl;
    v->io_wav = nw;
  }
  CTTS_CK(cudaMemcpyAsync(v->lat_dev, latent, nl * 4, cudaMemcpyHostToDevice, v->stream));
  int rc;
  if (vae_profile_env()) {
    if (v->slots.missing()) return set_error(CTTS_ERR_STATE, "VAE weights missing: " + v->slots.first_missing());
    if ((rc = vae_ws_ensure(v, batch, T))) return rc;
    if ((rc = vae_tc_prepare(v))) return rc;
    VaeProf prof;
    if ((rc = vae_enqueue(v, batch, v->lat_dev, T, v->wav_dev, v->stream, &prof))) return rc;
    CTTS_CK(cudaStreamSynchronize(v->stream));
    prof.report();
  } else {
    rc = ctts_vae_decode_batch_dev(v, batch, v->lat_dev, T, v->wav_dev, v->stream);
    if (rc) return rc;
  }
  CTTS_CK(cudaStreamSynchronize(v->stream));
  if ((rc = vae_read_err(v))) return rc;
  CTTS_CK(cudaMemcpy(wav, v->wav_dev, nw * 4, cudaMemcpyDeviceToHost));
  return CTTS_OK;
}

extern "C" int ctts_op_causal_conv1d(const float* x, int batch, int c_in, int T, const void* w, int w_dtype,
                                     const float* bias, int c_out, int k, int dilation, int groups, int pad,
                                     float* y, void* stream) {
  CTTS_REQ(x && w && y && batch > 0 && c_in > 0 && c_out > 0 && T > 0 && k > 0 && dilation > 0 && pad >= 0,
           CTTS_ERR_ARG, "bad argument");
  CTTS_REQ(w_dtype == CTTS_F32 || w_dtype == CTTS_BF16, CTTS_ERR_ARG, "bad weight dtype");
  CTTS_REQ(groups == 1 || (groups == c_in && c_in == c_out), CTTS_ERR_ARG,
           "groups must be 1 or c_in == c_out (depthwise)");
  ConvArgs a;
  a.x = x; a.w = w; a.w_bf16 = w_dtype == CTTS_BF16; a.bias = bias; a.y = y;
  a.B = batch; a.Cin = c_in; a.Cout = c_out; a.Tin = T; a.Tout = T; a.k = k; a.dil = dilation;
  a.left = 2 * pad; a.groups = groups;
  CTTS_CK(launch_conv1d(a, as_stream(stream, nullptr)));
  return CTTS_OK;
}

// ----------------------------------------------- reference ffi.rs signatures

extern "C" void* cutetts_vae_load(const char* path) {
  if (!path) return nullptr;
  StFile f;
  if (!st_read(path, &f).empty()) return nullptr;
  const std::string pre = "decoder.";
  auto shape_of = [&](const std::string& n) -> std::vector<int64_t> {
    auto it = f.tensors.find(pre + n);
    if (it == f.tensors.end()) return {};
    return it->second.shape;
  };
  ctts_vae_config c{};
  auto wshape = [&](const std::string& n) {
    std::vector<int64_t> r = shape_of(n + ".weight_v");
    return r.empty() ? shape_of(n + ".weight") : r;
  };
  std::vector<int64_t> s0 = wshape("model.0");
  if (s0.size() != 3) return nullptr;
  int base = 1;
  if (s0[1] == 1) {  // depthwise front [latent, 1, 7] + pointwise [channels, latent, 1]
    std::vector<int64_t> s1 = wshape("model.1");
    if (s1.size() != 3 || s1[1] != s0[0] || s1[2] != 1) return nullptr;
    c.depthwise = 1;
    c.latent = (int)s0[0];
    c.channels = (int)s1[0];
    base = 2;
  } else {
    c.channels = (int)s0[0];
    c.latent = (int)s0[1];
  }
  for (int si = 0; si < 8; si++) {
    std::vector<int64_t> st = wshape("model." + std::to_string(base + si) + ".block.1");
    if (st.size() != 3) break;
    c.strides[si] = (int)st[2] / 2;
    c.n_stages = si + 1;
  }
  if (c.n_stages == 0) return nullptr;
  c.weight_dtype = CTTS_F32;
  int dev = 0;
  cudaGetDevice(&dev);
  ctts_vae* v = nullptr;
  if (ctts_vae_create(&c, dev, &v) != CTTS_OK) return nullptr;
  if (ctts_vae_load_file(v, path, pre.c_str()) != CTTS_OK || ctts_vae_missing(v) != 0) {
    ctts_vae_free(v);
    return nullptr;
  }
  return v;
}

extern "C" void cutetts_vae_free(void* handle) { ctts_vae_free(reinterpret_cast<ctts_vae*>(handle)); }

extern "C" int cutetts_vae_decode(void* handle, const float* latent, unsigned long frames, float* wav_out) {
  if (!handle || !latent || !wav_out || frames == 0 || frames > (1ul << 24)) return -1;
  return ctts_vae_decode_batch(reinterpret_cast<ctts_vae*>(handle), 1, latent, (int)frames, wav_out) == CTTS_OK
             ? 0
             : -1;
}
