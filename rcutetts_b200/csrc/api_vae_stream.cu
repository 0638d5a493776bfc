// api_vae_stream.cu -- C ABI: the streaming (chunked) VAE decoder
// (rust-codec/src/stream.rs:62-139 StreamingDecoder::new / reset /
// decode_chunk; modeling/audio_adapter.py:105-232).
//
// Every causal conv keeps its left history explicitly ((k-1)*dilation input
// columns per utterance and channel, zeros at stream start) and each
// transposed conv keeps one past input column.  A chunk runs the same conv
// kernels as the offline decoder on [history ++ chunk] with the history
// columns skipped at the output, so every output sample sees exactly the
// inputs, taps and accumulation order of the offline decode: chunked output
// is bit-identical to decoding the whole utterance at once.  The Snake of a
// conv's input is fused into its operand load, so histories hold the raw
// (pre-Snake) inputs.
#include <algorithm>
#include <vector>

#include "api_common.h"
#include "model.h"

using namespace ctts;

struct ctts_vae_stream {
  ctts_vae* v = nullptr;
  int batch = 0;
  int flip = 0;  // which of the two history buffers holds the current history
  // one history pair per conv with a left context, in decode order: front,
  // then per stage the transposed conv and the three dilated k7 convs, final
  struct Hist {
    int C = 0, H = 0;
    float* buf[2] = {nullptr, nullptr};
  };
  std::vector<Hist> hist;
  DevArena arena;
  // chunk workspace
  int cap_frames = 0;
  DevArena ws;
  float *ext = nullptr, *h = nullptr, *h2 = nullptr, *r = nullptr;
  float *lat_dev = nullptr, *wav_dev = nullptr;
};

namespace {

int stream_ws_ensure(ctts_vae_stream* st, int frames) {
  if (frames <= st->cap_frames) return CTTS_OK;
  ctts_vae* v = st->v;
  const int B = st->batch;
  size_t act = (size_t)std::max(v->cfg.channels, v->cfg.latent) * frames, ext = (size_t)v->cfg.latent * (frames + 6);
  int t = frames;
  ext = std::max(ext, (size_t)v->cfg.channels * (t + 1));
  for (auto& s : v->stages) {
    ext = std::max(ext, (size_t)s.cin * (t + 1));
    t *= s.stride;
    act = std::max(act, (size_t)s.cout * t);
    ext = std::max(ext, (size_t)s.cout * (t + 6 * 9));
  }
  cudaDeviceSynchronize();
  st->ws.~DevArena();
  new (&st->ws) DevArena();
  st->ext = st->ws.alloc<float>(ext * B);
  st->h = st->ws.alloc<float>(act * B);
  st->h2 = st->ws.alloc<float>(act * B);
  st->r = st->ws.alloc<float>(act * B);
  st->lat_dev = st->ws.alloc<float>((size_t)B * v->cfg.latent * frames);
  st->wav_dev = st->ws.alloc<float>((size_t)B * frames * v->hop);
  if (!st->ext || !st->h || !st->h2 || !st->r || !st->lat_dev || !st->wav_dev) {
    st->cap_frames = 0;
    return set_error(CTTS_ERR_NOMEM, "streaming VAE workspace");
  }
  st->cap_frames = frames;
  return CTTS_OK;
}

// One conv over [history ++ x] -> y (T output columns): builds ext, rotates
// the history, launches the conv with the history columns skipped.
int conv_streamed(ctts_vae_stream* st, size_t hi, ConvArgs a, const float* x, int T, cudaStream_t s, bool transpose) {
  ctts_vae_stream::Hist& h = st->hist[hi];
  CTTS_CK(launch_stream_ext(h.buf[st->flip], x, st->ext, h.buf[st->flip ^ 1], st->batch, h.C, h.H, T, s));
  a.x = st->ext;
  a.Tin = h.H + T;
  a.xoff = h.H;
  a.Tout = transpose ? T * a.stride : T;
  if (transpose)
    CTTS_CK(launch_conv_transpose(a, s));
  else
    CTTS_CK(launch_conv1d(a, s));
  return CTTS_OK;
}

int stream_enqueue(ctts_vae_stream* st, const float* lat, int T, float* wav, cudaStream_t s) {
  ctts_vae* v = st->v;
  const int B = st->batch, bf = v->bf16;
  float* h = st->h;
  float* h2 = st->h2;
  float* r = st->r;
  size_t hi = 0;
  int rc;
  const int dw = v->cfg.depthwise;
  {
    ConvArgs a;
    a.w = v->front_w; a.w_bf16 = bf; a.bias = v->front_b; a.y = dw ? r : h;
    a.B = B; a.Cin = v->cfg.latent; a.Cout = dw ? v->cfg.latent : v->cfg.channels; a.k = 7; a.dil = 1; a.left = 6;
    a.groups = dw ? v->cfg.latent : 1;
    if (!dw) use_tc(v, a, v->front_tc);
    if ((rc = conv_streamed(st, hi++, a, lat, T, s, false))) return rc;
  }
  if (dw) {  // pointwise latent -> channels: no context
    ConvArgs p;
    p.x = r; p.w = v->front_pw_w; p.w_bf16 = bf; p.bias = v->front_pw_b; p.y = h;
    p.B = B; p.Cin = v->cfg.latent; p.Cout = v->cfg.channels; p.Tin = T; p.Tout = T; p.k = 1; p.dil = 1; p.left = 0;
    use_tc(v, p, v->front_pw_tc);
    CTTS_CK(launch_conv1d(p, s));
  }
  int t = T;
  static const int dils[3] = {1, 3, 9};
  for (auto& sg : v->stages) {
    ConvArgs tr;
    tr.w = sg.tw; tr.w_bf16 = bf; tr.bias = sg.tb; tr.y = h2; tr.snake_alpha = sg.alpha;
    tr.B = B; tr.Cin = sg.cin; tr.Cout = sg.cout; tr.k = 2; tr.dil = 1; tr.left = 1; tr.stride = sg.stride;
    use_tc(v, tr, sg.tw_tc);
    if ((rc = conv_streamed(st, hi++, tr, h, t, s, true))) return rc;
    t *= sg.stride;
    std::swap(h, h2);
    for (int ri = 0; ri < 3; ri++) {
      const VaeRes& R = sg.res[ri];
      ConvArgs c7;
      c7.w = R.w0; c7.w_bf16 = bf; c7.bias = R.b0; c7.y = r; c7.snake_alpha = R.a0;
      c7.B = B; c7.Cin = sg.cout; c7.Cout = sg.cout; c7.k = 7; c7.dil = dils[ri]; c7.left = 6 * dils[ri];
      c7.groups = dw ? sg.cout : 1;
      use_tc(v, c7, R.w0_tc);
      if ((rc = conv_streamed(st, hi++, c7, h, t, s, false))) return rc;
      ConvArgs c1;  // pointwise: no context
      c1.x = r; c1.w = R.w1; c1.w_bf16 = bf; c1.bias = R.b1; c1.y = h; c1.res = h; c1.snake_alpha = R.a1;
      c1.B = B; c1.Cin = sg.cout; c1.Cout = sg.cout; c1.Tin = t; c1.Tout = t; c1.k = 1; c1.dil = 1; c1.left = 0;
      use_tc(v, c1, R.w1_tc);
      CTTS_CK(launch_conv1d(c1, s));
    }
  }
  ConvArgs f;
  f.w = v->final_w; f.w_bf16 = bf; f.bias = v->final_b; f.y = wav; f.snake_alpha = v->final_alpha;
  f.B = B; f.Cin = v->cfg.channels >> v->cfg.n_stages; f.Cout = 1; f.k = 7; f.dil = 1; f.left = 6;
  f.tanh_out = 1;
  if ((rc = conv_streamed(st, hi++, f, h, t, s, false))) return rc;
  st->flip ^= 1;  // every history advanced into the other buffer
  return CTTS_OK;
}

}  // namespace

extern "C" int ctts_vae_stream_create(ctts_vae* v, int batch, ctts_vae_stream** out) {
  CTTS_REQ(v && out && batch > 0, CTTS_ERR_ARG, "bad argument");
  if (v->slots.missing()) return set_error(CTTS_ERR_STATE, "VAE weights missing: " + v->slots.first_missing());
  CTTS_CK(cudaSetDevice(v->device));
  auto* st = new ctts_vae_stream();
  st->v = v;
  st->batch = batch;
  auto add = [&](int C, int H) {
    ctts_vae_stream::Hist h;
    h.C = C;
    h.H = H;
    h.buf[0] = st->arena.alloc<float>((size_t)batch * C * H);  // zeroed: causal left padding
    h.buf[1] = st->arena.alloc<float>((size_t)batch * C * H);
    st->hist.push_back(h);
    return h.buf[0] && h.buf[1];
  };
  bool ok = add(v->cfg.latent, 6);
  for (auto& sg : v->stages) {
    ok = ok && add(sg.cin, 1);
    for (int d : {1, 3, 9}) ok = ok && add(sg.cout, 6 * d);
  }
  ok = ok && add(v->cfg.channels >> v->cfg.n_stages, 6);
  if (!ok) {
    delete st;
    return set_error(CTTS_ERR_NOMEM, "streaming VAE history allocation failed");
  }
  *out = st;
  return CTTS_OK;
}

extern "C" int ctts_vae_stream_reset(ctts_vae_stream* st) {
  CTTS_REQ(st, CTTS_ERR_ARG, "null stream");
  CTTS_CK(cudaSetDevice(st->v->device));
  for (auto& h : st->hist)
    for (float* b : h.buf) CTTS_CK(cudaMemsetAsync(b, 0, sizeof(float) * st->batch * h.C * h.H, st->v->stream));
  CTTS_CK(cudaStreamSynchronize(st->v->stream));
  st->flip = 0;
  return CTTS_OK;
}

extern "C" int ctts_vae_stream_decode_chunk_dev(ctts_vae_stream* st, const float* latent_dev, int frames,
                                                float* wav_dev, void* stream) {
  CTTS_REQ(st && latent_dev && wav_dev && frames > 0, CTTS_ERR_ARG, "bad argument");
  CTTS_CK(cudaSetDevice(st->v->device));
  int rc = stream_ws_ensure(st, frames);
  if (rc) return rc;
  if ((rc = vae_tc_prepare(st->v))) return rc;
  return stream_enqueue(st, latent_dev, frames, wav_dev, as_stream(stream, st->v->stream));
}

extern "C" int ctts_vae_stream_decode_chunk(ctts_vae_stream* st, const float* latent, int frames, float* wav) {
  CTTS_REQ(st && latent && wav && frames > 0, CTTS_ERR_ARG, "bad argument");
  ctts_vae* v = st->v;
  CTTS_CK(cudaSetDevice(v->device));
  int rc = stream_ws_ensure(st, frames);
  if (rc) return rc;
  const size_t nl = (size_t)st->batch * v->cfg.latent * frames, nw = (size_t)st->batch * frames * v->hop;
  if ((rc = vae_tc_prepare(v))) return rc;
  CTTS_CK(cudaMemcpyAsync(st->lat_dev, latent, nl * 4, cudaMemcpyHostToDevice, v->stream));
  rc = stream_enqueue(st, st->lat_dev, frames, st->wav_dev, v->stream);
  if (rc) return rc;
  CTTS_CK(cudaMemcpyAsync(wav, st->wav_dev, nw * 4, cudaMemcpyDeviceToHost, v->stream));
  CTTS_CK(cudaStreamSynchronize(v->stream));
  if ((rc = vae_read_err(v))) return rc;
  return CTTS_OK;
}

extern "C" void ctts_vae_stream_free(ctts_vae_stream* st) {
  if (!st) return;
  cudaSetDevice(st->v->device);
  cudaDeviceSynchronize();
  delete st;
}
