// api_dit.cu -- C ABI: the DiT flow head (dit.rs / diffusion_head.py) and
// the per-frame engine (bin/cutetts.rs:429-523 loop body) captured as one
// CUDA graph per frame.
#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstring>
#include <cstdlib>

#include "api_common.h"
#include "model.h"

using namespace ctts;

namespace {

// Injected wait fault of the small-batch DiT grid loop (error-path tests;
// ctts_debug_inject_wait_fault), read when a launch is enqueued.
std::atomic<int> g_fault_skip{0};
std::atomic<uint32_t> g_fault_spin_limit{0};

int dit_ws_ensure(ctts_dit* d, DitWs& w, int rows, int steps) {
  if (w.rows >= rows && w.steps >= steps) return CTTS_OK;
  rows = std::max(rows, w.rows);
  steps = std::max(steps, w.steps);
  cudaDeviceSynchronize();
  w.arena.~DevArena();
  new (&w.arena) DevArena();
  const ctts_dit_config& c = d->cfg;
  const int H = c.hidden, P = c.patch, S = 1 + 2 * P, L = c.latent;
  const int qkvw = (c.n_heads + 2 * c.n_kv_heads) * c.head_dim, qd = c.n_heads * c.head_dim;
  w.seq = w.arena.alloc<float>((size_t)rows * S * H);
  w.qkv = w.arena.alloc<float>((size_t)rows * S * qkvw);
  w.att = w.arena.alloc<float>((size_t)rows * S * qd);
  w.act = w.arena.alloc<float>((size_t)rows * S * c.ffn);
  w.mu = w.arena.alloc<float>((size_t)rows * H);
  w.ad = w.arena.alloc<float>((size_t)rows * c.n_layers * 6 * H);
  w.condh = w.arena.alloc<float>((size_t)rows * P * H);
  w.temb = w.arena.alloc<float>((size_t)steps * H);
  w.dtemb = w.arena.alloc<float>(H);
  w.stemb = w.arena.alloc<float>(H);
  w.tmp = w.arena.alloc<float>((size_t)(steps + 2) * H);
  w.se = w.arena.alloc<float>((size_t)(steps + 2) * H);
  w.tv = w.arena.alloc<float>(TGrid::kMax);
  w.x = w.arena.alloc<float>((size_t)rows * P * L);
  w.v = w.arena.alloc<float>((size_t)rows * P * L);
  w.z = w.arena.alloc<float>((size_t)rows * c.cond_dim);
  w.cond = w.arena.alloc<float>((size_t)rows * P * L);
  w.spk = w.arena.alloc<float>((size_t)rows * std::max(c.spk_dim, 1));
  w.hbuf = w.arena.alloc<float>((size_t)2 * H);
  w.err = w.arena.alloc<int>(1);
  w.gbar = w.arena.alloc<unsigned>((size_t)dit_grid_counters(c.n_layers, steps));
  w.gll = w.arena.alloc<unsigned long long>(
      ctts::dit_grid_ll_words(std::min(rows, ctts::DitGridArgs::kMaxRows / 3), H, c.n_heads, c.n_kv_heads, c.head_dim, c.ffn, L));
  if (!w.seq || !w.qkv || !w.att || !w.act || !w.ad || !w.x || !w.spk || !w.hbuf || !w.err || !w.gbar || !w.gll)
    return set_error(CTTS_ERR_NOMEM, "DiT workspace allocation failed");
  if (d->bf16) {
    const int SR = rows * S;
    w.xb = w.arena.alloc<uint16_t>((size_t)SR * std::max(std::max(H, c.spk_dim), c.ffn));
    w.attb = w.arena.alloc<uint16_t>((size_t)SR * qd);
    w.actb = w.arena.alloc<uint16_t>((size_t)SR * c.ffn);
    std::vector<std::array<int, 3>> shapes = {
        {SR, qkvw, H}, {SR, H, qd}, {SR, 2 * c.ffn, H}, {SR, H, c.ffn},
        {rows, c.n_layers * 6 * H, std::max(c.spk_dim, 64)}};
    int rc = tc_alloc(w.arena, &w.tc, shapes, w.err);
    if (rc) return rc;
    if (!w.xb || !w.attb || !w.actb) return set_error(CTTS_ERR_NOMEM, "DiT workspace allocation failed");
  }
  w.rows = rows;
  w.steps = steps;
  return CTTS_OK;
}

struct DitRun {
  int R = 0;                 // rows (utterance-branches)
  const float* z = nullptr;  // [R, cond_dim]
  const float* cond = nullptr;  // [R, P*L]
  const float* spk = nullptr;   // [R, spk_dim] or null (plain residual path)
  int zero_adaln_from = -1;     // rows >= this get zero AdaLN (CFG uncond branch)
  float* x = nullptr;           // latent being integrated [X, P*L]
  int x_rows = 0;               // rows of x (R, or R/2 for CFG where both halves read x)
  int steps = 0;
  const float* times = nullptr;  // host: t per step
  const float* dts = nullptr;    // host: dt per step (Euler / CFG modes)
  int mode = 0;                  // 0 euler, 1 predict (single v -> out), 2 cfg
  float cfg = 0.0f;
  float cfg_w = 0.0f;            // cfg_strength embedding input (distill)
  float step_dt = 0.0f;          // step-size embedding input (distill)
  float* out = nullptr;          // predict: v [R, P*L]
  // the time / delta-time / step-size / cfg-strength embeddings already sit
  // in the workspace from an earlier run with the same grid, dt and
  // strength (the frame engine: constant across frames)
  bool consts_cached = false;
};

// Packs (or, after a weight upload, repacks in place) the cluster loop's
// weights from the layer tensors.  Synchronous: waits for the device first,
// so no launch still reads the buffers being rewritten.
cudaError_t dit_cluster_pack_all(ctts_dit* d, ctts::DitClusterW& W) {
  std::vector<const void*> q, o, g, dn;
  std::vector<const float*> n1, n2;
  for (const DitLayer& L : d->layers) {
    q.push_back(L.wqkv);
    o.push_back(L.wo);
    g.push_back(L.wgu);
    dn.push_back(L.wd);
    n1.push_back(L.norm1);
    n2.push_back(L.norm2);
  }
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess)
    e = ctts::dit_cluster_pack(W, d->cfg.n_layers, q.data(), o.data(), g.data(), dn.data(), n1.data(), n2.data());
  return e;
}

// Brings the packed weights up to date after an upload, unless `s` is
// being captured (the repack is synchronous): returns false then, and the
// run takes the launch chain, which reads the uploaded tensors directly.
bool dit_cluster_fresh(ctts_dit* d, cudaStream_t s) {
  if (d->cl_state != 1) return false;
  if (!d->cl_dirty) return true;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(s, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) {
    (void)cudaGetLastError();
    return false;
  }
  if (dit_cluster_pack_all(d, *d->cl) != cudaSuccess) {
    (void)cudaGetLastError();
    d->cl_state = -1;
    return false;
  }
  d->cl_dirty = false;
  return true;
}

// The cluster-resident Euler loop runs when the head has the shapes it is
// specialised for, the weights are bf16, 16-CTA clusters fit on the GPU,
// CTTS_DIT_CLUSTER is not 0 and no run of it has reported a split-K partial
// outside the fp16 exchange range.  The first call packs the weights
// (synchronous; the engine's first frame runs outside graph capture).
bool dit_cluster_ready(ctts_dit* d, int steps, cudaStream_t s) {
  using Sh = ctts::DitClusterShape;
  const ctts_dit_config& c = d->cfg;
  if (!d->bf16 || c.hidden != Sh::kH || c.ffn != Sh::kF || c.n_heads != Sh::kNH || c.n_kv_heads != Sh::kNH ||
      c.head_dim != Sh::kHD || c.patch != 1 || c.latent != Sh::kL || c.n_layers > Sh::kMaxNL ||
      steps > Sh::kMaxSteps)
    return false;
  if (d->cl_state == 0) {
    d->cl_state = -1;
    const char* env = getenv("CTTS_DIT_CLUSTER");
    if ((!env || atoi(env) != 0) && ctts::dit_cluster_max_active() > 0) {
      auto* W = new ctts::DitClusterW();
      if (dit_cluster_pack_all(d, *W) == cudaSuccess) {
        d->cl = W;
        d->cl_state = 1;
        d->cl_dirty = false;
      } else {
        (void)cudaGetLastError();
        ctts::dit_cluster_free(*W);
        delete W;
      }
    }
  }
  return dit_cluster_fresh(d, s);
}

// Enqueues one DiT sample / predict on stream s with workspace w (sized by
// dit_ws_ensure).  All pointers device.
int dit_enqueue(ctts_dit* d, DitWs& w, const DitRun& r, cudaStream_t s, int* launches) {
  const ctts_dit_config& c = d->cfg;
  const int H = c.hidden, P = c.patch, S = 1 + 2 * P, L = c.latent, PL = P * L;
  const int qd = c.n_heads * c.head_dim, qkvw = qd + 2 * c.n_kv_heads * c.head_dim;
  const int F = c.ffn, R = r.R, NL = c.n_layers;
  const long adld = (long)NL * 6 * H;
  const int bf = d->bf16;
  int nl = 0;
  auto lin = [&](LinearArgs a) -> int {
    a.w_bf16 = bf;
    cudaError_t e = launch_linear(a, s);
    if (e != cudaSuccess) {
      (void)cudaGetLastError();
      return set_error(CTTS_ERR_CUDA, std::string("linear: ") + cudaGetErrorString(e));
    }
    nl++;
    return CTTS_OK;
  };
#define RUN(x)                      \
  do {                              \
    int _rc = (x);                  \
    if (_rc != CTTS_OK) return _rc; \
  } while (0)

  // ---- once per sample (sample_prologue, dit.rs:756-772)
  TGrid g;
  g.n = r.steps + 1 + (d->st1_w ? 1 : 0);
  CTTS_REQ(g.n <= TGrid::kMax, CTTS_ERR_ARG, "too many Euler steps");
  for (int i = 0; i < r.steps; i++) g.t[i] = r.times[i];
  g.t[r.steps] = 0.0f;  // delta_time_mlp input (legacy dt = 0)
  if (d->st1_w) g.t[r.steps + 1] = r.step_dt;
  if (!r.consts_cached) {
    CTTS_CK(launch_fill_tv(w.tv, g, s)); nl++;
    CTTS_CK(launch_sin_emb(w.tv, g.n, H, w.se, s)); nl++;
  }
  if (!r.consts_cached) {
    LinearArgs a; a.x = w.se; a.x_ld = H; a.M = r.steps; a.K = H; a.N = H; a.w = d->t1_w;
    a.bias = d->t1_b; a.act = 1; a.y = w.tmp; a.y_ld = H; RUN(lin(a));
    LinearArgs b; b.x = w.tmp; b.x_ld = H; b.M = r.steps; b.K = H; b.N = H; b.w = d->t2_w;
    b.bias = d->t2_b; b.y = w.temb; b.y_ld = H; RUN(lin(b));
    LinearArgs c1; c1.x = w.se + (size_t)r.steps * H; c1.x_ld = H; c1.M = 1; c1.K = H; c1.N = H;
    c1.w = d->dt1_w; c1.bias = d->dt1_b; c1.act = 1; c1.y = w.tmp + (size_t)r.steps * H; c1.y_ld = H;
    RUN(lin(c1));
    LinearArgs c2; c2.x = w.tmp + (size_t)r.steps * H; c2.x_ld = H; c2.M = 1; c2.K = H; c2.N = H;
    c2.w = d->dt2_w; c2.bias = d->dt2_b; c2.y = w.dtemb; c2.y_ld = H; RUN(lin(c2));
  }
  // mu = mu_proj(z) (+ cfg_strength) (+ step_size)   diffusion_head.py:601-627
  // (bf16 weights with >= 16 rows: on the tensor cores)
  bool xb_holds_z = false;  // w.xb = bf16(z) rows [0, R)
  if (d->mu_w && bf && R >= 16 && c.cond_dim % 64 == 0) {
    PrepArgs pa; pa.x = r.z; pa.x_ld = c.cond_dim; pa.y = w.xb; pa.y_ld = c.cond_dim; pa.M = R; pa.K = c.cond_dim;
    CTTS_CK(launch_prep_bf16(pa, s)); nl++;
    xb_holds_z = true;
    TcArgs e; e.y = w.mu; e.y_ld = H; e.bias = d->mu_b;
    RUN(tc_run(w.tc, w.xb, R, c.cond_dim, d->mu_w, H, e, s, &nl));
  } else if (d->mu_w) {
    LinearArgs a; a.x = r.z; a.x_ld = c.cond_dim; a.M = R; a.K = c.cond_dim; a.N = H; a.w = d->mu_w;
    a.bias = d->mu_b; a.y = w.mu; a.y_ld = H; RUN(lin(a));
  } else {
    CTTS_CK(cudaMemcpyAsync(w.mu, r.z, sizeof(float) * R * H, cudaMemcpyDeviceToDevice, s));
  }
  if (d->cfg2_w) {
    // silu(cfg0 * cfg_w/5) on the host (a [H,1] x scalar product), then cfg2.
    if (!r.consts_cached) {
      LinearArgs a; a.x = w.hbuf; a.x_ld = H; a.M = 1; a.K = H; a.N = H; a.w = d->cfg2_w;
      a.y = w.hbuf + H; a.y_ld = H; RUN(lin(a));
    }
    CTTS_CK(launch_add_rows(w.mu, R, H, w.hbuf + H, s)); nl++;
  }
  if (d->st1_w) {
    if (!r.consts_cached) {
      LinearArgs a; a.x = w.se + (size_t)(r.steps + 1) * H; a.x_ld = H; a.M = 1; a.K = H; a.N = H;
      a.w = d->st1_w; a.bias = d->st1_b; a.act = 1; a.y = w.tmp + (size_t)(r.steps + 1) * H; a.y_ld = H;
      RUN(lin(a));
      LinearArgs b; b.x = w.tmp + (size_t)(r.steps + 1) * H; b.x_ld = H; b.M = 1; b.K = H; b.N = H;
      b.w = d->st2_w; b.bias = d->st2_b; b.y = w.stemb; b.y_ld = H; RUN(lin(b));
    }
    CTTS_CK(launch_add_rows(w.mu, R, H, w.stemb, s)); nl++;
  }
  const bool use_ad = c.adaln && r.spk;
  // bf16 weights with >= 16 rows: the tensor-core linears (tc_linear.cu)
  const bool tc = bf && R * S >= 16;
  if (use_ad) {
    int rows = r.zero_adaln_from >= 0 ? r.zero_adaln_from : R;
    if (bf && rows >= 16 && c.spk_dim % 64 == 0) {
      // AdaLN conditioned on the LM state itself: its bf16 rows are already
      // the mu_proj operand
      if (!(xb_holds_z && r.spk == r.z && c.spk_dim == c.cond_dim)) {
        PrepArgs pa; pa.x = r.spk; pa.x_ld = c.spk_dim; pa.y = w.xb; pa.y_ld = c.spk_dim; pa.M = rows;
        pa.K = c.spk_dim;
        CTTS_CK(launch_prep_bf16(pa, s)); nl++;
      }
      TcArgs e; e.y = w.ad; e.y_ld = adld;
      RUN(tc_run(w.tc, w.xb, rows, c.spk_dim, d->adaln, (int)adld, e, s, &nl));
    } else {
      LinearArgs a; a.x = r.spk; a.x_ld = c.spk_dim; a.M = rows; a.K = c.spk_dim; a.N = (int)adld;
      a.w = d->adaln; a.y = w.ad; a.y_ld = adld; RUN(lin(a));
    }
    if (rows < R) CTTS_CK(cudaMemsetAsync(w.ad + (size_t)rows * adld, 0, sizeof(float) * (R - rows) * adld, s));
  }
  // cond_proj(cond) rows [R*P, L]: tensor cores for a long contraction; the
  // latent-sized one (L <= 128) on the short-contraction CUDA-core linear
  if (bf && R * P >= 16 && L % 64 == 0 && L > 128) {
    PrepArgs pa; pa.x = r.cond; pa.x_ld = L; pa.y = w.xb; pa.y_ld = L; pa.M = R * P; pa.K = L;
    CTTS_CK(launch_prep_bf16(pa, s)); nl++;
    TcArgs e; e.y = w.condh; e.y_ld = H; e.bias = d->cond_b;
    RUN(tc_run(w.tc, w.xb, R * P, L, d->cond_w, H, e, s, &nl));
  } else {
    LinearArgs a; a.x = r.cond; a.x_ld = L; a.M = R * P; a.K = L; a.N = H; a.w = d->cond_w;
    a.bias = d->cond_b; a.y = w.condh; a.y_ld = H; RUN(lin(a));
  }

  // ---- Euler steps (predict_cached, dit.rs:775-814)
  // small batches with fp32 weights: the whole loop as one grid-persistent
  // launch (dit_grid.cu) unless CTTS_DIT_GRID=0
  const char* grid_e = getenv("CTTS_DIT_GRID");
  const int grid_env = grid_e ? atoi(grid_e) : 1;
  if (r.mode == 0 && r.x_rows == R && !bf && P == 1 && grid_env != 0 &&
      ctts::dit_grid_supported(R, NL, r.steps, H, c.n_heads, c.n_kv_heads, c.head_dim, F, L)) {
    ctts::DitGridArgs ga;
    ga.R = R; ga.NL = NL; ga.steps = r.steps; ga.H = H; ga.nq = c.n_heads; ga.nkv = c.n_kv_heads;
    ga.hd = c.head_dim; ga.F = F; ga.L = L; ga.eps = c.rms_eps;
    for (int i = 0; i < r.steps; i++) ga.dts[i] = r.dts[i];
    ga.x = r.x;
    ga.mu = w.mu; ga.temb = w.temb; ga.dtemb = w.dtemb; ga.condh = w.condh; ga.ad = use_ad ? w.ad : nullptr;
    ga.inv_freq = d->inv_freq; ga.final_norm = d->final_norm;
    ga.in_w = static_cast<const float*>(d->in_w); ga.in_b = d->in_b;
    ga.out_w = static_cast<const float*>(d->out_w); ga.out_b = d->out_b;
    for (int l = 0; l < NL; l++) {
      const DitLayer& Ly = d->layers[l];
      ga.wqkv[l] = static_cast<const float*>(Ly.wqkv); ga.wo[l] = static_cast<const float*>(Ly.wo);
      ga.wgu[l] = static_cast<const float*>(Ly.wgu); ga.wd[l] = static_cast<const float*>(Ly.wd);
      ga.norm1[l] = Ly.norm1; ga.norm2[l] = Ly.norm2;
    }
    ga.bar = w.gbar; ga.ll = w.gll; ga.err = w.err;
    ga.skip_qkv_cta0 = g_fault_skip.load(std::memory_order_relaxed);
    ga.spin_limit = g_fault_spin_limit.load(std::memory_order_relaxed);
    CTTS_CK(ctts::launch_dit_grid(ga, s)); nl++;
    if (launches) *launches += nl;
    return CTTS_OK;
  }
  if (r.mode == 0 && r.x_rows == R && dit_cluster_ready(d, r.steps, s)) {
    ctts::DitClusterArgs ca;
    ca.R = R; ca.NL = NL; ca.steps = r.steps; ca.adaln = use_ad ? 1 : 0; ca.eps = c.rms_eps;
    for (int i = 0; i < r.steps; i++) ca.dts[i] = r.dts[i];
    ca.x = r.x; ca.mu = w.mu; ca.temb = w.temb; ca.dtemb = w.dtemb; ca.condh = w.condh;
    ca.ad = use_ad ? w.ad : nullptr; ca.norms = d->cl->norms; ca.fnorm = d->final_norm;
    ca.out_w = static_cast<const uint16_t*>(d->out_w); ca.out_b = d->out_b;
    ca.in_w = static_cast<const uint16_t*>(d->in_w); ca.in_b = d->in_b; ca.inv_freq = d->inv_freq;
    ca.err = w.err;
    CTTS_CK(ctts::launch_dit_cluster(*d->cl, ca, s)); nl++;
    if (launches) *launches += nl;
    return CTTS_OK;
  }
  const int xrows = r.x_rows;
  // Euler mode: the step tail (final norm, out_proj, x += dt*v) and the
  // next step's head (in_proj, seq fill) run as one kernel per utterance.
  const bool fused_tail = r.mode == 0 && H % 8 == 0 && L % 8 == 0 && H <= 1024 && L <= 64;
  DitTailArgs ta;
  ta.seq = w.seq; ta.x = r.x; ta.R = R; ta.P = P; ta.H = H; ta.L = L;
  ta.out_w = d->out_w; ta.out_b = d->out_b; ta.in_w = d->in_w; ta.in_b = d->in_b; ta.w_bf16 = bf;
  ta.final_norm = d->final_norm; ta.eps = c.rms_eps;
  ta.mu = w.mu; ta.dtemb = w.dtemb; ta.condh = w.condh;
  if (fused_tail) {
    DitTailArgs t0 = ta;
    t0.do_out = 0; t0.fill = 1; t0.temb = w.temb;
    CTTS_CK(launch_dit_tail(t0, s)); nl++;
  }
  for (int st = 0; st < r.steps; st++) {
    if (!fused_tail) {  // in_proj(x) -> seq rows 1+P.. ; rows of x repeat for CFG's second half
      LinearArgs a; a.x = r.x; a.x_ld = L; a.x_div = xrows * P; a.x_ld_outer = 0;
      a.M = R * P; a.K = L; a.N = H; a.w = d->in_w; a.bias = d->in_b;
      a.y = w.seq + (size_t)(1 + P) * H; a.y_ld = H; a.y_div = P; a.y_ld_outer = (long)S * H;
      RUN(lin(a));
      CTTS_CK(launch_dit_seq_fill(w.seq, w.mu, w.temb + (size_t)st * H, w.dtemb, w.condh, R, P, H, s)); nl++;
    }
    for (int l = 0; l < NL; l++) {
      const DitLayer& Ly = d->layers[l];
      const float* ad = use_ad ? w.ad + (size_t)l * 6 * H : nullptr;
      if (tc) {
        const int SR = R * S;
        PrepArgs pq; pq.x = w.seq; pq.x_ld = H; pq.y = w.xb; pq.y_ld = H; pq.M = SR; pq.K = H;
        pq.norm_w = Ly.norm1; pq.eps = c.rms_eps;
        if (ad) { pq.mod = ad; pq.mod_ld = adld; pq.mod_div = S; pq.mod_shift = 0; pq.mod_scale = H; }
        CTTS_CK(launch_prep_bf16(pq, s)); nl++;
        TcArgs eq; eq.y = w.qkv; eq.y_ld = qkvw;
        RUN(tc_run(w.tc, w.xb, SR, H, Ly.wqkv, qkvw, eq, s, &nl));
        CTTS_CK(launch_dit_attn(w.qkv, R, S, c.n_heads, c.n_kv_heads, c.head_dim, d->inv_freq, nullptr,
                                w.attb, s)); nl++;
        TcArgs eo; eo.y = w.seq; eo.y_ld = H; eo.res = w.seq;
        if (ad) { eo.gate = ad; eo.gate_ld = adld; eo.gate_div = S; eo.gate_off = 2 * H; }
        RUN(tc_run(w.tc, w.attb, SR, qd, Ly.wo, H, eo, s, &nl));
        PrepArgs pg; pg.x = w.seq; pg.x_ld = H; pg.y = w.xb; pg.y_ld = H; pg.M = SR; pg.K = H;
        pg.norm_w = Ly.norm2; pg.eps = c.rms_eps;
        if (ad) { pg.mod = ad; pg.mod_ld = adld; pg.mod_div = S; pg.mod_shift = 3 * H; pg.mod_scale = 4 * H; }
        CTTS_CK(launch_prep_bf16(pg, s)); nl++;
        TcArgs eg; eg.act = 2; eg.yb = w.actb; eg.y_ld = F;
        RUN(tc_run(w.tc, w.xb, SR, H, Ly.wgu, 2 * F, eg, s, &nl));
        TcArgs ed; ed.y = w.seq; ed.y_ld = H; ed.res = w.seq;
        if (ad) { ed.gate = ad; ed.gate_ld = adld; ed.gate_div = S; ed.gate_off = 5 * H; }
        RUN(tc_run(w.tc, w.actb, SR, F, Ly.wd, H, ed, s, &nl));
        continue;
      }
      LinearArgs q; q.x = w.seq; q.x_ld = H; q.M = R * S; q.K = H; q.N = qkvw; q.w = Ly.wqkv;
      q.y = w.qkv; q.y_ld = qkvw; q.norm_w = Ly.norm1; q.eps = c.rms_eps;
      if (ad) { q.mod = ad; q.mod_ld = adld; q.mod_div = S; q.mod_shift = 0; q.mod_scale = H; }
      RUN(lin(q));
      CTTS_CK(launch_dit_attn(w.qkv, R, S, c.n_heads, c.n_kv_heads, c.head_dim, d->inv_freq, w.att, nullptr,
                              s)); nl++;
      LinearArgs o; o.x = w.att; o.x_ld = qd; o.M = R * S; o.K = qd; o.N = H; o.w = Ly.wo;
      o.y = w.seq; o.y_ld = H; o.res = w.seq;
      if (ad) { o.gate = ad; o.gate_ld = adld; o.gate_div = S; o.gate_off = 2 * H; }
      RUN(lin(o));
      LinearArgs gu; gu.x = w.seq; gu.x_ld = H; gu.M = R * S; gu.K = H; gu.N = F; gu.w = Ly.wgu;
      gu.y = w.act; gu.y_ld = F; gu.act = 2; gu.norm_w = Ly.norm2; gu.eps = c.rms_eps;
      if (ad) { gu.mod = ad; gu.mod_ld = adld; gu.mod_div = S; gu.mod_shift = 3 * H; gu.mod_scale = 4 * H; }
      RUN(lin(gu));
      LinearArgs dn; dn.x = w.act; dn.x_ld = F; dn.M = R * S; dn.K = F; dn.N = H; dn.w = Ly.wd;
      dn.y = w.seq; dn.y_ld = H; dn.res = w.seq;
      if (ad) { dn.gate = ad; dn.gate_ld = adld; dn.gate_div = S; dn.gate_off = 5 * H; }
      RUN(lin(dn));
    }
    if (fused_tail) {
      DitTailArgs tt = ta;
      tt.do_out = 1; tt.dt = r.dts[st];
      tt.fill = st + 1 < r.steps;
      tt.temb = w.temb + (size_t)(st + 1 < r.steps ? st + 1 : st) * H;
      CTTS_CK(launch_dit_tail(tt, s)); nl++;
      continue;
    }
    // final norm + out_proj on the x rows (+ Euler update)
    LinearArgs f; f.x = w.seq + (size_t)(1 + P) * H; f.x_ld = H; f.x_div = P; f.x_ld_outer = (long)S * H;
    f.M = R * P; f.K = H; f.N = L; f.w = d->out_w; f.bias = d->out_b; f.norm_w = d->final_norm;
    f.eps = c.rms_eps;
    const float dt = r.mode == 1 ? 0.0f : r.dts[st];
    if (r.mode == 0) {
      f.y = r.x; f.y_ld = L; f.res = r.x; f.scale = dt;
      RUN(lin(f));
    } else if (r.mode == 1) {
      f.y = r.out; f.y_ld = L;
      RUN(lin(f));
    } else {
      f.y = w.v; f.y_ld = L;
      RUN(lin(f));
      CTTS_CK(launch_cfg_euler(r.x, w.v, xrows * PL, r.cfg, dt, s)); nl++;
    }
  }
#undef RUN
  if (launches) *launches += nl;
  return CTTS_OK;
}

// A run of the cluster loop reported a split-K partial outside the fp16
// exchange range (its output is invalid): later runs of this head take the
// fp32-partial launch chain.
int dit_cluster_range_error(ctts_dit* d) {
  d->cl_state = -1;
  return set_error(CTTS_ERR_RANGE,
                   "a DiT split-K partial exceeded the fp16 exchange range (or an input was not finite): the "
                   "run's output is invalid, and this head now runs the fp32-partial launch chain");
}

// Reads back the workspace's device error flag after a synchronized run;
// a reported error is cleared, so the next run starts clean.
int dit_read_err(ctts_dit* d, const DitWs& w) {
  int err = 0;
  CTTS_CK(cudaMemcpy(&err, w.err, sizeof(int), cudaMemcpyDeviceToHost));
  if (err != 0) CTTS_CK(cudaMemset(w.err, 0, sizeof(int)));
  if (err == ctts::kDitClusterErrRange) return dit_cluster_range_error(d);
  CTTS_REQ(err == 0, CTTS_ERR_TIMEOUT, "a DiT kernel gave up waiting on its pipeline, grid barrier or exchange words");
  return CTTS_OK;
}

int dit_check(ctts_dit* d) {
  CTTS_REQ(d, CTTS_ERR_ARG, "null handle");
  if (d->slots.missing())
    return set_error(CTTS_ERR_STATE, "DiT weights missing: " + d->slots.first_missing());
  return CTTS_OK;
}

// host-side cfg-strength hidden: silu(cfg0[:,0] * cfg_w / 5) (dit.rs:657-662)
// into the first H floats of `hbuf` (a workspace's hbuf)
int dit_upload_cfg_hidden(ctts_dit* d, float* hbuf, float cfg_w, cudaStream_t s) {
  if (!d->cfg2_w) return CTTS_OK;
  const int H = d->cfg.hidden;
  std::vector<float> w0(H), h(H);
  CTTS_CK(cudaMemcpy(w0.data(), d->cfg0_w, H * 4, cudaMemcpyDeviceToHost));
  const float wn = cfg_w / 5.0f;
  for (int i = 0; i < H; i++) {
    float v = fmaf(w0[i], wn, 0.0f);
    h[i] = v / (1.0f + expf(-v));
  }
  CTTS_CK(cudaMemcpyAsync(hbuf, h.data(), H * 4, cudaMemcpyHostToDevice, s));
  CTTS_CK(cudaStreamSynchronize(s));
  return CTTS_OK;
}

}  // namespace

// ----------------------------------------------------------------- create

extern "C" int ctts_dit_create(const ctts_dit_config* cfg, int device, ctts_dit** out) {
  CTTS_REQ(cfg && out, CTTS_ERR_ARG, "null argument");
  const ctts_dit_config& c = *cfg;
  CTTS_REQ(c.latent > 0 && c.hidden > 0 && c.n_heads > 0 && c.n_kv_heads > 0 && c.head_dim > 0 &&
               c.ffn > 0 && c.n_layers > 0 && c.patch > 0 && c.cond_dim > 0,
           CTTS_ERR_ARG, "non-positive dimension");
  CTTS_REQ(1 + 2 * c.patch <= 5, CTTS_ERR_ARG, "patch must be 1 or 2");
  CTTS_REQ(c.n_heads % c.n_kv_heads == 0, CTTS_ERR_ARG, "n_heads % n_kv_heads != 0");
  CTTS_REQ(c.head_dim % 64 == 0 && c.head_dim <= 128, CTTS_ERR_ARG, "head_dim must be 64 or 128");
  CTTS_REQ(c.hidden % 64 == 0 && c.ffn % 64 == 0 && c.latent % 8 == 0 && c.cond_dim % 8 == 0 &&
               (!c.adaln || c.spk_dim % 8 == 0),
           CTTS_ERR_ARG, "hidden/ffn must be multiples of 64, latent/cond/spk of 8");
  CTTS_REQ(c.weight_dtype == CTTS_F32 || c.weight_dtype == CTTS_BF16, CTTS_ERR_ARG, "bad weight dtype");
  CTTS_CK(cudaSetDevice(device));
  auto* d = new ctts_dit();
  d->cfg = c;
  d->device = device;
  d->bf16 = c.weight_dtype == CTTS_BF16;
  d->slots.model_bf16 = d->bf16;
  cudaStreamCreateWithFlags(&d->stream, cudaStreamNonBlocking);
  const int H = c.hidden, L = c.latent, F = c.ffn, hd = c.head_dim;
  const int qd = c.n_heads * hd, kvd = c.n_kv_heads * hd;
  const size_t es = d->bf16 ? 2 : 4;
  DevArena& A = d->arena;
  auto W = [&](size_t n) -> void* { return A.alloc<uint8_t>(n * es); };
  auto lin = [&](const std::string& name, void** w, float** b, int o, int i, bool bias, bool opt) {
    *w = W((size_t)o * i);
    d->slots.add(name + ".weight", *w, {o, i}, true, opt);
    if (bias) {
      *b = A.alloc<float>(o);
      d->slots.add(name + ".bias", *b, {o}, false, opt);
    }
  };
  lin("in_proj", &d->in_w, &d->in_b, H, L, true, false);
  lin("cond_proj", &d->cond_w, &d->cond_b, H, L, true, false);
  if (c.cond_dim != H) lin("mu_proj", &d->mu_w, &d->mu_b, H, c.cond_dim, true, false);
  lin("out_proj", &d->out_w, &d->out_b, L, H, true, false);
  lin("time_mlp.linear_1", &d->t1_w, &d->t1_b, H, H, true, false);
  lin("time_mlp.linear_2", &d->t2_w, &d->t2_b, H, H, true, false);
  lin("delta_time_mlp.linear_1", &d->dt1_w, &d->dt1_b, H, H, true, false);
  lin("delta_time_mlp.linear_2", &d->dt2_w, &d->dt2_b, H, H, true, false);
  if (c.step_emb) {
    lin("step_size_embedding.linear_1", &d->st1_w, &d->st1_b, H, H, true, false);
    lin("step_size_embedding.linear_2", &d->st2_w, &d->st2_b, H, H, true, false);
  }
  if (c.cfg_emb) {
    d->cfg0_w = A.alloc<float>(H);
    d->slots.add("cfg_strength_embedding.0.weight", d->cfg0_w, {H, 1}, false);
    d->cfg2_w = W((size_t)H * H);
    d->slots.add("cfg_strength_embedding.2.weight", d->cfg2_w, {H, H}, true);
  }
  if (c.adaln) d->adaln = W((size_t)c.n_layers * 6 * H * c.spk_dim);
  d->layers.resize(c.n_layers);
  for (int i = 0; i < c.n_layers; i++) {
    DitLayer& Ly = d->layers[i];
    std::string p = "decoder.layers." + std::to_string(i) + ".";
    Ly.norm1 = A.alloc<float>(H);
    Ly.norm2 = A.alloc<float>(H);
    Ly.wqkv = W((size_t)(qd + 2 * kvd) * H);
    Ly.wo = W((size_t)H * qd);
    Ly.wgu = W((size_t)2 * F * H);
    Ly.wd = W((size_t)H * F);
    char* qkv = reinterpret_cast<char*>(Ly.wqkv);
    char* gu = reinterpret_cast<char*>(Ly.wgu);
    d->slots.add(p + "input_layernorm.weight", Ly.norm1, {H}, false);
    d->slots.add(p + "post_attention_layernorm.weight", Ly.norm2, {H}, false);
    d->slots.add(p + "self_attn.q_proj.weight", qkv, {qd, H}, true);
    d->slots.add(p + "self_attn.k_proj.weight", qkv + (size_t)qd * H * es, {kvd, H}, true);
    d->slots.add(p + "self_attn.v_proj.weight", qkv + (size_t)(qd + kvd) * H * es, {kvd, H}, true);
    d->slots.add(p + "self_attn.o_proj.weight", Ly.wo, {H, qd}, true);
    d->slots.add(p + "mlp.gate_proj.weight", gu, {F, H}, true);
    d->slots.add(p + "mlp.up_proj.weight", gu + (size_t)64 * H * es, {F, H}, true);
    for (const char* nm : {"mlp.gate_proj.weight", "mlp.up_proj.weight"}) {
      Slot& sl = d->slots.slots[p + nm];
      sl.transform = kXformRowInterleave;
      sl.t_b = H;
    }
    d->slots.add(p + "mlp.down_proj.weight", Ly.wd, {H, F}, true);
    if (c.adaln)
      d->slots.add(p + "speaker_adaln.weight",
                   reinterpret_cast<char*>(d->adaln) + (size_t)i * 6 * H * c.spk_dim * es,
                   {6 * H, c.spk_dim}, true);
  }
  d->final_norm = A.alloc<float>(H);
  d->slots.add("decoder.norm.weight", d->final_norm, {H}, false);
  std::vector<float> inv = rope_inv_freq(hd, c.rope_theta);
  d->inv_freq = A.alloc<float>(hd / 2);
  if (!d->final_norm || !d->inv_freq ||
      cudaMemcpy(d->inv_freq, inv.data(), inv.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaStreamSynchronize(cudaStreamLegacy) != cudaSuccess) {
    delete d;
    return set_error(CTTS_ERR_NOMEM, "device allocation failed");
  }
  *out = d;
  return CTTS_OK;
}

extern "C" int ctts_dit_set_tensor(ctts_dit* d, const char* name, const void* host, int dtype,
                                   const int64_t* shape, int ndim) {
  CTTS_REQ(d, CTTS_ERR_ARG, "null handle");
  CTTS_CK(cudaSetDevice(d->device));
  const int rc = slot_set(d->slots, name, host, dtype, shape, ndim);
  // the cluster loop's packed copy is rebuilt before its next run
  if (rc == CTTS_OK && d->cl) d->cl_dirty = true;
  return rc;
}

extern "C" int ctts_dit_load(ctts_dit* d, const char* path, const char* prefix) {
  CTTS_REQ(d, CTTS_ERR_ARG, "null handle");
  return load_safetensors(path, prefix, [&](const char* n, const void* p, int dt, const int64_t* s, int nd) {
    return ctts_dit_set_tensor(d, n, p, dt, s, nd);
  });
}

extern "C" int ctts_dit_missing(const ctts_dit* d) { return d ? d->slots.missing() : -1; }

extern "C" void ctts_dit_free(ctts_dit* d) {
  if (!d) return;
  cudaSetDevice(d->device);
  cudaStreamSynchronize(d->stream);
  cudaStreamDestroy(d->stream);
  if (d->cl) {
    cudaDeviceSynchronize();
    ctts::dit_cluster_free(*d->cl);
    delete d->cl;
  }
  delete d;
}

extern "C" int ctts_sway_timesteps(int steps, float coeff, float* out) {
  CTTS_REQ(steps > 0 && out, CTTS_ERR_ARG, "bad argument");
  const float ub = 2.0f / (3.14159265358979f - 2.0f);
  CTTS_REQ(coeff >= -1.0f && coeff <= ub, CTTS_ERR_ARG, "sway coefficient outside [-1, 2/(pi-2)]");
  for (int s = 0; s <= steps; s++) {
    float u = (float)s / (float)steps;
    out[s] = u + coeff * (cosf(0.5f * 3.14159265358979f * u) - 1.0f + u);
  }
  return CTTS_OK;
}

// ------------------------------------------------------------- sampling

namespace {

// host -> device, ordered before the kernels later enqueued on `s`
int copy_in(float* dst, const float* src, size_t n, cudaStream_t s) {
  CTTS_CK(cudaMemcpyAsync(dst, src, n * 4, cudaMemcpyHostToDevice, s));
  return CTTS_OK;
}

}  // namespace

extern "C" int ctts_dit_euler_sample_dev(ctts_dit* d, int batch, const float* x0_dev, const float* z_dev,
                                         const float* cond_dev, const float* spk_dev, int steps,
                                         float cfg_w, float* x_out_dev, void* stream) {
  int rc = dit_check(d);
  if (rc) return rc;
  CTTS_REQ(batch > 0 && steps > 0 && x0_dev && z_dev && cond_dev && x_out_dev, CTTS_ERR_ARG, "bad argument");
  CTTS_CK(cudaSetDevice(d->device));
  rc = dit_ws_ensure(d, d->ws, batch, steps);
  if (rc) return rc;
  cudaStream_t s = as_stream(stream, d->stream);
  rc = dit_upload_cfg_hidden(d, d->ws.hbuf, cfg_w, s);
  if (rc) return rc;
  const int PL = d->cfg.patch * d->cfg.latent;
  if (x_out_dev != x0_dev)
    CTTS_CK(cudaMemcpyAsync(x_out_dev, x0_dev, sizeof(float) * batch * PL, cudaMemcpyDeviceToDevice, s));
  // euler_sample (dit.rs:819-842): t_s = s*dt, x += v*dt, dt = 1/steps
  std::vector<float> times(steps), dts(steps);
  const float dt = 1.0f / (float)steps;
  for (int i = 0; i < steps; i++) {
    times[i] = (float)i * dt;
    dts[i] = dt;
  }
  DitRun r;
  r.R = batch; r.z = z_dev; r.cond = cond_dev; r.spk = spk_dev; r.x = x_out_dev; r.x_rows = batch;
  r.steps = steps; r.times = times.data(); r.dts = dts.data(); r.mode = 0; r.cfg_w = cfg_w;
  r.step_dt = dt;
  return dit_enqueue(d, d->ws, r, s, nullptr);
}

extern "C" int ctts_dit_euler_sample(ctts_dit* d, int batch, const float* x0, const float* z,
                                     const float* cond, const float* spk, int steps, float cfg_w,
                                     float* x_out) {
  int rc = dit_check(d);
  if (rc) return rc;
  CTTS_REQ(batch > 0 && steps > 0 && x0 && z && cond && x_out, CTTS_ERR_ARG, "bad argument");
  CTTS_CK(cudaSetDevice(d->device));
  rc = dit_ws_ensure(d, d->ws, batch, steps);
  if (rc) return rc;
  DitWs& w = d->ws;
  const int PL = d->cfg.patch * d->cfg.latent;
  if ((rc = copy_in(w.z, z, (size_t)batch * d->cfg.cond_dim, d->stream))) return rc;
  if ((rc = copy_in(w.cond, cond, (size_t)batch * PL, d->stream))) return rc;
  if (spk && (rc = copy_in(w.spk, spk, (size_t)batch * d->cfg.spk_dim, d->stream))) return rc;
  for (int attempt = 0;; attempt++) {
    if ((rc = copy_in(w.x, x0, (size_t)batch * PL, d->stream))) return rc;
    rc = ctts_dit_euler_sample_dev(d, batch, w.x, w.z, w.cond, spk ? w.spk : nullptr, steps, cfg_w, w.x,
                                   d->stream);
    if (rc) return rc;
    CTTS_CK(cudaStreamSynchronize(d->stream));
    rc = dit_read_err(d, w);
    // the cluster loop gave up on the fp16 partials and is now off: the
    // rerun takes the fp32-partial launch chain
    if (rc == CTTS_ERR_RANGE && attempt == 0) continue;
    if (rc) return rc;
    break;
  }
  CTTS_CK(cudaMemcpy(x_out, w.x, sizeof(float) * batch * PL, cudaMemcpyDeviceToHost));
  return CTTS_OK;
}

extern "C" int ctts_dit_predict(ctts_dit* d, int batch, const float* x, float t, const float* z,
                                const float* cond, float dt, const float* spk, float cfg_w, float* v) {
  int rc = dit_check(d);
  if (rc) return rc;
  CTTS_REQ(batch > 0 && x && z && cond && v, CTTS_ERR_ARG, "bad argument");
  CTTS_CK(cudaSetDevice(d->device));
  rc = dit_ws_ensure(d, d->ws, batch, 1);
  if (rc) return rc;
  DitWs& w = d->ws;
  const int PL = d->cfg.patch * d->cfg.latent;
  if ((rc = copy_in(w.x, x, (size_t)batch * PL, d->stream))) return rc;
  if ((rc = copy_in(w.z, z, (size_t)batch * d->cfg.cond_dim, d->stream))) return rc;
  if ((rc = copy_in(w.cond, cond, (size_t)batch * PL, d->stream))) return rc;
  if (spk && (rc = copy_in(w.spk, spk, (size_t)batch * d->cfg.spk_dim, d->stream))) return rc;
  rc = dit_upload_cfg_hidden(d, d->ws.hbuf, cfg_w, d->stream);
  if (rc) return rc;
  float times[1] = {t};
  DitRun r;
  r.R = batch; r.z = w.z; r.cond = w.cond; r.spk = spk ? w.spk : nullptr; r.x = w.x; r.x_rows = batch;
  r.steps = 1; r.times = times; r.mode = 1; r.out = w.v; r.cfg_w = cfg_w; r.step_dt = dt;
  rc = dit_enqueue(d, d->ws, r, d->stream, nullptr);
  if (rc) return rc;
  CTTS_CK(cudaStreamSynchronize(d->stream));
  if ((rc = dit_read_err(d, w))) return rc;
  CTTS_CK(cudaMemcpy(v, w.v, sizeof(float) * batch * PL, cudaMemcpyDeviceToHost));
  return CTTS_OK;
}

extern "C" int ctts_dit_euler_sample_cfg(ctts_dit* d, int batch, const float* x0, const float* z_c,
                                         const float* z_u, const float* cond, const float* uncond,
                                         const float* spk, int steps, float coeff, float cfg,
                                         float* x_out) {
  int rc = dit_check(d);
  if (rc) return rc;
  CTTS_REQ(batch > 0 && steps > 0 && x0 && z_c && z_u && cond && uncond && x_out, CTTS_ERR_ARG,
           "bad argument");
  CTTS_CK(cudaSetDevice(d->device));
  rc = dit_ws_ensure(d, d->ws, 2 * batch, steps);
  if (rc) return rc;
  DitWs& w = d->ws;
  const int PL = d->cfg.patch * d->cfg.latent, CD = d->cfg.cond_dim;
  if ((rc = copy_in(w.x, x0, (size_t)batch * PL, d->stream))) return rc;
  if ((rc = copy_in(w.z, z_c, (size_t)batch * CD, d->stream))) return rc;
  if ((rc = copy_in(w.z + (size_t)batch * CD, z_u, (size_t)batch * CD, d->stream))) return rc;
  if ((rc = copy_in(w.cond, cond, (size_t)batch * PL, d->stream))) return rc;
  if ((rc = copy_in(w.cond + (size_t)batch * PL, uncond, (size_t)batch * PL, d->stream))) return rc;
  if (spk) {
    if ((rc = copy_in(w.spk, spk, (size_t)batch * d->cfg.spk_dim, d->stream))) return rc;
  }
  rc = dit_upload_cfg_hidden(d, d->ws.hbuf, cfg, d->stream);
  if (rc) return rc;
  std::vector<float> times(steps + 1), dts(steps);
  rc = ctts_sway_timesteps(steps, coeff, times.data());
  if (rc) return rc;
  for (int i = 0; i < steps; i++) dts[i] = times[i + 1] - times[i];
  DitRun r;
  r.R = 2 * batch; r.z = w.z; r.cond = w.cond; r.spk = spk ? w.spk : nullptr;
  r.zero_adaln_from = spk ? batch : -1;
  r.x = w.x; r.x_rows = batch; r.steps = steps; r.times = times.data(); r.dts = dts.data();
  r.mode = 2; r.cfg = cfg;
  r.cfg_w = cfg; r.step_dt = 1.0f / (float)steps;
  rc = dit_enqueue(d, d->ws, r, d->stream, nullptr);
  if (rc) return rc;
  CTTS_CK(cudaStreamSynchronize(d->stream));
  if ((rc = dit_read_err(d, w))) return rc;
  CTTS_CK(cudaMemcpy(x_out, w.x, sizeof(float) * batch * PL, cudaMemcpyDeviceToHost));
  return CTTS_OK;
}

// ------------------------------------------------------------------ engine

namespace {

// One sub-batch of the engine: its own KV cache, DiT workspace and stream.
// Sub-batches are independent utterances, so their frame chains run as
// parallel branches of the frame graph and overlap on the GPU.
int engine_enqueue_group(ctts_engine* e, EngineGroup& g, cudaStream_t s, int* launches) {
  ctts_lm* lm = e->lm;
  ctts_dit* d = e->dit;
  const int B = g.nb, H = lm->cfg.hidden;
  const int PL = d->cfg.patch * d->cfg.latent;
  // with CFG a group's LM states and latent conditions are 2B rows:
  // [conditional B | unconditional B]
  const int zm = e->cfg_on ? 2 : 1;
  float* z = e->z + (size_t)zm * g.b0 * H;
  float* x = e->x + (size_t)g.b0 * PL;
  float* cond = e->cond + (size_t)zm * g.b0 * PL;
  float* lat = e->lat + (size_t)g.b0 * PL;
  float* stop = e->stop + (size_t)g.b0 * 2;
  const float* noise = e->noise + (size_t)g.b0 * PL;
  int nl = 0;
  // phase boundaries of the profiling mode (one sub-batch only)
  const bool prof = e->profile && e->groups.size() == 1;
  auto mark = [&](int i) -> int {
    if (prof) CTTS_CK(cudaEventRecord(e->pev[i], s));
    return CTTS_OK;
  };
  if (int rcm = mark(0)) return rcm;
  CTTS_CK(cudaMemcpyAsync(x, noise, sizeof(float) * B * PL, cudaMemcpyDeviceToDevice, s));
  // stop logits (e2e.rs:83-92) read z like the DiT prologue; outside the
  // profiling mode they run on the group's side stream, concurrently with
  // the DiT, joined before the LM step rewrites z
  const bool side = !prof && g.side;
  if (side) {
    CTTS_CK(cudaEventRecord(g.side_fork, s));
    CTTS_CK(cudaStreamWaitEvent(g.side, g.side_fork, 0));
  }
  {
    LinearArgs a; a.x = z; a.x_ld = H; a.M = B; a.K = H; a.N = 2; a.w = e->stop_w;
    a.bias = e->stop_b; a.y = stop; a.y_ld = 2;
    CTTS_CK(launch_linear(a, side ? g.side : s)); nl++;
  }
  if (side) CTTS_CK(cudaEventRecord(g.side_join, g.side));
  const int steps = e->cfg.euler_steps;
  std::vector<float> times(steps + 1), dts(steps);
  const float dt = 1.0f / (float)steps;
  for (int i = 0; i < steps; i++) {
    times[i] = (float)i * dt;
    dts[i] = dt;
  }
  DitRun r;
  const float* spk = !d->cfg.adaln ? nullptr : e->use_spk ? e->spk + (size_t)zm * g.b0 * d->cfg.spk_dim : z;
  r.R = B; r.z = z; r.cond = cond; r.spk = spk;
  r.x = x; r.x_rows = B; r.steps = steps; r.times = times.data(); r.dts = dts.data(); r.mode = 0;
  r.step_dt = dt; r.cfg_w = d->cfg.cfg_emb ? e->cfg.cfg_strength : 0.0f;
  // the first (eager) frame computes the frame-constant embeddings into the
  // group's workspace; later frames (and the captured graph) reuse them
  r.consts_cached = e->steps_done > 0;
  if (e->cfg_on) {
    // euler_sample_cfg (dit.rs:862-904) on the sway grid: both branches in
    // one 2B-row pass, the unconditional rows without AdaLN conditioning
    int rc0 = ctts_sway_timesteps(steps, e->cfg.sway_coeff, times.data());
    if (rc0) return rc0;
    for (int i = 0; i < steps; i++) dts[i] = times[i + 1] - times[i];
    r.R = 2 * B; r.mode = 2; r.cfg = e->cfg.cfg_strength; r.cfg_w = e->cfg.cfg_strength;
    r.zero_adaln_from = d->cfg.adaln ? B : -1;
  }
  if (int rcm = mark(1)) return rcm;
  int rc = dit_enqueue(d, *g.ws, r, s, &nl);
  if (rc) return rc;
  CTTS_CK(launch_affine(x, B * PL, e->cfg.latent_scale, e->cfg.latent_bias, lat, s)); nl++;
  for (int h = 0; h < zm; h++)  // the raw latent conditions both branches (bin/cutetts.rs:474-480)
    CTTS_CK(cudaMemcpyAsync(cond + (size_t)h * B * PL, x, sizeof(float) * B * PL, cudaMemcpyDeviceToDevice, s));
  if (int rcm = mark(2)) return rcm;
  {  // feedback projection straight into the LM residual stream
    LinearArgs a; a.x = x; a.x_ld = PL; a.M = B; a.K = PL; a.N = H; a.w = e->proj_w;
    a.bias = e->proj_b; a.y = g.kv->h; a.y_ld = H;
    CTTS_CK(launch_linear(a, s)); nl++;
  }
  if (e->cfg_on)  // the same acoustic input feeds the unconditional branch (bin/cutetts.rs:503-509)
    CTTS_CK(cudaMemcpyAsync(g.kv->h + (size_t)B * H, g.kv->h, sizeof(float) * B * H, cudaMemcpyDeviceToDevice, s));
  if (int rcm = mark(3)) return rcm;
  if (side) CTTS_CK(cudaStreamWaitEvent(s, g.side_join, 0));
  rc = lm_forward_rows(lm, g.kv, zm * B, -1, 0, z, s, &nl);
  if (rc) return rc;
  if (int rcm = mark(4)) return rcm;
  if (launches) *launches += nl;
  return CTTS_OK;
}

int engine_enqueue(ctts_engine* e, cudaStream_t s, int* launches) {
  int n = 0;
  if (e->groups.size() == 1) {
    int rc = engine_enqueue_group(e, e->groups[0], s, &n);
    if (rc) return rc;
  } else {
    // fork: every sub-batch branch waits for the work already on s ...
    CTTS_CK(cudaEventRecord(e->fork, s));
    for (auto& g : e->groups) {
      CTTS_CK(cudaStreamWaitEvent(g.stream, e->fork, 0));
      int rc = engine_enqueue_group(e, g, g.stream, &n);
      if (rc) return rc;
      CTTS_CK(cudaEventRecord(g.done, g.stream));
    }
    // ... join: s continues once every branch is done
    for (auto& g : e->groups) CTTS_CK(cudaStreamWaitEvent(s, g.done, 0));
  }
  if (launches) *launches = n;
  return CTTS_OK;
}

void engine_destroy(ctts_engine* e) {
  cudaSetDevice(e->lm->device);
  if (e->stream) cudaStreamSynchronize(e->stream);
  for (auto& g : e->groups) {
    if (g.stream) cudaStreamSynchronize(g.stream);
  }
  if (e->exec) cudaGraphExecDestroy(e->exec);
  if (e->graph) cudaGraphDestroy(e->graph);
  for (auto& ev : e->pev)
    if (ev) cudaEventDestroy(ev);
  if (e->h_noise) cudaFreeHost(e->h_noise);
  if (e->h_lat) cudaFreeHost(e->h_lat);
  if (e->h_stop) cudaFreeHost(e->h_stop);
  if (e->h_err) cudaFreeHost(e->h_err);
  for (auto& g : e->groups) {
    if (g.kv) ctts_kv_free(g.kv);
    delete g.ws;
    if (g.done) cudaEventDestroy(g.done);
    if (g.stream) cudaStreamDestroy(g.stream);
    if (g.side) {
      cudaStreamSynchronize(g.side);
      cudaStreamDestroy(g.side);
    }
    if (g.side_fork) cudaEventDestroy(g.side_fork);
    if (g.side_join) cudaEventDestroy(g.side_join);
  }
  if (e->fork) cudaEventDestroy(e->fork);
  if (e->stream) cudaStreamDestroy(e->stream);
  delete e;
}

}  // namespace

extern "C" int ctts_engine_create(ctts_lm* lm, ctts_dit* dit, const ctts_engine_config* cfg,
                                  ctts_engine** out) {
  CTTS_REQ(lm && dit && cfg && out, CTTS_ERR_ARG, "null argument");
  CTTS_REQ(lm->device == dit->device, CTTS_ERR_ARG, "LM and DiT on different devices");
  CTTS_REQ(dit->cfg.cond_dim == lm->cfg.hidden, CTTS_ERR_ARG, "DiT cond_dim must equal LM hidden");
  CTTS_REQ(cfg->batch > 0 && cfg->capacity > 0 && cfg->euler_steps > 0, CTTS_ERR_ARG, "bad config");
  CTTS_REQ(cfg->latent_scale != 0.0f, CTTS_ERR_ARG, "latent_scale must be non-zero");
  const int G = cfg->groups <= 0 ? 1 : cfg->groups;
  CTTS_REQ(cfg->batch % G == 0, CTTS_ERR_ARG, "batch must be a multiple of groups");
  int rc = lm_check_ready(lm);
  if (rc) return rc;
  rc = dit_check(dit);
  if (rc) return rc;
  CTTS_REQ(cfg->cfg_strength >= 0.0f, CTTS_ERR_ARG, "cfg_strength must be >= 0");
  // a head with a cfg-strength embedding (the distill checkpoint) takes the
  // strength as a condition of its single branch (bin/cutetts.rs:460-461);
  // a base head runs the two-branch CFG when the strength is positive
  const bool cfg_on = cfg->cfg_strength > 0.0f && !dit->cfg.cfg_emb;
  const int zm = cfg_on ? 2 : 1;
  CTTS_CK(cudaSetDevice(lm->device));
  auto* e = new ctts_engine();
  e->lm = lm;
  e->dit = dit;
  e->cfg = *cfg;
  e->cfg.groups = G;
  cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking);
  cudaEventCreateWithFlags(&e->fork, cudaEventDisableTiming);
  const int per = cfg->batch / G;
  e->groups.resize(G);
  for (int gi = 0; gi < G; gi++) {
    EngineGroup& g = e->groups[gi];
    g.b0 = gi * per;
    g.nb = per;
    g.ws = new DitWs();
    cudaStreamCreateWithFlags(&g.stream, cudaStreamNonBlocking);
    cudaEventCreateWithFlags(&g.done, cudaEventDisableTiming);
    cudaStreamCreateWithFlags(&g.side, cudaStreamNonBlocking);
    cudaEventCreateWithFlags(&g.side_fork, cudaEventDisableTiming);
    cudaEventCreateWithFlags(&g.side_join, cudaEventDisableTiming);
    rc = ctts_kv_alloc(lm, zm * per, cfg->capacity, &g.kv);
    if (!rc) rc = dit_ws_ensure(dit, *g.ws, zm * per, cfg->euler_steps);
    if (!rc && dit->cfg.cfg_emb) rc = dit_upload_cfg_hidden(dit, g.ws->hbuf, cfg->cfg_strength, g.stream);
    if (rc) {
      engine_destroy(e);
      return rc;
    }
  }
  e->kv = e->groups[0].kv;
  const int B = cfg->batch, H = lm->cfg.hidden, PL = dit->cfg.patch * dit->cfg.latent;
  DevArena& A = e->arena;
  e->stop_w = A.alloc<float>(2 * H);
  e->stop_b = A.alloc<float>(2);
  e->proj_w = A.alloc<float>((size_t)H * PL);
  e->proj_b = A.alloc<float>(H);
  e->cfg_on = cfg_on;
  e->z = A.alloc<float>((size_t)zm * B * H);
  e->x = A.alloc<float>((size_t)B * PL);
  e->cond = A.alloc<float>((size_t)zm * B * PL);
  e->lat = A.alloc<float>((size_t)B * PL);
  e->stop = A.alloc<float>((size_t)B * 2);
  e->noise = A.alloc<float>((size_t)B * PL);
  if (cudaMallocHost(&e->h_noise, sizeof(float) * B * PL) != cudaSuccess ||
      cudaMallocHost(&e->h_lat, sizeof(float) * B * PL) != cudaSuccess ||
      cudaMallocHost(&e->h_stop, sizeof(float) * B * 2) != cudaSuccess ||
      cudaMallocHost(&e->h_err, sizeof(int) * 2 * e->groups.size()) != cudaSuccess || !e->noise) {
    engine_destroy(e);
    return set_error(CTTS_ERR_NOMEM, "engine buffers");
  }
  e->prefilled.assign(B, false);
  e->prefilled_u.assign(B, !cfg_on);
  if (dit->cfg.adaln) {
    e->spk = A.alloc<float>((size_t)zm * B * dit->cfg.spk_dim);
    if (!e->spk) {
      engine_destroy(e);
      return set_error(CTTS_ERR_NOMEM, "engine speaker buffer");
    }
    e->use_spk = dit->cfg.spk_dim != H;
  }
  e->spk_set.assign(B, false);
  *out = e;
  return CTTS_OK;
}

extern "C" int ctts_engine_set_heads(ctts_engine* e, const float* stop_w, const float* stop_b,
                                     const float* proj_w, const float* proj_b) {
  CTTS_REQ(e && stop_w && stop_b && proj_w && proj_b, CTTS_ERR_ARG, "null argument");
  CTTS_CK(cudaSetDevice(e->lm->device));
  const int H = e->lm->cfg.hidden, PL = e->dit->cfg.patch * e->dit->cfg.latent;
  CTTS_CK(cudaMemcpy(e->stop_w, stop_w, sizeof(float) * 2 * H, cudaMemcpyHostToDevice));
  CTTS_CK(cudaMemcpy(e->stop_b, stop_b, sizeof(float) * 2, cudaMemcpyHostToDevice));
  CTTS_CK(cudaMemcpy(e->proj_w, proj_w, sizeof(float) * H * PL, cudaMemcpyHostToDevice));
  CTTS_CK(cudaMemcpy(e->proj_b, proj_b, sizeof(float) * H, cudaMemcpyHostToDevice));
  CTTS_CK(cudaStreamSynchronize(cudaStreamLegacy));
  e->heads_set = true;
  return CTTS_OK;
}

namespace {
// Prefill of utterance b's conditional (unc = false) or unconditional branch.
int engine_prefill(ctts_engine* e, int b, const float* x, int T, const float* cond0, bool unc) {
  CTTS_REQ(e && x && cond0, CTTS_ERR_ARG, "null argument");
  CTTS_REQ(b >= 0 && b < e->cfg.batch && T > 0, CTTS_ERR_ARG, "bad utterance index or length");
  CTTS_REQ(!unc || e->cfg_on, CTTS_ERR_STATE, "unconditional prefill needs cfg_strength > 0");
  CTTS_REQ(e->steps_done == 0, CTTS_ERR_STATE, "prefill after the first frame step");
  CTTS_CK(cudaSetDevice(e->lm->device));
  EngineGroup& g = e->groups[b / e->groups[0].nb];
  ctts_kv* kv = g.kv;
  const int zm = e->cfg_on ? 2 : 1;
  const int slot = (b - g.b0) + (unc ? g.nb : 0);            // KV slot within the group
  const size_t row = (size_t)zm * g.b0 + slot;               // z / cond row
  const int H = e->lm->cfg.hidden, PL = e->dit->cfg.patch * e->dit->cfg.latent;
  CTTS_REQ(T <= kv->ws_rows, CTTS_ERR_RANGE, "prefill length outside workspace");
  CTTS_CK(cudaMemcpyAsync(kv->xin, x, sizeof(float) * T * H, cudaMemcpyHostToDevice, e->stream));
  int rc = ctts_lm_prefill_dev(e->lm, kv, slot, kv->xin, T, kv->xout, e->stream);
  if (rc) return rc;
  CTTS_CK(cudaMemcpyAsync(e->z + row * H, kv->xout + (size_t)(T - 1) * H, sizeof(float) * H,
                          cudaMemcpyDeviceToDevice, e->stream));
  CTTS_CK(cudaMemcpyAsync(e->cond + row * PL, cond0, sizeof(float) * PL, cudaMemcpyHostToDevice, e->stream));
  CTTS_CK(cudaStreamSynchronize(e->stream));
  (unc ? e->prefilled_u : e->prefilled)[b] = true;
  return CTTS_OK;
}
}  // namespace

extern "C" int ctts_engine_set_speaker(ctts_engine* e, int b, const float* spk) {
  CTTS_REQ(e && spk, CTTS_ERR_ARG, "null argument");
  CTTS_REQ(b >= 0 && b < e->cfg.batch, CTTS_ERR_ARG, "bad utterance index");
  CTTS_REQ(e->dit->cfg.adaln, CTTS_ERR_STATE, "the DiT head has no AdaLN conditioning");
  // switching z -> speaker rows changes the captured frame graph: only
  // before the first step
  CTTS_REQ(e->use_spk || e->steps_done == 0, CTTS_ERR_STATE, "first speaker embedding after the first frame step");
  CTTS_CK(cudaSetDevice(e->lm->device));
  EngineGroup& g = e->groups[b / e->groups[0].nb];
  const int zm = e->cfg_on ? 2 : 1, S = e->dit->cfg.spk_dim;
  // the unconditional branch's row gets the same vector (its AdaLN is zeroed)
  for (int h = 0; h < zm; h++) {
    const size_t row = (size_t)zm * g.b0 + (b - g.b0) + (size_t)h * g.nb;
    CTTS_CK(cudaMemcpyAsync(e->spk + row * S, spk, sizeof(float) * S, cudaMemcpyHostToDevice, e->stream));
  }
  CTTS_CK(cudaStreamSynchronize(e->stream));
  if (!e->use_spk) std::fill(e->spk_set.begin(), e->spk_set.end(), false);
  e->use_spk = true;
  e->spk_set[b] = true;
  return CTTS_OK;
}

extern "C" int ctts_engine_prefill(ctts_engine* e, int b, const float* x, int T, const float* cond0) {
  return engine_prefill(e, b, x, T, cond0, false);
}

extern "C" int ctts_engine_prefill_uncond(ctts_engine* e, int b, const float* x, int T, const float* cond0) {
  return engine_prefill(e, b, x, T, cond0, true);
}

// Releases the captured frame graph: the next graph-mode frame captures
// again (after the DiT head changed path).
static void engine_drop_graph(ctts_engine* e) {
  if (e->exec) cudaGraphExecDestroy(e->exec);
  if (e->graph) cudaGraphDestroy(e->graph);
  e->exec = nullptr;
  e->graph = nullptr;
}

extern "C" int ctts_engine_step_dev(ctts_engine* e, const float* noise_dev, float* latents_dev,
                                    float* stop_dev, void* stream) {
  CTTS_REQ(e && noise_dev, CTTS_ERR_ARG, "null argument");
  CTTS_REQ(e->heads_set, CTTS_ERR_STATE, "engine heads not set");
  for (int b = 0; b < e->cfg.batch; b++) {
    CTTS_REQ(e->prefilled[b], CTTS_ERR_STATE, "utterance " + std::to_string(b) + " not prefilled");
    CTTS_REQ(!e->use_spk || e->spk_set[b], CTTS_ERR_STATE,
             "utterance " + std::to_string(b) + ": speaker embedding not set");
    CTTS_REQ(e->prefilled_u[b], CTTS_ERR_STATE,
             "utterance " + std::to_string(b) + ": unconditional branch not prefilled");
  }
  for (auto& g : e->groups)
    for (int b = 0; b < g.nb; b++) CTTS_REQ(g.kv->pos_host[b] < g.kv->cap, CTTS_ERR_RANGE, "KV cache full");
  CTTS_CK(cudaSetDevice(e->lm->device));
  cudaStream_t s = as_stream(stream, e->stream);
  const int B = e->cfg.batch, PL = e->dit->cfg.patch * e->dit->cfg.latent;
  if (noise_dev != e->noise)
    CTTS_CK(cudaMemcpyAsync(e->noise, noise_dev, sizeof(float) * B * PL, cudaMemcpyDeviceToDevice, s));
  if (!e->cfg.use_graph || e->steps_done == 0 || e->profile) {
    // first frame runs eagerly (sets kernel attributes outside any capture);
    // so does every frame of the profiling mode (events between phases)
    int n = 0;
    int rc = engine_enqueue(e, s, &n);
    if (rc) return rc;
    if (!e->profile) e->launches = n;
    if (e->profile && e->groups.size() == 1) {
      CTTS_CK(cudaEventSynchronize(e->pev[ctts_engine::kPhases]));
      for (int i = 0; i < ctts_engine::kPhases; i++) {
        float ms = 0.0f;
        CTTS_CK(cudaEventElapsedTime(&ms, e->pev[i], e->pev[i + 1]));
        e->ptimes[i].push_back(ms);
      }
    }
  } else {
    // weights uploaded since the last frame: repack the DiT cluster loop's
    // copy in place before the graph runs or is captured (the graph's
    // launch reads the same buffers); a failed repack switches the head to
    // the launch chain, which needs a new capture
    if (e->dit->cl_state == 1 && e->dit->cl_dirty && !dit_cluster_fresh(e->dit, s)) engine_drop_graph(e);
    if (!e->exec) {
      CTTS_CK(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
      int n = 0;
      int rc = engine_enqueue(e, s, &n);
      cudaGraph_t gr = nullptr;
      cudaError_t ce = cudaStreamEndCapture(s, &gr);
      if (rc) {
        if (gr) cudaGraphDestroy(gr);
        return rc;
      }
      CTTS_CK(ce);
      e->launches = n;  // the steady-state frame (constants computed by the first frame)
      e->graph = gr;
      CTTS_CK(cudaGraphInstantiate(&e->exec, gr, 0));
    }
    CTTS_CK(cudaGraphLaunch(e->exec, s));
  }
  for (auto& g : e->groups)
    for (int b = 0; b < g.nb; b++) g.kv->pos_host[b]++;
  e->steps_done++;
  if (latents_dev && latents_dev != e->lat)
    CTTS_CK(cudaMemcpyAsync(latents_dev, e->lat, sizeof(float) * B * PL, cudaMemcpyDeviceToDevice, s));
  if (stop_dev && stop_dev != e->stop)
    CTTS_CK(cudaMemcpyAsync(stop_dev, e->stop, sizeof(float) * B * 2, cudaMemcpyDeviceToDevice, s));
  return CTTS_OK;
}

extern "C" int ctts_engine_step(ctts_engine* e, const float* noise, float* latents_out, float* stop_out) {
  CTTS_REQ(e && noise && latents_out, CTTS_ERR_ARG, "null argument");
  CTTS_CK(cudaSetDevice(e->lm->device));
  const int B = e->cfg.batch, PL = e->dit->cfg.patch * e->dit->cfg.latent;
  memcpy(e->h_noise, noise, sizeof(float) * B * PL);
  CTTS_CK(cudaMemcpyAsync(e->noise, e->h_noise, sizeof(float) * B * PL, cudaMemcpyHostToDevice, e->stream));
  int rc = ctts_engine_step_dev(e, e->noise, e->lat, e->stop, e->stream);
  if (rc) return rc;
  CTTS_CK(cudaMemcpyAsync(e->h_lat, e->lat, sizeof(float) * B * PL, cudaMemcpyDeviceToHost, e->stream));
  if (stop_out)
    CTTS_CK(cudaMemcpyAsync(e->h_stop, e->stop, sizeof(float) * B * 2, cudaMemcpyDeviceToHost, e->stream));
  // the groups' error words come back with the latents: one sync per step
  for (size_t gi = 0; gi < e->groups.size(); gi++) {
    CTTS_CK(cudaMemcpyAsync(e->h_err + 2 * gi, e->groups[gi].kv->err, sizeof(int), cudaMemcpyDeviceToHost, e->stream));
    CTTS_CK(cudaMemcpyAsync(e->h_err + 2 * gi + 1, e->groups[gi].ws->err, sizeof(int), cudaMemcpyDeviceToHost,
                            e->stream));
  }
  CTTS_CK(cudaStreamSynchronize(e->stream));
  for (size_t gi = 0; gi < e->groups.size(); gi++) {
    EngineGroup& g = e->groups[gi];
    const int err = e->h_err[2 * gi], derr = e->h_err[2 * gi + 1];
    if (err != 0) CTTS_CK(cudaMemset(g.kv->err, 0, sizeof(int)));
    if (derr != 0) CTTS_CK(cudaMemset(g.ws->err, 0, sizeof(int)));
    CTTS_REQ(err != 1, CTTS_ERR_RANGE, "device reported a KV position outside capacity");
    if (derr == ctts::kDitClusterErrRange) {
      // the next frame is captured again, on the launch chain
      engine_drop_graph(e);
      return dit_cluster_range_error(e->dit);
    }
    CTTS_REQ(err == 0 && derr == 0, CTTS_ERR_TIMEOUT, "a DiT kernel gave up waiting on its pipeline, grid barrier or exchange words");
  }
  memcpy(latents_out, e->h_lat, sizeof(float) * B * PL);
  if (stop_out) memcpy(stop_out, e->h_stop, sizeof(float) * B * 2);
  return CTTS_OK;
}

extern "C" int ctts_engine_launches_per_step(const ctts_engine* e) { return e ? e->launches : -1; }

extern "C" void* ctts_engine_stream(const ctts_engine* e) { return e ? (void*)e->stream : nullptr; }

extern "C" void ctts_engine_free(ctts_engine* e) {
  if (!e) return;
  engine_destroy(e);
}

extern "C" int ctts_debug_inject_wait_fault(int skip, unsigned spin_limit) {
  g_fault_skip.store(skip ? 1 : 0, std::memory_order_relaxed);
  g_fault_spin_limit.store(spin_limit, std::memory_order_relaxed);
  return CTTS_OK;
}

// ------------------------------------------------------- phase timers
// Per-frame phase timers of the frame engine: the --profile-steps
// instrument of bin/cutetts.rs:328-350,466-478 (dit / locenc / lm phases;
// here stop head, DiT sample, feedback projection, LM step), measured on
// the device with CUDA events.  While on, frames run eagerly (not as the
// captured graph) and each step synchronizes its stream.

static const char* kPhaseNames[ctts_engine::kPhases] = {"stop", "dit", "feedback", "lm"};

extern "C" int ctts_engine_set_profile(ctts_engine* e, int on) {
  CTTS_REQ(e, CTTS_ERR_ARG, "null engine");
  CTTS_REQ(!on || e->groups.size() == 1, CTTS_ERR_STATE, "phase timers need a single sub-batch group");
  CTTS_CK(cudaSetDevice(e->lm->device));
  if (on && !e->pev[0])
    for (auto& ev : e->pev) CTTS_CK(cudaEventCreate(&ev));
  for (auto& v : e->ptimes) v.clear();
  e->profile = on != 0;
  return CTTS_OK;
}

// mean / p50 / p99 (milliseconds) of phase `phase` over the profiled frames;
// *n receives the frame count
extern "C" int ctts_engine_profile_stats(const ctts_engine* e, int phase, float* mean_p50_p99, int* n) {
  CTTS_REQ(e && mean_p50_p99 && phase >= 0 && phase < ctts_engine::kPhases, CTTS_ERR_ARG, "bad argument");
  std::vector<float> v = e->ptimes[phase];
  if (n) *n = (int)v.size();
  mean_p50_p99[0] = mean_p50_p99[1] = mean_p50_p99[2] = 0.0f;
  if (v.empty()) return CTTS_OK;
  std::sort(v.begin(), v.end());
  double sum = 0.0;
  for (float x : v) sum += x;
  const size_t k = v.size();
  mean_p50_p99[0] = (float)(sum / (double)k);
  mean_p50_p99[1] = v[k / 2];
  mean_p50_p99[2] = v[std::min(k - 1, k * 99 / 100)];
  return CTTS_OK;
}

// One line per phase, "name: n=N mean=Xms p50=Yms p99=Zms" (the format of
// bin/cutetts.rs:338-350 profile_report); returns the bytes written.
extern "C" int ctts_engine_profile_report(const ctts_engine* e, char* buf, int len) {
  CTTS_REQ(e && buf && len > 0, CTTS_ERR_ARG, "bad argument");
  std::string out;
  for (int i = 0; i < ctts_engine::kPhases; i++) {
    float st[3];
    int n = 0;
    ctts_engine_profile_stats(e, i, st, &n);
    char line[160];
    if (n == 0)
      snprintf(line, sizeof(line), "%s: n/a\n", kPhaseNames[i]);
    else
      snprintf(line, sizeof(line), "%s: n=%d mean=%.3fms p50=%.3fms p99=%.3fms\n", kPhaseNames[i], n, st[0], st[1],
               st[2]);
    out += line;
  }
  const int w = (int)std::min<size_t>(out.size(), (size_t)len - 1);
  memcpy(buf, out.data(), (size_t)w);
  buf[w] = 0;
  return w;
}
