// lm_grid.cu -- one LM decode step (every layer, the final RMSNorm and the
// cache-length advance) as ONE grid-persistent launch for small batches
// with fp32 weights (the batch-1 fp32 decode of config[2]).
//
// Replaces the per-layer launch chain of qwen.rs:229-406 decode_step
// (fused QKV / attention / o-proj / gate-up / down launches, linear.cu and
// attention.cu) at batch 1..4, where 60 dependent launches of a few
// microseconds each dominate the step.  One CTA per SM (cooperative launch,
// so every CTA is resident); phases are separated by grid barriers (a
// global counter per barrier, zeroed again by the last CTA to leave):
//   Q  RMSNorm1 (every CTA, all rows, redundant) -> this CTA's QKV columns
//   A  every (utterance, query head) over gridDim / (R nq) CTAs, each a
//      contiguous range of the keys: QK-Norm + RoPE of the query and of the
//      new key, append of the new key/value row (the head group's first
//      query head), online-softmax partials per range
//   O  the ranges' partials merged (every CTA) -> this CTA's o-proj
//      columns + residual
//   G  RMSNorm2 (redundant) -> this CTA's gate/up columns -> SwiGLU
//   D  this CTA's down columns + residual
// then the final RMSNorm and pos += 1.  Each GEMV column's weight row is
// streamed from HBM into shared memory by bulk copies two phases ahead
// (double-buffered), so the copies overlap the barriers and the phases in
// between.  Intra-kernel data is read with L2-coherent loads (ld.global.cg).
#include <cstdio>

#include "common.cuh"
#include "launch_state.h"
#include "lm_grid.cuh"

namespace ctts {

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr uint32_t kSpinLimit = 1u << 22;
constexpr int kMaxCtas = 1024;  // grid size bound (one CTA per SM)

CTTS_DEV float4 ldcg4(const float* p) { return __ldcg(reinterpret_cast<const float4*>(p)); }

CTTS_DEV uint32_t ld_acquire(const unsigned* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// grid barrier k: arrival as one release reduction (cumulative over this
// CTA's writes, ordered before it by the block barrier), acquire polling
CTTS_DEV void grid_sync(const LmGridArgs& a, int k) {
  __syncthreads();
  if (threadIdx.x == 0) {
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(a.bar + k) : "memory");
    const unsigned n = gridDim.x;
    uint32_t it = 0;
    while (ld_acquire(a.bar + k) < n) {
      // a CTA that already gave up waiting somewhere makes every later wait
      // end at once (a position error, code 1, does not stop the barriers)
      if (++it == kSpinLimit || ((it & 1023u) == 0 && a.err && *reinterpret_cast<volatile int*>(a.err) == 4)) {
        if (a.err) atomicExch(a.err, 4);
        break;
      }
    }
  }
  __syncthreads();
}

// ---- GEMV phases: kind, geometry, this CTA's output columns
enum Kind { kQ = 0, kO = 1, kG = 2, kD = 3 };
struct Geo {
  int N, K, rows_per;  // output columns, weight row length, weight rows per column
};
CTTS_DEV Geo geo(const LmGridArgs& a, int kind) {
  const int qkvw = (a.nq + 2 * a.nkv) * a.hd, qd = a.nq * a.hd;
  switch (kind) {
    case kQ: return {qkvw, a.H, 1};
    case kO: return {a.H, qd, 1};
    case kG: return {a.F, a.H, 2};
    default: return {a.H, a.F, 1};
  }
}
CTTS_DEV const float* weights(const LmGridArgs& a, int kind, int l) {
  switch (kind) {
    case kQ: return a.wqkv[l];
    case kO: return a.wo[l];
    case kG: return a.wgu[l];
    default: return a.wd[l];
  }
}
// weight row of output column n (row j of its rows_per): SwiGLU columns
// pair gate row 128(n/64) + n%64 with the up row 64 further
CTTS_DEV int weight_row(int kind, int n, int j) { return kind == kG ? 128 * (n / 64) + n % 64 + 64 * j : n; }
__host__ __device__ inline void cols_of(int N, int b, int G, int& n0, int& n1) {
  n0 = (int)(((long)N * b) / G);
  n1 = (int)(((long)N * (b + 1)) / G);
}

// Shared memory: two weight staging buffers, the activation rows, the
// attention scratch, two mbarriers.
struct Smem {
  size_t buf_bytes;  // one staging buffer
  size_t xs_floats;  // activation rows [R][max K]
  __host__ __device__ size_t xs_off() const { return 2 * buf_bytes; }
  __host__ __device__ size_t att_off() const { return xs_off() + xs_floats * 4; }
  // attention: q, new k, new v [3][hd], warp partials [8][hd + 2]
  // (the o-proj phase reuses it for the attention merge factors, one per CTA: kMaxCtas)
  __host__ __device__ size_t att_floats(int hd) const {
    const size_t f = (size_t)3 * hd + (size_t)kWarps * (hd + 2);
    return f > (size_t)kMaxCtas ? f : (size_t)kMaxCtas;
  }
  __host__ __device__ size_t bar_off(int hd) const { return (att_off() + att_floats(hd) * 4 + 15) & ~size_t(15); }
  __host__ __device__ size_t total(int hd) const { return bar_off(hd) + 16; }
};
__host__ __device__ inline Smem smem_of(int R, int H, int nq, int nkv, int hd, int F, int G) {
  const int qkvw = (nq + 2 * nkv) * hd, qd = nq * hd;
  const int N[4] = {qkvw, H, F, H}, K[4] = {H, qd, H, F}, rp[4] = {1, 1, 2, 1};
  Smem m;
  m.buf_bytes = 0;
  for (int i = 0; i < 4; i++) {
    const size_t cols = (size_t)(N[i] + G - 1) / G + 1;
    const size_t b = cols * rp[i] * K[i] * 4;
    if (b > m.buf_bytes) m.buf_bytes = b;
  }
  m.buf_bytes = (m.buf_bytes + 127) & ~size_t(127);
  int kmax = H > qd ? H : qd;
  if (F > kmax) kmax = F;
  m.xs_floats = (size_t)R * kmax;
  return m;
}

// Staging: warp 0 copies the weight rows of this CTA's columns of phase
// `kind` of layer l into buffer b as a few large bulk copies (lane 0 arms
// the buffer's mbarrier with the byte count), completing on the buffer's
// mbarrier.  A CTA's columns are consecutive weight rows, except that the
// gate/up rows of SwiGLU columns sit in 64-row tiles (gate rows
// 128(n/64) + n%64, up rows 64 further): per 64-column segment one gate and
// one up copy.  Buffer layout: [j][column - n0][K] (j: gate, up).
struct Stage {
  uint8_t* buf[2];
  uint32_t bar[2];  // shared addresses
  uint32_t ph[2];   // waits so far per buffer (parity of the next)
};
CTTS_DEV void stage(const LmGridArgs& a, Stage& st, int kind, int l, int b) {
  if (threadIdx.x >= 32) return;
  const int lane = threadIdx.x;
  const Geo g = geo(a, kind);
  int n0, n1;
  cols_of(g.N, blockIdx.x, gridDim.x, n0, n1);
  const uint32_t row_bytes = (uint32_t)g.K * 4u, cols = (uint32_t)(n1 - n0);
  if (lane == 0) {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(st.bar[b]),
                 "r"(cols * g.rows_per * row_bytes)
                 : "memory");
  }
  __syncwarp();
  const float* base = weights(a, kind, l);
  const uint32_t dst0 = static_cast<uint32_t>(__cvta_generic_to_shared(st.buf[b]));
  // copy c: segment c / rows_per of the column range, row set j = c % rows_per
  const int seg0 = kind == kG ? n0 / 64 : 0;
  const int nseg = kind == kG ? (n1 > n0 ? (n1 - 1) / 64 - seg0 + 1 : 0) : (n1 > n0 ? 1 : 0);
  for (int c = lane; c < nseg * g.rows_per; c += 32) {
    const int sg = c / g.rows_per, j = c % g.rows_per;
    const int a0 = kind == kG ? max(n0, 64 * (seg0 + sg)) : n0;
    const int a1 = kind == kG ? min(n1, 64 * (seg0 + sg + 1)) : n1;
    const float* src = base + (size_t)weight_row(kind, a0, j) * g.K;
    const uint32_t dst = dst0 + ((uint32_t)j * cols + (uint32_t)(a0 - n0)) * row_bytes;
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"((uint32_t)(a1 - a0) * row_bytes), "r"(st.bar[b])
                 : "memory");
  }
}
CTTS_DEV void wait_stage(const LmGridArgs& a, Stage& st, int b) {
  bool done = false;
  for (uint32_t it = 0; it < kSpinLimit && !done; ++it) {
    uint32_t d;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(d)
        : "r"(st.bar[b]), "r"(st.ph[b] & 1u)
        : "memory");
    done = d != 0;
  }
  if (!done && threadIdx.x == 0 && a.err) atomicExch(a.err, 4);
  st.ph[b]++;
}

// RMSNorm of the R rows of h (every CTA, one warp per row) -> xs[r][H]
// (x * inv * gain, prep/linear_rows semantics); every load of the row is
// issued before the first use (H <= 128 * kMaxH4)
constexpr int kMaxH4 = 8;
CTTS_DEV void norm_rows(const LmGridArgs& a, const float* gain, float* xs) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, H = a.H, nv = H >> 7;
  for (int r = warp; r < a.R; r += kWarps) {
    const float* src = a.h + (size_t)r * H;
    float* dst = xs + (size_t)r * H;
    float4 v[kMaxH4], gv[kMaxH4];  // the row and the gains, all loads in flight together
#pragma unroll
    for (int i = 0; i < kMaxH4; i++)
      if (i < nv) {
        v[i] = ldcg4(src + lane * 4 + 128 * i);
        gv[i] = *reinterpret_cast<const float4*>(gain + lane * 4 + 128 * i);
      }
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < kMaxH4; i++)
      if (i < nv) ss = fmaf(v[i].x, v[i].x, fmaf(v[i].y, v[i].y, fmaf(v[i].z, v[i].z, fmaf(v[i].w, v[i].w, ss))));
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / (float)H + a.eps);
#pragma unroll
    for (int i = 0; i < kMaxH4; i++) {
      if (i >= nv) break;
      const int k = lane * 4 + 128 * i;
      *reinterpret_cast<float4*>(dst + k) = make_float4(v[i].x * inv * gv[i].x, v[i].y * inv * gv[i].y,
                                                        v[i].z * inv * gv[i].z, v[i].w * inv * gv[i].w);
    }
  }
}

// n floats of intra-kernel data (global, L2-coherent) -> xs: four 16-byte
// loads per thread issued before any of their stores (a store through a
// generic pointer would otherwise hold back the next load)
CTTS_DEV void load_rows(const float* src, int n, float* xs) {
  for (int i0 = threadIdx.x * 4; i0 < n; i0 += kThreads * 16) {
    float4 v[4];
#pragma unroll
    for (int q = 0; q < 4; q++)
      if (i0 + q * kThreads * 4 < n) v[q] = ldcg4(src + i0 + q * kThreads * 4);
#pragma unroll
    for (int q = 0; q < 4; q++)
      if (i0 + q * kThreads * 4 < n) *reinterpret_cast<float4*>(xs + i0 + q * kThreads * 4) = v[q];
  }
}

// This CTA's output columns of phase `kind`: each warp takes two columns
// (n and n + kWarps) per pass, lanes over 4-element groups of K, the RW
// rows of xs [RW][K] loaded once for both columns; the warp reductions of
// all (column, weight row, row) sums run interleaved, not one after another.
// The residual entries an o-proj / down column updates (written by this
// CTA's own earlier phases) are fetched before the dot products.
template <int RW>
CTTS_DEV void gemv(const LmGridArgs& a, Stage& st, int kind, int b, const float* xs) {
  const Geo g = geo(a, kind);
  int n0, n1;
  cols_of(g.N, blockIdx.x, gridDim.x, n0, n1);
  wait_stage(a, st, b);
  __syncthreads();  // xs complete
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, K = g.K;
  const bool resid = kind == kO || kind == kD;
  const float* wb = reinterpret_cast<const float*>(st.buf[b]);
  for (int n = n0 + warp; n < n1; n += 2 * kWarps) {
    const int nb = n + kWarps;
    const bool two = nb < n1;
    float yold[2][RW];
#pragma unroll
    for (int c = 0; c < 2; c++)
#pragma unroll
      for (int r = 0; r < RW; r++)
        yold[c][r] = (resid && lane == 0 && (c == 0 || two)) ? __ldcg(a.h + (size_t)r * a.H + (c ? nb : n)) : 0.0f;
    float acc[2][2][RW];  // [column][weight row j][activation row]
#pragma unroll
    for (int c = 0; c < 2; c++)
#pragma unroll
      for (int j = 0; j < 2; j++)
#pragma unroll
        for (int r = 0; r < RW; r++) acc[c][j][r] = 0.0f;
    for (int k = lane * 4; k < K; k += 128) {
      float4 xv[RW];
#pragma unroll
      for (int r = 0; r < RW; r++) xv[r] = *reinterpret_cast<const float4*>(xs + (size_t)r * K + k);
#pragma unroll
      for (int c = 0; c < 2; c++) {
        if (c == 1 && !two) break;
        const int nc = c ? nb : n;
#pragma unroll
        for (int j = 0; j < 2; j++) {
          if (j >= g.rows_per) break;
          const float4 wv = *reinterpret_cast<const float4*>(wb + ((size_t)j * (n1 - n0) + (nc - n0)) * K + k);
#pragma unroll
          for (int r = 0; r < RW; r++)
            acc[c][j][r] = fmaf(wv.x, xv[r].x, fmaf(wv.y, xv[r].y, fmaf(wv.z, xv[r].z, fmaf(wv.w, xv[r].w, acc[c][j][r]))));
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int c = 0; c < 2; c++)
#pragma unroll
        for (int j = 0; j < 2; j++)
#pragma unroll
          for (int r = 0; r < RW; r++)
            if ((c == 0 || two) && j < g.rows_per) acc[c][j][r] += __shfl_xor_sync(0xffffffffu, acc[c][j][r], o);
    if (lane == 0) {
      const int qkvw = (a.nq + 2 * a.nkv) * a.hd;
#pragma unroll
      for (int c = 0; c < 2; c++) {
        if (c == 1 && !two) break;
        const int nc = c ? nb : n;
#pragma unroll
        for (int r = 0; r < RW; r++) {
          if (kind == kQ) {
            a.qkv[(size_t)r * qkvw + nc] = acc[c][0][r];
          } else if (kind == kG) {
            a.act[(size_t)r * a.F + nc] = silu(acc[c][0][r]) * acc[c][1][r];
          } else {  // o-proj / down: residual
            a.h[(size_t)r * a.H + nc] = yold[c][r] + acc[c][0][r];
          }
        }
      }
    }
  }
}

// Attention, keys split over CTAs: job = (utterance, query head), S =
// gridDim / jobs CTAs per job, CTA s of a job walks the contiguous key range
// s of the job's p + 1 keys (cached rows 0..p-1 and the new row p, which the
// last range holds).  Warp 0 prepares the query (QK-Norm + RoPE at the
// utterance's position); in the last range warps 1, 2 prepare the new key
// and value and the head group's first query head appends them to the
// cache.  Warp w walks keys j0 + w, j0 + w + 8, ... with its own online
// softmax (lane = HD/32 consecutive dims, scores by warp reduction); the
// warp states merge in warp order into this CTA's partial
// part[cta] = (max, sum, acc[HD]), merged across ranges by merge_attn.
constexpr int kMaxSplits = 8;  // key ranges per job (the merge reads them all)
CTTS_DEV int attn_splits(const LmGridArgs& a) {
  const int jobs = a.R * a.nq;
  const int S = (int)gridDim.x / jobs;
  return S < 1 ? 1 : S > kMaxSplits ? kMaxSplits : S;
}
template <int HD>
CTTS_DEV void attn_phase(const LmGridArgs& a, int l, float* sa) {
  const int S = attn_splits(a), jobs = a.R * a.nq;
  const int job = blockIdx.x / S, sp = blockIdx.x % S;
  if (job >= jobs) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = job / a.nq, hq = job % a.nq, G = a.nq / a.nkv, kvh = hq / G;
  const int qkvw = (a.nq + 2 * a.nkv) * HD;
  float* part = a.part + (size_t)blockIdx.x * (HD + 2);
  const int p = a.pos[b];
  if (p < 0 || p >= a.cap) {
    if (threadIdx.x == 0 && a.err) atomicExch(a.err, 1);
    for (int d = threadIdx.x; d < HD + 2; d += kThreads) part[d] = d == 0 ? -INFINITY : 0.0f;
    return;
  }
  const int j0 = (int)(((long)(p + 1) * sp) / S), j1 = (int)(((long)(p + 1) * (sp + 1)) / S);
  const bool last = j1 == p + 1;  // this range holds the new row
  constexpr int PER = HD / 32, DPL = HD / 32;
  float* qv = sa;
  float* knew = sa + HD;
  float* vnew = sa + 2 * HD;
  float* wpart = sa + 3 * HD;  // [8][HD + 2]
  const float* kc = a.kcache + (size_t)l * a.layer_elems;
  const float* vc = a.vcache + (size_t)l * a.layer_elems;
  const size_t row0 = ((size_t)b * a.nkv + kvh) * a.cap;
  if (warp == 0 || (last && warp < 3)) {
    const float* src =
        a.qkv + (size_t)b * qkvw + (size_t)(warp == 0 ? hq : warp == 1 ? a.nq + kvh : a.nq + a.nkv + kvh) * HD;
    // the row, its QK-Norm gains and the RoPE frequencies: loads in flight together
    const float* gn = warp == 0 ? a.qn[l] : warp == 1 ? a.kn[l] : nullptr;
    float v[PER], gw[PER], fr[PER / 2];
#pragma unroll
    for (int j = 0; j < PER; j++) {
      v[j] = __ldcg(src + lane + 32 * j);
      gw[j] = gn ? gn[lane + 32 * j] : 1.0f;
    }
#pragma unroll
    for (int j = 0; j < PER / 2; j++) fr[j] = warp < 2 ? a.inv_freq[lane + 32 * j] : 0.0f;
    if (warp < 2) {
      if (gn) {
        float ss = 0.0f;
#pragma unroll
        for (int j = 0; j < PER; j++) ss = fmaf(v[j], v[j], ss);
        ss = warp_sum(ss);
        const float inv = 1.0f / sqrtf(ss / (float)HD + a.eps);
#pragma unroll
        for (int j = 0; j < PER; j++) v[j] = v[j] * inv * gw[j];
      }
#pragma unroll
      for (int j = 0; j < PER / 2; j++) {  // rotate-half pairs (i, i + HD/2)
        float sn, cs;
        sincosf((float)p * fr[j], &sn, &cs);
        const float x1 = v[j], x2 = v[j + PER / 2];
        v[j] = x1 * cs - x2 * sn;
        v[j + PER / 2] = x1 * sn + x2 * cs;
      }
    }
    float* dst = warp == 0 ? qv : warp == 1 ? knew : vnew;
    float* cache = warp == 1 ? a.kcache : a.vcache;
#pragma unroll
    for (int j = 0; j < PER; j++) {
      const int d = lane + 32 * j;
      if (warp > 0 && hq % G == 0) cache[(size_t)l * a.layer_elems + (row0 + p) * HD + d] = v[j];
      dst[d] = v[j];
    }
  }
  __syncthreads();
  float q[DPL];
#pragma unroll
  for (int e = 0; e < DPL; e++) q[e] = qv[DPL * lane + e];
  const float scale = 1.0f / sqrtf((float)HD);
  float m = -INFINITY, lsum = 0.0f, acc[DPL];
#pragma unroll
  for (int e = 0; e < DPL; e++) acc[e] = 0.0f;
  // key/value row j of this (utterance, KV head): cached rows from global
  // memory (written by earlier launches), the new row from shared memory
  auto load_row = [&](const float* cache, const float* fresh, int j, float* out) {
    if (j == p) {
#pragma unroll
      for (int e = 0; e < DPL; e++) out[e] = fresh[DPL * lane + e];
      return;
    }
    const float* rp = cache + (row0 + j) * HD + (size_t)DPL * lane;
    if constexpr (DPL == 2) {
      const float2 t = *reinterpret_cast<const float2*>(rp);
      out[0] = t.x; out[1] = t.y;
    } else {
      const float4 t = *reinterpret_cast<const float4*>(rp);
      out[0] = t.x; out[1] = t.y; out[2] = t.z; out[3] = t.w;
    }
  };
  constexpr int U = 4;  // keys in flight per warp
  for (int jb = j0 + warp; jb < j1; jb += kWarps * U) {
    float kk[U][DPL], vv[U][DPL], s[U];
#pragma unroll
    for (int u = 0; u < U; u++) {
      const int j = jb + kWarps * u;
      if (j < j1) {
        load_row(kc, knew, j, kk[u]);
        load_row(vc, vnew, j, vv[u]);
      } else {  // past the range: weight 0, and 0 x (stale register) must not be NaN
#pragma unroll
        for (int e = 0; e < DPL; e++) kk[u][e] = vv[u][e] = 0.0f;
      }
    }
    float mx = -INFINITY;
#pragma unroll
    for (int u = 0; u < U; u++) {
      const int j = jb + kWarps * u;
      float d = 0.0f;
#pragma unroll
      for (int e = 0; e < DPL; e++) d = fmaf(q[e], kk[u][e], d);
      d = warp_sum(d);
      s[u] = j < j1 ? d * scale : -INFINITY;
      mx = fmaxf(mx, s[u]);
    }
    const float mn = fmaxf(m, mx);
    const float f = m == -INFINITY ? 0.0f : expf(m - mn);
    lsum *= f;
#pragma unroll
    for (int e = 0; e < DPL; e++) acc[e] *= f;
#pragma unroll
    for (int u = 0; u < U; u++) {
      const float pu = s[u] == -INFINITY ? 0.0f : expf(s[u] - mn);
      lsum += pu;
#pragma unroll
      for (int e = 0; e < DPL; e++) acc[e] = fmaf(pu, vv[u][e], acc[e]);
    }
    m = mn;
  }
  if (lane == 0) {
    wpart[warp * (HD + 2)] = m;
    wpart[warp * (HD + 2) + 1] = lsum;
  }
#pragma unroll
  for (int e = 0; e < DPL; e++) wpart[warp * (HD + 2) + 2 + DPL * lane + e] = acc[e];
  __syncthreads();
  // this range's partial (unnormalised, relative to its max), warp order
  float M = -INFINITY;
#pragma unroll
  for (int w = 0; w < kWarps; w++) M = fmaxf(M, wpart[w * (HD + 2)]);
  for (int d = threadIdx.x; d < HD + 2; d += kThreads) {
    if (d == 0) {
      part[0] = M;
      continue;
    }
    float o = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarps; w++) {
      const float mw = wpart[w * (HD + 2)];
      const float fw = mw == -INFINITY ? 0.0f : expf(mw - M);
      o = fmaf(wpart[w * (HD + 2) + d], fw, o);  // d == 1: the sum, d >= 2: acc
    }
    part[d] = o;
  }
}

// The o-proj operand: every job's key-range partials merged in range order
// (every CTA, redundantly) -> xs[r][hq * HD + d] = softmax(.) V.  The
// partials of a thread's elements (kE at a time) are requested before the
// range factors are computed, so the factors' loads and the values' loads
// share one L2 round trip.
template <int HD>
CTTS_DEV void merge_attn(const LmGridArgs& a, float* xs, float* fac) {
  const int S = attn_splits(a), jobs = a.R * a.nq, qd = a.nq * HD, n = a.R * qd;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int kE = 4;
  for (int i0 = 0; i0 < n; i0 += kE * kThreads) {
    float v[kE][kMaxSplits];
#pragma unroll
    for (int e = 0; e < kE; e++) {
      const int i = i0 + threadIdx.x + e * kThreads;
      const int r = i / qd, hq = (i % qd) / HD, d = i % HD, job = r * a.nq + hq;
      const float* pp = a.part + (size_t)job * S * (HD + 2) + 2 + d;
#pragma unroll
      for (int sp = 0; sp < kMaxSplits; sp++) v[e][sp] = (i < n && sp < S) ? __ldcg(pp + (size_t)sp * (HD + 2)) : 0.0f;
    }
    if (i0 == 0) {
      // a warp per job: lane sp holds range sp's (max, sum)
      for (int job = warp; job < jobs; job += kWarps) {
        const float* pp = a.part + (size_t)(job * S + lane) * (HD + 2);
        const float ms = lane < S ? __ldcg(pp) : -INFINITY;
        const float ls = lane < S ? __ldcg(pp + 1) : 0.0f;
        float M = ms;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        const float f = ms == -INFINITY ? 0.0f : expf(ms - M);
        // the sum in range order (lane 0 gathers), deterministic
        float L = 0.0f;
        for (int sp = 0; sp < S; sp++) L = fmaf(__shfl_sync(0xffffffffu, ls, sp), __shfl_sync(0xffffffffu, f, sp), L);
        if (lane < S) fac[job * S + lane] = f / L;
      }
      __syncthreads();
    }
#pragma unroll
    for (int e = 0; e < kE; e++) {
      const int i = i0 + threadIdx.x + e * kThreads;
      if (i >= n) continue;
      const int r = i / qd, hq = (i % qd) / HD, job = r * a.nq + hq;
      float o = 0.0f;
#pragma unroll
      for (int sp = 0; sp < kMaxSplits; sp++)
        if (sp < S) o = fmaf(v[e][sp], fac[job * S + sp], o);
      xs[i] = o;
    }
  }
}

template <int HD, int RW>
__global__ void __launch_bounds__(kThreads, 1) lm_grid_kernel(const LmGridArgs a) {
  extern __shared__ __align__(128) uint8_t smraw[];
  const Smem m = smem_of(a.R, a.H, a.nq, a.nkv, HD, a.F, gridDim.x);
  Stage st;
  st.buf[0] = smraw;
  st.buf[1] = smraw + m.buf_bytes;
  float* xs = reinterpret_cast<float*>(smraw + m.xs_off());
  float* sa = reinterpret_cast<float*>(smraw + m.att_off());
  st.bar[0] = static_cast<uint32_t>(__cvta_generic_to_shared(smraw + m.bar_off(HD)));
  st.bar[1] = st.bar[0] + 8u;
  st.ph[0] = st.ph[1] = 0u;
  if (threadIdx.x == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(st.bar[0]));
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(st.bar[1]));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  // weight phases Q, O, G, D of every layer alternate buffers 0, 1, 0, 1;
  // each buffer is refilled two weight phases ahead, as soon as its phase
  // has been computed
  stage(a, st, kQ, 0, 0);
  stage(a, st, kO, 0, 1);
  int k = 0;
  for (int l = 0; l < a.NL; l++) {
    norm_rows(a, a.norm1[l], xs);
    gemv<RW>(a, st, kQ, 0, xs);
    __syncthreads();
    stage(a, st, kG, l, 0);
    grid_sync(a, k++);
    attn_phase<HD>(a, l, sa);
    grid_sync(a, k++);
    merge_attn<HD>(a, xs, sa);
    gemv<RW>(a, st, kO, 1, xs);
    __syncthreads();
    stage(a, st, kD, l, 1);
    grid_sync(a, k++);
    norm_rows(a, a.norm2[l], xs);
    gemv<RW>(a, st, kG, 0, xs);
    __syncthreads();
    if (l + 1 < a.NL) stage(a, st, kQ, l + 1, 0);
    grid_sync(a, k++);
    load_rows(a.act, a.R * a.F, xs);
    gemv<RW>(a, st, kD, 1, xs);
    __syncthreads();
    if (l + 1 < a.NL) stage(a, st, kO, l + 1, 1);
    grid_sync(a, k++);
  }
  // final RMSNorm of the last layer's rows and the cache-length advance
  // (every CTA is past its last attention phase)
  if (blockIdx.x == 0) {
    norm_rows(a, a.final_norm, a.out);
    if (threadIdx.x < a.R) a.pos[threadIdx.x] += 1;
  }
  // the last CTA to leave zeroes the counters for the next launch
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(a.bar + k, 1u) == gridDim.x - 1) {
      for (int i = 0; i <= k; i++) a.bar[i] = 0u;
      __threadfence();
    }
  }
}

// one CTA per SM of the current device (0: no cooperative launch)
int grid_ctas() { return device_coop() ? device_sms() : 0; }

template <int HD, int RW>
cudaError_t launch_t(const LmGridArgs& a, size_t smem, cudaStream_t s) {
  auto kern = lm_grid_kernel<HD, RW>;
  static SmemOptIn opt;
  if (cudaError_t e = opt.ensure((const void*)kern, smem)) return e;
  int per_sm = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem);
  if (e != cudaSuccess || per_sm < 1) return e != cudaSuccess ? e : cudaErrorInvalidConfiguration;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid_ctas());
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: the grid barriers need it
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, a);
  if (e != cudaSuccess) (void)cudaGetLastError();
  return e;
}

}  // namespace

int lm_grid_counters(int NL) { return 5 * NL + 1; }

size_t lm_grid_part_floats(int hd) { return (size_t)(grid_ctas() > 0 ? grid_ctas() : 1) * (hd + 2); }

bool lm_grid_supported(int R, int NL, int H, int nq, int nkv, int hd, int F) {
  if (R < 1 || R > LmGridArgs::kMaxRows || NL < 1 || NL > LmGridArgs::kMaxNL) return false;
  if ((hd != 64 && hd != 128) || nkv < 1 || nq % nkv || H % 128 || H > 128 * kMaxH4 || F % 128 || (nq * hd) % 128 ||
      ((nq + 2 * nkv) * hd) % 4)
    return false;
  const int G = grid_ctas();
  if (G <= 0 || G > kMaxCtas || R * nq > G) return false;
  return smem_of(R, H, nq, nkv, hd, F, G).total(hd) <= 220 * 1024;
}

cudaError_t launch_lm_grid(const LmGridArgs& a, cudaStream_t s) {
  if (!lm_grid_supported(a.R, a.NL, a.H, a.nq, a.nkv, a.hd, a.F) || !a.bar || !a.h || !a.out || !a.pos || !a.part)
    return cudaErrorInvalidValue;
  const size_t smem = smem_of(a.R, a.H, a.nq, a.nkv, a.hd, a.F, grid_ctas()).total(a.hd);
  // the utterance count is a template parameter: the GEMV accumulators of
  // exactly R rows stay in registers
  switch (a.R) {
    case 1: return a.hd == 64 ? launch_t<64, 1>(a, smem, s) : launch_t<128, 1>(a, smem, s);
    case 2: return a.hd == 64 ? launch_t<64, 2>(a, smem, s) : launch_t<128, 2>(a, smem, s);
    case 3: return a.hd == 64 ? launch_t<64, 3>(a, smem, s) : launch_t<128, 3>(a, smem, s);
    default: return a.hd == 64 ? launch_t<64, 4>(a, smem, s) : launch_t<128, 4>(a, smem, s);
  }
}

}  // namespace ctts
