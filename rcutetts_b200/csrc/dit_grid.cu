// dit_grid.cu -- the DiT Euler loop of one frame (every step, every layer,
// the output/feedback tail) as ONE grid-persistent launch for small batches
// with fp32 weights (the batch-1 fp32 decode of config[2]).
//
// Replaces the per-step launch chain of dit.rs:775-814 predict_cached /
// euler_sample (dit.rs:819-842) at batch 1..4, where ~200 dependent
// launches of a few microseconds each dominate the frame.  One CTA per SM
// (cooperative launch, so every CTA is resident).  Each phase splits its
// output columns over all CTAs and streams each column's weight row once
// per step (fp32; the weights stay L2-resident across the ten steps), so
// the work per phase is a few microseconds of L2 bandwidth spread over the
// whole GPU:
//   P1  RMSNorm1 + AdaLN modulate (every CTA, all rows, redundant) -> QKV
//   P2  3-token RoPE attention (every CTA, redundant) -> o-proj -> gated
//       residual into the CTA's columns of the residual stream
//   P3  RMSNorm2 + modulate -> gate/up -> SwiGLU
//   P4  down -> gated residual
//   T1  final norm -> out_proj -> x += dt * v
//   T2  in_proj(x) and the next step's sequence rows
// Every phase consumes what all CTAs produced in the phase before it, and
// only that.  The hand-over needs no grid barrier: each value travels as one
// 64-bit word (tag << 32 | float bits) written with a single store, the tag
// naming the launch generation and the producing phase, and a consumer
// polls the words it needs (L2, not L1) until every tag is the one it
// expects: one L2 round trip per phase instead of a barrier's arrival, its
// poll and the data load after it.  A word is rewritten only two phases
// later, by a CTA that has already consumed the next phase's output of
// every CTA, which each CTA produces after its own reads: no word is
// overwritten while a consumer may still need it.
#include <cstdio>

#include "common.cuh"
#include "launch_state.h"
#include "dit_grid.cuh"

namespace ctts {

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr uint32_t kSpinLimit = 1u << 22;  // polls of about 1 us: seconds
constexpr int kMaxH4 = 8;  // hidden <= 1024: 16-byte groups per lane of a row
// The last warp issues the weight staging of the next phase while the
// others start polling its inputs (no row poll and no bulk poll uses it).
constexpr int kStageWarp = kWarps - 1;
constexpr int kPollThreads = kStageWarp * 32;
constexpr int kRedFloats = kWarps * 4 * 12;  // K-split partial sums: warps x 4 columns x rows

CTTS_DEV float ldcg(const float* p) { return __ldcg(p); }

// ---- flag-tagged exchange words
using u64 = unsigned long long;
// Polls of one exchange word before a consumer gives up.
CTTS_DEV uint32_t spin_limit(const DitGridArgs& a) { return a.spin_limit ? a.spin_limit : kSpinLimit; }
CTTS_DEV void ll_put(u64* p, float v, uint32_t tag) {
  const u64 w = ((u64)tag << 32) | __float_as_uint(v);
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
CTTS_DEV void ld4(const u64* p, u64 (&w)[4]) {
  asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(w[0]), "=l"(w[1]) : "l"(p) : "memory");
  asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(w[2]), "=l"(w[3]) : "l"(p + 2) : "memory");
}
CTTS_DEV bool tags_are(const u64 (&w)[4], uint32_t tag) {
  return (uint32_t)(w[0] >> 32) == tag && (uint32_t)(w[1] >> 32) == tag && (uint32_t)(w[2] >> 32) == tag &&
         (uint32_t)(w[3] >> 32) == tag;
}
// Polls groups of four words (group i at p[i]; none where p[i] is null)
// until every tag equals `tag`; group i's values go to v[i].  Only groups
// still pending are reloaded.  Bounded: a thread that gives up (or sees
// that another one did) records error 4 and goes on with what it has.
// (not inlined: inside the phases its load registers pushed the dot
// products into local memory)
template <int NG>
__device__ __noinline__ void ll_poll(const DitGridArgs& a, const u64* const (&p)[NG], uint32_t tag, float4 (&v)[NG]) {
  uint32_t pend = 0;
#pragma unroll
  for (int i = 0; i < NG; i++)
    if (p[i]) pend |= 1u << i;
  for (uint32_t it = 0; pend; ++it) {
    u64 w[NG][4];
#pragma unroll
    for (int i = 0; i < NG; i++)
      if ((pend >> i) & 1u) ld4(p[i], w[i]);
#pragma unroll
    for (int i = 0; i < NG; i++)
      if (((pend >> i) & 1u) && tags_are(w[i], tag)) {
        v[i] = make_float4(__uint_as_float((uint32_t)w[i][0]), __uint_as_float((uint32_t)w[i][1]),
                           __uint_as_float((uint32_t)w[i][2]), __uint_as_float((uint32_t)w[i][3]));
        pend &= ~(1u << i);
      }
    if (pend && (it == spin_limit(a) || ((it & 255u) == 255u && a.err && *reinterpret_cast<volatile int*>(a.err)))) {
      if (a.err) atomicExch(a.err, 4);
      break;
    }
  }
}
// One word, polled the same way.
CTTS_DEV float ll_get1(const DitGridArgs& a, const u64* p, uint32_t tag) {
  for (uint32_t it = 0;; ++it) {
    u64 w;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    if ((uint32_t)(w >> 32) == tag) return __uint_as_float((uint32_t)w);
    if (it == spin_limit(a) || ((it & 255u) == 255u && a.err && *reinterpret_cast<volatile int*>(a.err))) {
      if (a.err) atomicExch(a.err, 4);
      return 0.0f;
    }
  }
}

// One row of H = 128 nv exchange words for a warp: lane's groups at
// lane * 4 + 128 i, polled four groups at a time.
CTTS_DEV void poll_row(const DitGridArgs& a, const u64* src, int nv, uint32_t tag, float4 (&v)[kMaxH4]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int h = 0; h < kMaxH4; h += 4) {
    if (h < nv) {
      const u64* ps[4];
      float4 t[4];
#pragma unroll
      for (int q = 0; q < 4; q++) ps[q] = h + q < nv ? src + lane * 4 + 128 * (h + q) : nullptr;
      ll_poll<4>(a, ps, tag, t);
#pragma unroll
      for (int q = 0; q < 4; q++) v[h + q] = t[q];
    }
  }
}

// Exchange areas inside a.ll: residual rows [3R][H], QKV rows [3R][qkvw],
// SwiGLU rows [3R][F], latent x [R][L] (the device code and
// dit_grid_ll_words() agree on this layout).
struct LLMap {
  u64 *seq, *qkv, *act, *x;
};
__host__ __device__ inline size_t ll_offsets(int R, int H, int qkvw, int F, size_t (&o)[4]) {
  const size_t rows = 3 * (size_t)R;
  o[0] = 0;
  o[1] = o[0] + rows * H;
  o[2] = o[1] + rows * qkvw;
  o[3] = o[2] + rows * F;
  return o[3] + (size_t)R * 64;
}
CTTS_DEV LLMap ll_map(const DitGridArgs& a) {
  size_t o[4];
  ll_offsets(a.R, a.H, (a.nq + 2 * a.nkv) * a.hd, a.F, o);
  return {a.ll + o[0], a.ll + o[1], a.ll + o[2], a.ll + o[3]};
}

// n exchange words (n a multiple of 4) -> floats in shared memory: the
// threads of every warp but the staging one, eight 16-byte groups each per
// pass (one pass for the QKV and SwiGLU rows of one utterance).
CTTS_DEV void load_rows(const DitGridArgs& a, float* dst, const u64* src, int n, uint32_t tag) {
  if (threadIdx.x >= kPollThreads) return;
  for (int i0 = threadIdx.x * 4; i0 < n; i0 += kPollThreads * 32) {
    float4 v[8];
    const u64* ps[8];
#pragma unroll
    for (int q = 0; q < 8; q++) {
      const int i = i0 + q * kPollThreads * 4;
      ps[q] = i < n ? src + i : nullptr;
    }
    ll_poll<8>(a, ps, tag, v);
#pragma unroll
    for (int q = 0; q < 8; q++) {
      const int i = i0 + q * kPollThreads * 4;
      if (i < n) *reinterpret_cast<float4*>(dst + i) = v[q];
    }
  }
}

// One output column for every row: acc[r] = w[:] . xs[r, :] with the weight
// row already staged in shared memory (warp, lanes over 4-element groups).
template <int RW>
CTTS_DEV void row_dots(const float* w, int K, const float* xs, float* acc) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int r = 0; r < RW; r++) acc[r] = 0.0f;
#pragma unroll 4
  for (int k = lane * 4; k < K; k += 128) {
    const float4 wv = *reinterpret_cast<const float4*>(w + k);
#pragma unroll
    for (int r = 0; r < RW; r++) {
      const float4 xv = *reinterpret_cast<const float4*>(xs + (size_t)r * K + k);
      acc[r] = fmaf(wv.x, xv.x, fmaf(wv.y, xv.y, fmaf(wv.z, xv.z, fmaf(wv.w, xv.w, acc[r]))));
    }
  }
#pragma unroll
  for (int r = 0; r < RW; r++) acc[r] = warp_sum(acc[r]);
}

CTTS_DEV float4 lds4(const float* p) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(static_cast<uint32_t>(__cvta_generic_to_shared(p))));
  return v;
}

// Dot products of NC weight rows w[c] (c < nc; the rest skipped) with RW
// activation rows xs[r][K], all in shared memory: lanes over 4-element
// groups of K, each activation group loaded once for every weight row,
// and the NC x RW warp reductions independent of one another (their
// shuffles overlap instead of running one reduction after the other).
template <int RW, int NC>
CTTS_DEV void warp_dots(const float* const (&w)[NC], int nc, int K, const float* xs, float (&acc)[NC][RW]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int c = 0; c < NC; c++)
#pragma unroll
    for (int r = 0; r < RW; r++) acc[c][r] = 0.0f;
#pragma unroll 2
  for (int k = lane * 4; k < K; k += 128) {
    float4 xv[RW];
#pragma unroll
    for (int r = 0; r < RW; r++) xv[r] = lds4(xs + (size_t)r * K + k);
#pragma unroll
    for (int c = 0; c < NC; c++) {
      if (c < nc) {
        const float4 wv = lds4(w[c] + k);
#pragma unroll
        for (int r = 0; r < RW; r++)
          acc[c][r] = fmaf(wv.x, xv[r].x, fmaf(wv.y, xv[r].y, fmaf(wv.z, xv[r].z, fmaf(wv.w, xv[r].w, acc[c][r]))));
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int c = 0; c < NC; c++)
#pragma unroll
      for (int r = 0; r < RW; r++) acc[c][r] += __shfl_xor_sync(0xffffffffu, acc[c][r], o);
}

// This warp's columns n0 + warp + kWarps t of the CTA's share [n0, n1),
// two at a time.  Column n has PER staged weight rows (row j at
// wbuf + (j (n1 - n0) + n - n0) K: gate then up for the SwiGLU columns);
// emit(n, acc of row 0, acc of row PER - 1) runs on every lane.
template <int RW, int PER, class Emit>
CTTS_DEV void gemv_cols(const float* wbuf, int K, int n0, int n1, const float* xs, Emit emit) {
  const int warp = threadIdx.x >> 5;
  constexpr int NC = 2 * PER;
  for (int n = n0 + warp; n < n1; n += 2 * kWarps) {
    const int n2 = n + kWarps;
    const bool two = n2 < n1;
    const float* w[NC];
#pragma unroll
    for (int j = 0; j < PER; j++) {
      w[j] = wbuf + ((size_t)j * (n1 - n0) + (n - n0)) * K;
      w[PER + j] = two ? wbuf + ((size_t)j * (n1 - n0) + (n2 - n0)) * K : w[j];
    }
    float acc[NC][RW];
    warp_dots<RW, NC>(w, two ? NC : PER, K, xs, acc);
    emit(n, acc[0], acc[PER - 1]);
    if (two) emit(n2, acc[PER], acc[NC - 1]);
  }
}

// The CTA's few output columns [n0, n1) (4 per pass) with K split over all
// warps: each warp sums its K slice for every column and row, the warp
// sums go through shared memory `red` and are added in warp order
// (deterministic); emit(n, r, value) runs once per (column, row).
template <int RW, class Emit>
CTTS_DEV void gemv_ksplit(const float* wbuf, int K, int n0, int n1, const float* xs, float* red, Emit emit) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ks = ((K / 4 + kWarps - 1) / kWarps) * 4;
  const int k0 = warp * ks, k1 = min(K, k0 + ks);
  for (int c0 = n0; c0 < n1; c0 += 4) {
    const int nc = min(4, n1 - c0);
    float acc[4][RW];
#pragma unroll
    for (int c = 0; c < 4; c++)
#pragma unroll
      for (int r = 0; r < RW; r++) acc[c][r] = 0.0f;
    for (int k = k0 + lane * 4; k < k1; k += 128) {
      float4 xv[RW];
#pragma unroll
      for (int r = 0; r < RW; r++) xv[r] = lds4(xs + (size_t)r * K + k);
#pragma unroll
      for (int c = 0; c < 4; c++) {
        if (c < nc) {
          const float4 wv = lds4(wbuf + (size_t)(c0 - n0 + c) * K + k);
#pragma unroll
          for (int r = 0; r < RW; r++)
            acc[c][r] = fmaf(wv.x, xv[r].x, fmaf(wv.y, xv[r].y, fmaf(wv.z, xv[r].z, fmaf(wv.w, xv[r].w, acc[c][r]))));
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int c = 0; c < 4; c++)
#pragma unroll
        for (int r = 0; r < RW; r++) acc[c][r] += __shfl_xor_sync(0xffffffffu, acc[c][r], o);
    if (lane == 0)
#pragma unroll
      for (int c = 0; c < 4; c++)
#pragma unroll
        for (int r = 0; r < RW; r++) red[(warp * 4 + c) * RW + r] = acc[c][r];
    __syncthreads();
    for (int i = threadIdx.x; i < nc * RW; i += kThreads) {
      const int c = i / RW, r = i % RW;
      float v = 0.0f;
#pragma unroll
      for (int w = 0; w < kWarps; w++) v += red[(w * 4 + c) * RW + r];
      emit(c0 + c, r, v);
    }
    __syncthreads();
  }
}

// This CTA's share [n0, n1) of N output columns.
// (32-bit arithmetic: N * gridDim.x stays far below 2^32 for the supported
// shapes, and a 64-bit division costs hundreds of cycles per phase.)
CTTS_DEV void my_cols(int N, int& n0, int& n1) {
  n0 = (int)(((uint32_t)N * blockIdx.x) / gridDim.x);
  n1 = (int)(((uint32_t)N * (blockIdx.x + 1)) / gridDim.x);
}

// ---- weight staging: before the phase polls its inputs, the staging warp
// copies the weight rows of this CTA's output columns of that phase into
// the staging buffer with bulk copies (the weights do not depend on the
// barrier), completing on one mbarrier; the phase waits on it.
enum Kind { kQKV, kO, kGU, kD, kOut, kFill };

struct Stage {
  float* wbuf;
  float* aux;    // the phase's small operands: norm gains, AdaLN rows, embeddings
  float* rope;   // [3 positions][cos 32, sin 32]
  float* resv;   // [rows][kMaxCols] this CTA's columns of the residual stream
  float* red;    // [kWarps][4][rows] per-warp sums of the K-split GEMVs
  uint32_t bar;  // shared address of the mbarrier
  uint32_t ph;   // uses so far (parity of the next wait)
  LLMap ll;      // exchange areas
  uint32_t tag;  // tag of the running phase; its inputs carry tag - 1
};
constexpr int kMaxCols = 8;  // residual columns per CTA (hidden / CTAs)

struct KindGeom {
  const float* base;
  int N, K, rows_per;  // output columns, row length, weight rows per column
};
CTTS_DEV KindGeom geom(const DitGridArgs& a, int kind, int l) {
  const int qkvw = (a.nq + 2 * a.nkv) * a.hd, qd = a.nq * a.hd;
  switch (kind) {
    case kQKV: return {a.wqkv[l], qkvw, a.H, 1};
    case kO: return {a.wo[l], a.H, qd, 1};
    case kGU: return {a.wgu[l], a.F, a.H, 2};
    case kD: return {a.wd[l], a.H, a.F, 1};
    case kOut: return {a.out_w, a.R * a.L, a.H, 1};
    default: return {a.in_w, a.H, a.L, 1};
  }
}
// weight row of output column n (and row j of its rows_per)
CTTS_DEV int weight_row(const DitGridArgs& a, int kind, int n, int j) {
  if (kind == kGU) return 128 * (n / 64) + n % 64 + 64 * j;  // gate, then up (tile interleave)
  if (kind == kOut) return n % a.L;
  return n;
}

CTTS_DEV void bulk_copy(uint32_t dst, const float* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

// The phase's small operands into st.aux (all 16-byte aligned vectors):
//   kQKV/kGU: norm gain [H], then per utterance [shift | scale] [2H]
//   kO/kD:    per utterance the AdaLN gate [H]
//   kOut:     final norm [H]
//   kFill:    mu [R][H], cond [R][H], temb(stn) [H], dtemb [H]
CTTS_DEV uint32_t stage_aux(const DitGridArgs& a, Stage& st, int kind, int l, int stn, bool issue) {
  const int H = a.H, R = a.R;
  const long adld = (long)a.NL * 6 * H;
  const uint32_t dst0 = static_cast<uint32_t>(__cvta_generic_to_shared(st.aux));
  const uint32_t hb = (uint32_t)H * 4u;
  uint32_t bytes = 0;
  auto cp = [&](const float* src, uint32_t nbytes) {
    if (issue) bulk_copy(dst0 + bytes, src, nbytes, st.bar);
    bytes += nbytes;
  };
  if (kind == kQKV || kind == kGU) {
    cp(kind == kQKV ? a.norm1[l] : a.norm2[l], hb);
    if (a.ad)
      for (int u = 0; u < R; u++) cp(a.ad + (size_t)u * adld + (size_t)l * 6 * H + (kind == kQKV ? 0 : 3) * H, 2 * hb);
  } else if (kind == kO || kind == kD) {
    if (a.ad)
      for (int u = 0; u < R; u++) cp(a.ad + (size_t)u * adld + (size_t)l * 6 * H + (kind == kO ? 2 : 5) * H, hb);
  } else if (kind == kOut) {
    cp(a.final_norm, hb);
  } else {
    cp(a.mu, (uint32_t)R * hb);
    cp(a.condh, (uint32_t)R * hb);
    cp(a.temb + (size_t)stn * H, hb);
    cp(a.dtemb, hb);
  }
  return bytes;
}

// staging warp: lane 0 arms the mbarrier with the phase's byte count and copies
// the small operands; the weight rows of this CTA's columns go as a few
// large bulk copies, one per run of consecutive rows (consecutive columns
// are consecutive rows except across a 64-column gate/up tile or, for the
// output projection, across an utterance's latent columns).  Buffer layout:
// [j][column - n0][K] (j: gate, up for the SwiGLU columns).
CTTS_DEV void stage_weights(const DitGridArgs& a, Stage& st, int kind, int l, int stn = 0) {
  if (threadIdx.x < kStageWarp * 32) return;
  const int lane = threadIdx.x - kStageWarp * 32;
  const KindGeom g = geom(a, kind, l);
  int n0, n1;
  my_cols(g.N, n0, n1);
  const uint32_t row_bytes = (uint32_t)g.K * 4u, cols = (uint32_t)(n1 - n0);
  if (lane == 0) {
    const uint32_t bytes = cols * g.rows_per * row_bytes + stage_aux(a, st, kind, l, stn, false);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(st.bar), "r"(bytes) : "memory");
    stage_aux(a, st, kind, l, stn, true);
  }
  __syncwarp();
  const int period = kind == kGU ? 64 : kind == kOut ? a.L : 0;
  const int seg0 = period ? n0 / period : 0;
  const int nseg = n1 > n0 ? (period ? (n1 - 1) / period - seg0 + 1 : 1) : 0;
  const uint32_t dst0 = static_cast<uint32_t>(__cvta_generic_to_shared(st.wbuf));
  for (int c = lane; c < nseg * g.rows_per; c += 32) {
    const int sg = c / g.rows_per, j = c % g.rows_per;
    const int a0 = period ? max(n0, period * (seg0 + sg)) : n0;
    const int a1 = period ? min(n1, period * (seg0 + sg + 1)) : n1;
    bulk_copy(dst0 + ((uint32_t)j * cols + (uint32_t)(a0 - n0)) * row_bytes,
              g.base + (size_t)weight_row(a, kind, a0, j) * g.K, (uint32_t)(a1 - a0) * row_bytes, st.bar);
  }
}

CTTS_DEV void wait_weights(const DitGridArgs& a, Stage& st) {
  bool done = false;
  for (uint32_t it = 0; it < kSpinLimit && !done; ++it) {
    uint32_t d;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(d)
        : "r"(st.bar), "r"(st.ph & 1u)
        : "memory");
    done = d != 0;
  }
  if (!done && threadIdx.x == 0 && a.err) atomicExch(a.err, 4);
  st.ph++;
}

// Rows of the residual stream -> RMSNorm (+ AdaLN modulate) into shared
// memory xs[rows][H]: one polling warp per row (prep/linear_rows semantics: x * inv
// * gain, then * (1 + scale) + shift).  Each warp polls its first row
// before waiting on the staged gains and weights, so the staging copies
// complete under the poll.
template <int RW>
CTTS_DEV void norm_rows(const DitGridArgs& a, Stage& st, float* xs) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int rows = RW;
  const int H = a.H, nv = H >> 7;
  const float* gain = st.aux;  // staged: gain [H], per utterance [shift | scale]
  float4 v[kMaxH4];
  if (warp < kStageWarp && warp < rows) poll_row(a, st.ll.seq + (size_t)warp * H, nv, st.tag - 1, v);
  wait_weights(a, st);
  for (int r = warp; warp < kStageWarp && r < rows; r += kStageWarp) {
    if (r != warp) poll_row(a, st.ll.seq + (size_t)r * H, nv, st.tag - 1, v);
    float* dst = xs + (size_t)r * H;
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < kMaxH4; i++)
      if (i < nv) ss = fmaf(v[i].x, v[i].x, fmaf(v[i].y, v[i].y, fmaf(v[i].z, v[i].z, fmaf(v[i].w, v[i].w, ss))));
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / (float)H + a.eps);
    const float* md = a.ad ? st.aux + H + (size_t)(r / 3) * 2 * H : nullptr;
#pragma unroll
    for (int i = 0; i < kMaxH4; i++) {
      if (i >= nv) break;
      const int k = lane * 4 + 128 * i;
      float e[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
      for (int j = 0; j < 4; j++) {
        e[j] = e[j] * inv * gain[k + j];
        if (md) e[j] = e[j] * (1.0f + md[H + k + j]) + md[k + j];
      }
      *reinterpret_cast<float4*>(dst + k) = make_float4(e[0], e[1], e[2], e[3]);
    }
  }
}

// A CTA without output columns in a phase reads none of its inputs (a
// later phase's producers wait only on the CTAs that produced something)
// and only retires the phase's staging wait.
CTTS_DEV bool idle_phase(const DitGridArgs& a, Stage& st, int N) {
  int n0, n1;
  my_cols(N, n0, n1);
  if (n0 < n1) return false;
  wait_weights(a, st);
  return true;
}

// P1: norm1 (+ modulate) -> this CTA's QKV columns.
template <int RW>
CTTS_DEV void phase_qkv(const DitGridArgs& a, Stage& st, int l, float* sm) {
  constexpr int rows = RW;
  const int H = a.H, qkvw = (a.nq + 2 * a.nkv) * a.hd;
  if (idle_phase(a, st, qkvw)) return;
  norm_rows<RW>(a, st, sm);
  __syncthreads();
  int n0, n1;
  my_cols(qkvw, n0, n1);
  const int lane = threadIdx.x & 31;
  const bool skip = a.skip_qkv_cta0 && blockIdx.x == 0;  // injected fault (tests only)
  gemv_cols<RW, 1>(st.wbuf, H, n0, n1, sm, [&](int n, const float* acc, const float*) {
    if (lane == 0 && !skip)
#pragma unroll
      for (int r = 0; r < rows; r++) ll_put(st.ll.qkv + (size_t)r * qkvw + n, acc[r], st.tag);
  });
}

// P2: 3-token bidirectional attention with RoPE at positions 0..2 (every
// CTA, all rows; dit.rs:277-306, 361-405) -> this CTA's o-proj columns ->
// gated residual (h += (1 + gate) * o).
template <int RW>
CTTS_DEV void phase_attn_o(const DitGridArgs& a, Stage& st, int l, float* sm) {
  constexpr int rows = RW;
  const int H = a.H, hd = a.hd, nq = a.nq, nkv = a.nkv;
  const int qkvw = (nq + 2 * nkv) * hd, qd = nq * hd, G = nq / nkv;
  if (idle_phase(a, st, H)) return;
  float* qs = sm;                         // [rows][qkvw]
  float* att = sm + (size_t)rows * qkvw;  // [rows][qd]
  load_rows(a, qs, st.ll.qkv, rows * qkvw, st.tag - 1);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float scale = 1.0f / sqrtf((float)hd);
  for (int job = warp; job < a.R * nq; job += kWarps) {
    const int u = job / nq, h = job % nq, kh = h / G;
    float q[3][2], k[3][2], v[3][2];
#pragma unroll
    for (int s = 0; s < 3; s++) {
      const float* row = qs + (size_t)(3 * u + s) * qkvw;
#pragma unroll
      for (int j = 0; j < 2; j++) {
        q[s][j] = row[h * hd + lane + 32 * j];
        k[s][j] = row[(nq + kh) * hd + lane + 32 * j];
        v[s][j] = row[(nq + nkv + kh) * hd + lane + 32 * j];
      }
      // rotate-half: dim lane pairs with lane + 32 (head_dim 64)
      const float cs = st.rope[s * 64 + lane], sn = st.rope[s * 64 + 32 + lane];
      float a1 = q[s][0], a2 = q[s][1];
      q[s][0] = a1 * cs - a2 * sn;
      q[s][1] = a1 * sn + a2 * cs;
      a1 = k[s][0];
      a2 = k[s][1];
      k[s][0] = a1 * cs - a2 * sn;
      k[s][1] = a1 * sn + a2 * cs;
    }
    // the nine query-key dot products reduced over the warp together
    float dots[3][3];
#pragma unroll
    for (int i = 0; i < 3; i++)
#pragma unroll
      for (int j2 = 0; j2 < 3; j2++) dots[i][j2] = fmaf(q[i][0], k[j2][0], q[i][1] * k[j2][1]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int i = 0; i < 3; i++)
#pragma unroll
        for (int j2 = 0; j2 < 3; j2++) dots[i][j2] += __shfl_xor_sync(0xffffffffu, dots[i][j2], o);
#pragma unroll
    for (int i = 0; i < 3; i++) {
      float sc[3], m = -INFINITY;
#pragma unroll
      for (int j2 = 0; j2 < 3; j2++) {
        sc[j2] = dots[i][j2] * scale;
        m = fmaxf(m, sc[j2]);
      }
      float lsum = 0.0f;
#pragma unroll
      for (int j2 = 0; j2 < 3; j2++) {
        sc[j2] = expf(sc[j2] - m);
        lsum += sc[j2];
      }
      const float inv = 1.0f / lsum;
      float* o = att + (size_t)(3 * u + i) * qd + h * hd;
#pragma unroll
      for (int j = 0; j < 2; j++) {
        float acc = 0.0f;
#pragma unroll
        for (int j2 = 0; j2 < 3; j2++) acc = fmaf(sc[j2] * inv, v[j2][j], acc);
        o[lane + 32 * j] = acc;
      }
    }
  }
  wait_weights(a, st);
  __syncthreads();
  int n0, n1;
  my_cols(H, n0, n1);
  gemv_ksplit<RW>(st.wbuf, qd, n0, n1, att, st.red, [&](int n, int r, float v) {
    const float coef = a.ad ? 1.0f + st.aux[(size_t)(r / 3) * H + n] : 1.0f;
    float* rv = st.resv + r * kMaxCols + (n - n0);
    *rv = *rv + coef * v;
    ll_put(st.ll.seq + (size_t)r * H + n, *rv, st.tag);
  });
}

// P3: norm2 (+ modulate) -> this CTA's SwiGLU columns (staged as the gate
// rows, then the up rows, of the CTA's columns).
template <int RW>
CTTS_DEV void phase_gate_up(const DitGridArgs& a, Stage& st, int l, float* sm) {
  constexpr int rows = RW;
  const int H = a.H, F = a.F;
  if (idle_phase(a, st, F)) return;
  norm_rows<RW>(a, st, sm);
  __syncthreads();
  int n0, n1;
  my_cols(F, n0, n1);
  const int lane = threadIdx.x & 31;
  gemv_cols<RW, 2>(st.wbuf, H, n0, n1, sm, [&](int j, const float* g, const float* u) {
    if (lane == 0)
#pragma unroll
      for (int r = 0; r < rows; r++) ll_put(st.ll.act + (size_t)r * F + j, silu(g[r]) * u[r], st.tag);
  });
}

// P4: down over the SwiGLU rows -> gated residual.
template <int RW>
CTTS_DEV void phase_down(const DitGridArgs& a, Stage& st, int l, float* sm) {
  constexpr int rows = RW;
  const int H = a.H, F = a.F;
  if (idle_phase(a, st, H)) return;
  load_rows(a, sm, st.ll.act, rows * F, st.tag - 1);
  wait_weights(a, st);
  __syncthreads();
  int n0, n1;
  my_cols(H, n0, n1);
  gemv_ksplit<RW>(st.wbuf, F, n0, n1, sm, st.red, [&](int n, int r, float v) {
    const float coef = a.ad ? 1.0f + st.aux[(size_t)(r / 3) * H + n] : 1.0f;
    float* rv = st.resv + r * kMaxCols + (n - n0);
    *rv = *rv + coef * v;
    ll_put(st.ll.seq + (size_t)r * H + n, *rv, st.tag);
  });
}

// T1: final norm of each utterance's x row (token 2), out_proj, Euler
// update x += dt * (v + b) on this CTA's outputs.
CTTS_DEV void phase_out(const DitGridArgs& a, Stage& st, int stp, float* sm) {
  const int H = a.H, L = a.L, R = a.R, nv = H >> 7;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (idle_phase(a, st, R * L)) return;
  const float* fnorm = st.aux;
  // warp u < R (<= 4) takes utterance u's x row; polled before the wait
  // on the staged weights
  float4 v[kMaxH4];
  if (warp < R) poll_row(a, st.ll.seq + (size_t)(3 * warp + 2) * H, nv, st.tag - 1, v);
  wait_weights(a, st);
  if (warp < R) {
    const int u = warp;
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
      *reinterpret_cast<float4*>(sm + (size_t)u * H + k) =
          make_float4(v[i].x * inv * fnorm[k], v[i].y * inv * fnorm[k + 1], v[i].z * inv * fnorm[k + 2],
                      v[i].w * inv * fnorm[k + 3]);
    }
  }
  __syncthreads();
  int o0, o1;
  my_cols(R * L, o0, o1);
  for (int o = o0 + warp; o < o1; o += kWarps) {
    const int u = o / L, l = o % L;
    // the same thread updates latent column o at every step: its current
    // value is fetched before the dot product instead of after
    float* x = a.x + (size_t)u * L + l;
    const float xo = lane == 0 ? ldcg(x) : 0.0f;
    float acc[1];
    row_dots<1>(st.wbuf + (size_t)(o - o0) * H, H, sm + (size_t)u * H, acc);
    if (lane == 0) {
      const float xn = xo + a.dts[stp] * (acc[0] + (a.out_b ? a.out_b[l] : 0.0f));
      *x = xn;
      ll_put(st.ll.x + o, xn, st.tag);
    }
  }
}

// T2: the sequence rows of step stn: [mu + temb + dtemb; cond; in_proj(x)]
// for this CTA's columns.
CTTS_DEV void phase_fill(const DitGridArgs& a, Stage& st, int stn, float* sm) {
  const int H = a.H, L = a.L, R = a.R;
  if (idle_phase(a, st, H)) return;
  // x0 comes from before the launch; later steps' x from the output phase
  if (threadIdx.x < kPollThreads)
    for (int i = threadIdx.x; i < R * L; i += kPollThreads)
      sm[i] = stn == 0 ? ldcg(a.x + i) : ll_get1(a, st.ll.x + i, st.tag - 1);
  wait_weights(a, st);
  __syncthreads();
  int n0, n1;
  my_cols(H, n0, n1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int n = n0 + warp; n < n1; n += kWarps) {
    const float* w = st.wbuf + (size_t)(n - n0) * L;
    for (int u = 0; u < R; u++) {
      float acc = 0.0f;
      for (int k = lane; k < L; k += 32) acc = fmaf(w[k], sm[u * L + k], acc);
      acc = warp_sum(acc);
      if (lane == 0) {
        const float* aux = st.aux;  // mu [R][H], cond [R][H], temb [H], dtemb [H]
        const float v0 = (aux[(size_t)u * H + n] + aux[(size_t)2 * R * H + n]) + aux[(size_t)(2 * R + 1) * H + n];
        const float v1 = aux[(size_t)(R + u) * H + n];
        const float v2 = acc + (a.in_b ? a.in_b[n] : 0.0f);
        u64* row = st.ll.seq + (size_t)(3 * u) * H + n;
        ll_put(row, v0, st.tag);
        ll_put(row + H, v1, st.tag);
        ll_put(row + 2 * H, v2, st.tag);
        float* rv = st.resv + (3 * u) * kMaxCols + (n - n0);
        rv[0] = v0;
        rv[kMaxCols] = v1;
        rv[2 * kMaxCols] = v2;
      }
    }
  }
}

// Shared memory: activations [act_floats], weight staging [w_floats], one
// mbarrier.  The staging buffer holds the largest per-CTA phase share.
struct GridSmem {
  size_t act_floats, w_floats, aux_floats;
  __host__ __device__ size_t aux_off() const { return act_floats + w_floats; }
  __host__ __device__ size_t rope_off() const { return aux_off() + aux_floats; }
  __host__ __device__ size_t resv_off() const { return rope_off() + 192; }
  __host__ __device__ size_t red_off() const { return (resv_off() + DitGridArgs::kMaxRows * kMaxCols + 3) & ~(size_t)3; }
  __host__ __device__ size_t bar_off() const { return red_off() + kRedFloats; }
};
__host__ __device__ inline size_t cdiv_sz(size_t a, size_t b) { return (a + b - 1) / b; }
__host__ __device__ inline GridSmem grid_smem(int R, int H, int F, int nq, int nkv, int hd, int L, int G) {
  const size_t rows = 3 * (size_t)R, qkvw = (size_t)(nq + 2 * nkv) * hd, qd = (size_t)nq * hd;
  GridSmem m;
  m.act_floats = rows * (size_t)H;
  if (rows * (size_t)F > m.act_floats) m.act_floats = rows * (size_t)F;
  if (rows * (qkvw + qd) > m.act_floats) m.act_floats = rows * (qkvw + qd);
  const size_t w[6] = {(cdiv_sz(qkvw, G) + 1) * H, (cdiv_sz(H, G) + 1) * qd, (cdiv_sz(F, G) + 1) * 2 * H,
                       (cdiv_sz(H, G) + 1) * F, (cdiv_sz((size_t)R * L, G) + 1) * H, (cdiv_sz(H, G) + 1) * L};
  m.w_floats = 0;
  for (size_t v : w) m.w_floats = v > m.w_floats ? v : m.w_floats;
  m.w_floats = (m.w_floats + 3) & ~(size_t)3;  // 16-byte aligned areas
  m.aux_floats = (size_t)(2 * R + 2) * H;
  return m;
}

template <int RW>
__global__ void __launch_bounds__(kThreads, 1) dit_grid_kernel(const DitGridArgs a) {
  extern __shared__ __align__(16) float sm[];
  const GridSmem gs = grid_smem(a.R, a.H, a.F, a.nq, a.nkv, a.hd, a.L, gridDim.x);
  Stage st;
  st.wbuf = sm + gs.act_floats;
  st.aux = sm + gs.aux_off();
  st.rope = sm + gs.rope_off();
  st.resv = sm + gs.resv_off();
  st.red = sm + gs.red_off();
  st.bar = static_cast<uint32_t>(__cvta_generic_to_shared(sm + gs.bar_off()));
  st.ph = 0;
  if (threadIdx.x < 96) {  // RoPE of token positions 0..2 (dit.rs:277-306)
    const int sp = threadIdx.x / 32, j = threadIdx.x % 32;
    float sn, cs;
    sincosf((float)sp * a.inv_freq[j], &sn, &cs);
    st.rope[sp * 64 + j] = cs;
    st.rope[sp * 64 + 32 + j] = sn;
  }
  if (threadIdx.x == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(st.bar));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  // phase tags: launch generation (bar[0], advanced by the last CTA to
  // leave) and phase number; never 0, the value of a fresh exchange word
  st.ll = ll_map(a);
  st.tag = ((__ldcg(a.bar) & 0x3fffffu) << 10) + 1u;
  // each phase's weights are staged right after the previous phase, before
  // the inputs of the phase are polled
  stage_weights(a, st, kFill, 0, 0);
  phase_fill(a, st, 0, sm);
  for (int stp = 0; stp < a.steps; stp++) {
    for (int l = 0; l < a.NL; l++) {
      __syncthreads();
      stage_weights(a, st, kQKV, l);
      st.tag++;
      phase_qkv<RW>(a, st, l, sm);
      __syncthreads();
      stage_weights(a, st, kO, l);
      st.tag++;
      phase_attn_o<RW>(a, st, l, sm);
      __syncthreads();
      stage_weights(a, st, kGU, l);
      st.tag++;
      phase_gate_up<RW>(a, st, l, sm);
      __syncthreads();
      stage_weights(a, st, kD, l);
      st.tag++;
      phase_down<RW>(a, st, l, sm);
    }
    __syncthreads();
    stage_weights(a, st, kOut, 0);
    st.tag++;
    phase_out(a, st, stp, sm);
    if (stp + 1 < a.steps) {
      __syncthreads();
      stage_weights(a, st, kFill, 0, stp + 1);
      st.tag++;
      phase_fill(a, st, stp + 1, sm);
    }
  }
  // the last CTA to leave advances the generation for the next launch
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(a.bar + 1, 1u) == gridDim.x - 1) {
      a.bar[1] = 0u;
      a.bar[0] = a.bar[0] + 1u;
      __threadfence();
    }
  }
}

size_t grid_smem_bytes(int R, int H, int F, int nq, int nkv, int hd, int L, int G) {
  const GridSmem m = grid_smem(R, H, F, nq, nkv, hd, L, G);
  return (m.bar_off() + 4) * sizeof(float);
}

// one CTA per SM of the current device (0: no cooperative launch)
int grid_ctas() { return device_coop() ? device_sms() : 0; }

}  // namespace

int dit_grid_counters(int, int) { return 2; }

size_t dit_grid_ll_words(int R, int H, int nq, int nkv, int hd, int F, int) {
  size_t o[4];
  return ll_offsets(R, H, (nq + 2 * nkv) * hd, F, o);
}

bool dit_grid_supported(int R, int NL, int steps, int H, int nq, int nkv, int hd, int F, int L) {
  if (R < 1 || 3 * R > DitGridArgs::kMaxRows || NL < 1 || NL > DitGridArgs::kMaxNL || steps < 1 ||
      steps > DitGridArgs::kMaxSteps)
    return false;
  if (hd != 64 || nkv < 1 || nq % nkv || H % 128 || F % 128 || L > 64 || (nq * hd) % 128 ||
      ((nq + 2 * nkv) * hd) % 4)
    return false;
  if (H > 128 * kMaxH4 || grid_ctas() <= 0 || (H + grid_ctas() - 1) / grid_ctas() > kMaxCols) return false;
  return grid_smem_bytes(R, H, F, nq, nkv, hd, L, grid_ctas()) <= 200 * 1024;
}

namespace {

template <int RW>
cudaError_t launch_rows(const DitGridArgs& a, size_t smem, cudaStream_t s) {
  static SmemOptIn opt;
  if (cudaError_t e = opt.ensure((const void*)dit_grid_kernel<RW>, smem)) return e;
  int per_sm = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, dit_grid_kernel<RW>, kThreads, smem);
  if (e != cudaSuccess || per_sm < 1) return e != cudaSuccess ? e : cudaErrorInvalidConfiguration;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid_ctas());
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: the polled hand-overs need it
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, dit_grid_kernel<RW>, a);
  if (e != cudaSuccess) (void)cudaGetLastError();
  return e;
}

}  // namespace

cudaError_t launch_dit_grid(const DitGridArgs& a, cudaStream_t s) {
  if (!dit_grid_supported(a.R, a.NL, a.steps, a.H, a.nq, a.nkv, a.hd, a.F, a.L) || !a.bar || !a.ll)
    return cudaErrorInvalidValue;
  const size_t smem = grid_smem_bytes(a.R, a.H, a.F, a.nq, a.nkv, a.hd, a.L, grid_ctas());
  switch (a.R) {
    case 1: return launch_rows<3>(a, smem, s);
    case 2: return launch_rows<6>(a, smem, s);
    case 3: return launch_rows<9>(a, smem, s);
    default: return launch_rows<12>(a, smem, s);
  }
}

}  // namespace ctts
