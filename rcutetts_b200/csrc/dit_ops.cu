// dit_ops.cu -- small DiT-head kernels (the linears run through linear.cu).
//
// dit_attn: LocalSelfAttention over the per-utterance [mu, cond, x] sequence
//   (diffusion_head.py:163-195, dit.rs:366-405): RoPE at positions 0..S-1,
//   bidirectional softmax, GQA head sharing.  One warp per (utterance, head);
//   q/k/v of all S tokens live in registers.
// sin_emb: SinusoidalPosEmb (diffusion_head.py:306-320, dit.rs:262-273).
// seq_fill: seq row 0 = (mu + t_emb) + dt_emb, rows 1..P = cond_proj(cond)
//   (diffusion_head.py:628-632).
#include <cmath>

#include "common.cuh"
#include "kernels.cuh"

namespace ctts {

namespace {

constexpr int kMaxS = 5;
constexpr int kPer = 4;  // head_dim <= 128

__global__ void __launch_bounds__(32) dit_attn_kernel(const float* qkv, int S, int nq, int nkv,
                                                      int hd, const float* inv_freq,
                                                      float* out, uint16_t* out_b) {
  grid_dep_enter();
  const int b = blockIdx.x, h = blockIdx.y, lane = threadIdx.x;
  const int G = nq / nkv, kh = h / G;
  const int width = (nq + 2 * nkv) * hd;
  const int per = hd / 32, half = per / 2;
  float q[kMaxS][kPer], k[kMaxS][kPer], v[kMaxS][kPer];
#pragma unroll
  for (int s = 0; s < kMaxS; s++) {
    if (s >= S) break;
    const float* row = qkv + (size_t)(b * S + s) * width;
#pragma unroll
    for (int j = 0; j < kPer; j++) {
      if (j >= per) break;
      q[s][j] = row[h * hd + lane + 32 * j];
      k[s][j] = row[(nq + kh) * hd + lane + 32 * j];
      v[s][j] = row[(nq + nkv + kh) * hd + lane + 32 * j];
    }
    // RoPE at position s (dit.rs:277-306)
#pragma unroll
    for (int j = 0; j < kPer / 2; j++) {
      if (j >= half) break;
      float ang = (float)s * inv_freq[lane + 32 * j];
      float sn, cs;
      sincosf(ang, &sn, &cs);
      float a1 = q[s][j], a2 = q[s][j + half];
      q[s][j] = a1 * cs - a2 * sn;
      q[s][j + half] = a1 * sn + a2 * cs;
      a1 = k[s][j];
      a2 = k[s][j + half];
      k[s][j] = a1 * cs - a2 * sn;
      k[s][j + half] = a1 * sn + a2 * cs;
    }
  }
  const float scale = 1.0f / sqrtf((float)hd);
#pragma unroll
  for (int i = 0; i < kMaxS; i++) {
    if (i >= S) break;
    float sc[kMaxS];
    float m = -INFINITY;
#pragma unroll
    for (int j2 = 0; j2 < kMaxS; j2++) {
      if (j2 >= S) break;
      float d = 0.0f;
#pragma unroll
      for (int j = 0; j < kPer; j++)
        if (j < per) d = fmaf(q[i][j], k[j2][j], d);
      sc[j2] = warp_sum(d) * scale;
      m = fmaxf(m, sc[j2]);
    }
    float l = 0.0f;
#pragma unroll
    for (int j2 = 0; j2 < kMaxS; j2++) {
      if (j2 >= S) break;
      sc[j2] = expf(sc[j2] - m);
      l += sc[j2];
    }
    const float inv = 1.0f / l;
    const size_t obase = (size_t)(b * S + i) * nq * hd + h * hd;
#pragma unroll
    for (int j = 0; j < kPer; j++) {
      if (j >= per) break;
      float acc = 0.0f;
#pragma unroll
      for (int j2 = 0; j2 < kMaxS; j2++) {
        if (j2 >= S) break;
        acc = fmaf(sc[j2] * inv, v[j2][j], acc);
      }
      if (out_b)
        out_b[obase + lane + 32 * j] = f2bf(acc);
      else
        out[obase + lane + 32 * j] = acc;
    }
  }
}

__global__ void sin_emb_kernel(const float* t, int H, float e, float* out) {
  grid_dep_enter();
  const int r = blockIdx.x, half = H / 2;
  const float x = t[r];
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    float f = expf((float)i * -e);
    float v = (1000.0f * x) * f;
    out[(size_t)r * H + i] = sinf(v);
    out[(size_t)r * H + half + i] = cosf(v);
  }
}

__global__ void seq_fill_kernel(float* seq, const float* mu, const float* temb,
                                const float* dtemb, const float* condh, int P, int H) {
  grid_dep_enter();
  const int b = blockIdx.x, S = 1 + 2 * P;
  float* base = seq + (size_t)b * S * H;
  for (int n = threadIdx.x; n < H; n += blockDim.x) {
    base[n] = (mu[(size_t)b * H + n] + temb[n]) + dtemb[n];
    for (int p = 0; p < P; p++) base[(size_t)(1 + p) * H + n] = condh[((size_t)b * P + p) * H + n];
  }
}

__global__ void affine_kernel(const float* x, int n, float scale, float bias, float* out) {
  grid_dep_enter();
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = x[i] / scale - bias;
}

__global__ void cfg_euler_kernel(float* x, const float* v2, int n, float cfg, float dt) {
  grid_dep_enter();
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    float vc = v2[i], vu = v2[n + i];
    x[i] += (vc + cfg * (vc - vu)) * dt;
  }
}

__global__ void fill_tv_kernel(float* tv, TGrid g) {
  grid_dep_enter();
  int i = threadIdx.x;
  if (i < g.n) tv[i] = g.t[i];
}

__global__ void add_rows_kernel(float* x, int R, int H, const float* v) {
  grid_dep_enter();
  int r = blockIdx.x;
  for (int n = threadIdx.x; n < H; n += blockDim.x) x[(size_t)r * H + n] += v[n];
}

template <bool BF>
CTTS_DEV float ldw(const void* w, size_t i) {
  if (BF) return bf2f(reinterpret_cast<const uint16_t*>(w)[i]);
  return reinterpret_cast<const float*>(w)[i];
}

constexpr int kTailThreads = 512;

// Dot product of a weight row (f32 or bf16, 16-byte aligned, n % 8 == 0)
// with an fp32 vector in shared memory, lane-strided over 8-element groups
// starting at group g0 with stride gs; every load of the row is issued
// before the first multiply.
template <bool BF, int MAXG>
CTTS_DEV float row_dot(const void* w, size_t off, const float* xs, int n, int g0, int gs) {
  float v[MAXG][8];
  const int ng = n >> 3;
#pragma unroll
  for (int i = 0; i < MAXG; i++) {
    const int g = g0 + i * gs;
    if (g < ng) {
      if (BF) {
        uint4 t = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(w) + off + g * 8);
        v[i][0] = bf_lo(t.x); v[i][1] = bf_hi(t.x); v[i][2] = bf_lo(t.y); v[i][3] = bf_hi(t.y);
        v[i][4] = bf_lo(t.z); v[i][5] = bf_hi(t.z); v[i][6] = bf_lo(t.w); v[i][7] = bf_hi(t.w);
      } else {
        const float* p = reinterpret_cast<const float*>(w) + off + g * 8;
        float4 t0 = *reinterpret_cast<const float4*>(p), t1 = *reinterpret_cast<const float4*>(p + 4);
        v[i][0] = t0.x; v[i][1] = t0.y; v[i][2] = t0.z; v[i][3] = t0.w;
        v[i][4] = t1.x; v[i][5] = t1.y; v[i][6] = t1.z; v[i][7] = t1.w;
      }
    }
  }
  float acc = 0.0f;
#pragma unroll
  for (int i = 0; i < MAXG; i++) {
    const int g = g0 + i * gs;
    if (g < ng)
#pragma unroll
      for (int e = 0; e < 8; e++) acc = fmaf(v[i][e], xs[g * 8 + e], acc);
  }
  return acc;
}

// grid R (one CTA per utterance), 512 threads.  Requires H % 8 == 0,
// L % 8 == 0, H <= 1024, L <= 64 (host-checked).
template <bool BF>
__global__ void __launch_bounds__(kTailThreads) dit_tail_kernel(const DitTailArgs a) {
  extern __shared__ __align__(16) float sm[];  // xn [P][H], xs [P*L]
  grid_dep_enter();
  const int b = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int NW = kTailThreads / 32;
  const int P = a.P, H = a.H, L = a.L, S = 1 + 2 * P, PL = P * L;
  float* xn = sm;
  float* xs = sm + P * H;
  __shared__ float red[NW];
  float* seqb = a.seq + (size_t)b * S * H;
  float* xb = a.x + (size_t)b * PL;
  if (a.do_out) {
    for (int p = 0; p < P; p++) {
      const float* row = seqb + (size_t)(1 + P + p) * H;
      const float v0 = tid < H ? row[tid] : 0.0f, v1 = tid + kTailThreads < H ? row[tid + kTailThreads] : 0.0f;
      float ss = warp_sum(fmaf(v0, v0, v1 * v1));
      if (lane == 0) red[warp] = ss;
      __syncthreads();
      float tot = 0.0f;
#pragma unroll
      for (int w = 0; w < NW; w++) tot += red[w];
      const float inv = 1.0f / sqrtf(tot / (float)H + a.eps);
      if (tid < H) xn[p * H + tid] = v0 * inv * a.final_norm[tid];
      if (tid + kTailThreads < H) xn[p * H + tid + kTailThreads] = v1 * inv * a.final_norm[tid + kTailThreads];
      __syncthreads();
    }
    // out_proj: a warp per output, lanes over 8-element groups of H (<= 4 each)
    for (int o = warp; o < PL; o += NW) {
      const int p = o / L, l = o % L;
      float acc = row_dot<BF, 4>(a.out_w, (size_t)l * H, xn + p * H, H, lane, 32);
      acc = warp_sum(acc);
      if (lane == 0) xb[o] = xb[o] + a.dt * (acc + (a.out_b ? a.out_b[l] : 0.0f));
    }
    __syncthreads();
  }
  if (!a.fill) return;
  for (int i = tid; i < PL; i += kTailThreads) xs[i] = xb[i];
  __syncthreads();
  // in_proj: a thread per output row n, the whole weight row (<= 64) in flight
  for (int n = tid; n < H; n += kTailThreads) {
    for (int p = 0; p < P; p++) {
      const float acc = row_dot<BF, 8>(a.in_w, (size_t)n * L, xs + p * L, L, 0, 1);
      seqb[(size_t)(1 + P + p) * H + n] = acc + (a.in_b ? a.in_b[n] : 0.0f);
    }
    seqb[n] = (a.mu[(size_t)b * H + n] + a.temb[n]) + a.dtemb[n];
    for (int p = 0; p < P; p++) seqb[(size_t)(1 + p) * H + n] = a.condh[((size_t)b * P + p) * H + n];
  }
}

}  // namespace

cudaError_t launch_dit_tail(const DitTailArgs& a, cudaStream_t s) {
  if (a.R <= 0) return cudaSuccess;
  const size_t smem = ((size_t)a.P * a.H + (size_t)a.P * a.L) * sizeof(float);
  if (smem > 48 * 1024 || a.H % 8 || a.L % 8 || a.H > 1024 || a.L > 64) return cudaErrorInvalidValue;
  if (a.w_bf16)
    CTTS_LK(launch_k(dit_tail_kernel<true>, dim3(a.R), dim3(kTailThreads), smem, s, a));
  else
    CTTS_LK(launch_k(dit_tail_kernel<false>, dim3(a.R), dim3(kTailThreads), smem, s, a));
  return cudaSuccess;
}

cudaError_t launch_fill_tv(float* tv, const TGrid& g, cudaStream_t s) {
  if (g.n > TGrid::kMax) return cudaErrorInvalidValue;
  CTTS_LK(launch_k(fill_tv_kernel, dim3(1), dim3(TGrid::kMax), 0, s, tv, g));
  return cudaGetLastError();
}

cudaError_t launch_add_rows(float* x, int R, int H, const float* v, cudaStream_t s) {
  if (R <= 0) return cudaSuccess;
  CTTS_LK(launch_k(add_rows_kernel, dim3(R), dim3(256), 0, s, x, R, H, v));
  return cudaGetLastError();
}

cudaError_t launch_dit_attn(const float* qkv, int B, int S, int nq, int nkv, int hd,
                            const float* inv_freq, float* out, uint16_t* out_b, cudaStream_t s) {
  if (S > kMaxS || hd % 64 != 0 || hd > 32 * kPer || nq % nkv) return cudaErrorInvalidValue;
  CTTS_LK(launch_k(dit_attn_kernel, dim3(B, nq), dim3(32), 0, s, qkv, S, nq, nkv, hd, inv_freq, out, out_b));
  return cudaGetLastError();
}

cudaError_t launch_sin_emb(const float* t, int rows, int H, float* out, cudaStream_t s) {
  const int half = H / 2;
  const float e = (float)(std::log(10000.0) / (double)(half - 1));
  CTTS_LK(launch_k(sin_emb_kernel, dim3(rows), dim3(256), 0, s, t, H, e, out));
  return cudaGetLastError();
}

cudaError_t launch_dit_seq_fill(float* seq, const float* mu, const float* temb,
                                const float* dtemb, const float* condh, int B, int P, int H,
                                cudaStream_t s) {
  CTTS_LK(launch_k(seq_fill_kernel, dim3(B), dim3(256), 0, s, seq, mu, temb, dtemb, condh, P, H));
  return cudaGetLastError();
}

cudaError_t launch_affine(const float* x, int n, float scale, float bias, float* out,
                          cudaStream_t s) {
  CTTS_LK(launch_k(affine_kernel, dim3((n + 255) / 256), dim3(256), 0, s, x, n, scale, bias, out));
  return cudaGetLastError();
}

cudaError_t launch_cfg_euler(float* x, const float* v2, int n, float cfg, float dt,
                             cudaStream_t s) {
  CTTS_LK(launch_k(cfg_euler_kernel, dim3((n + 255) / 256), dim3(256), 0, s, x, v2, n, cfg, dt));
  return cudaGetLastError();
}

}  // namespace ctts
