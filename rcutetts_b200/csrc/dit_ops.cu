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

}  // namespace

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
