// vae.cu -- causal Conv1d / ConvTranspose1d (+ fused Snake) for the VAE
// decoder (audio_vae.py:43-62,73-79; rust-codec/src/conv.rs, snake.rs,
// decode.rs).
//
// Dense convolutions run as an implicit GEMM on CUDA cores:
//   y[o, t] = bias[o] + sum_{c, j} W[o, c*k + j] * snake(x[c, t + j*dil - left])
// The Snake activation of the *input* is applied while the activation tile
// is staged into shared memory (the reference runs it as a separate pass,
// snake.rs:26-36), the residual add and the final tanh are applied in the
// epilogue.  A transposed conv with kernel 2s and stride s is s such
// convolutions with k = 2, dilation 1, left pad 1 on repacked weights, each
// writing every s-th output sample (the two-GEMM decomposition of
// decode.rs:39-80 / weights.rs:133-147).  Depthwise convolutions (the
// shipped topology's front conv and residual k7 convs) run as a
// per-channel stencil over a shared-memory window.
#include "common.cuh"
#include "kernels.cuh"

namespace ctts {

namespace {

constexpr int TO = 64;   // output channels per CTA
constexpr int TT = 64;   // output positions per CTA
constexpr int TK = 16;   // reduction chunk

template <bool BF>
CTTS_DEV float ldw(const void* w, size_t i) {
  if (BF) return bf2f(reinterpret_cast<const uint16_t*>(w)[i]);
  return reinterpret_cast<const float*>(w)[i];
}

CTTS_DEV float snake1(float v, float a) {
  float s = sinf(v * a);
  return v + (1.0f / (a + 1e-9f)) * s * s;
}

// grid (ceil(Tc/TT), ceil(Cout/TO), B*nphase); 256 threads, 4x4 outputs each.
// Tc = computed positions per phase; output sample = t*ostride + phase.
template <bool BF>
__global__ void __launch_bounds__(256) conv_kernel(const ConvArgs a, int Tc, int ostride,
                                                   int nphase, long wphase) {
  __shared__ __align__(16) float Ws[TK][TO];
  __shared__ __align__(16) float Xs[TK][TT];
  grid_dep_enter();
  const int b = blockIdx.z / nphase, ph = blockIdx.z % nphase;
  const int o0 = blockIdx.y * TO, t0 = blockIdx.x * TT;
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int k = a.k, KK = a.Cin * k;
  const void* w = BF ? (const void*)(reinterpret_cast<const uint16_t*>(a.w) + ph * wphase)
                     : (const void*)(reinterpret_cast<const float*>(a.w) + ph * wphase);
  const float* xb = a.x + (size_t)b * a.Cin * a.Tin;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int j = 0; j < 4; j++) acc[i][j] = 0.0f;

  for (int kc = 0; kc < KK; kc += TK) {
#pragma unroll
    for (int e = 0; e < 4; e++) {
      int idx = tid + e * 256;        // 0..1023
      int kk = idx & (TK - 1), oo = idx >> 4;
      int o = o0 + oo, kidx = kc + kk;
      Ws[kk][oo] = (o < a.Cout && kidx < KK) ? ldw<BF>(w, (size_t)o * KK + kidx) : 0.0f;
      int tt = idx & (TT - 1), kk2 = idx >> 6;
      int kidx2 = kc + kk2;
      float v = 0.0f;
      if (kidx2 < KK && t0 + tt < Tc) {
        int c = kidx2 / k, j = kidx2 % k;
        int src = t0 + tt + a.xoff + j * a.dil - a.left;
        if (src >= 0 && src < a.Tin) {
          v = xb[(size_t)c * a.Tin + src];
          if (a.snake_alpha) v = snake1(v, a.snake_alpha[c]);
        }
      }
      Xs[kk2][tt] = v;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < TK; kk++) {
      float4 wv = *reinterpret_cast<const float4*>(&Ws[kk][ty * 4]);
      float4 xv = *reinterpret_cast<const float4*>(&Xs[kk][tx * 4]);
      float wr[4] = {wv.x, wv.y, wv.z, wv.w}, xr[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = fmaf(wr[i], xr[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; i++) {
    int o = o0 + ty * 4 + i;
    if (o >= a.Cout) continue;
    float bo = a.bias ? a.bias[o] : 0.0f;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      int t = t0 + tx * 4 + j;
      if (t >= Tc) continue;
      size_t oi = ((size_t)b * a.Cout + o) * a.Tout + (size_t)t * ostride + ph;
      float v = acc[i][j] + bo;
      if (a.res) v += a.res[oi];
      if (a.tanh_out) v = tanhf(v);
      a.y[oi] = v;
    }
  }
}

// Depthwise causal conv (groups == Cin == Cout: conv.rs:53-117 with one
// input channel per group; audio_vae.py CausalResidualUnit with
// groups = dim):
//   y[c, t] = bias[c] + sum_j w[c, j] * snake(x[c, t + xoff + j*dil - left])
// One CTA per (position block, channel, utterance); the input window of the
// block, Snake applied once per sample, is staged in shared memory.  Memory
// bound: every input sample is read once per block, every output written once.
constexpr int kDwT = 1024;  // output positions per CTA
constexpr int kDwMaxK = 16;

template <bool BF>
__global__ void __launch_bounds__(256) dw_conv_kernel(const ConvArgs a) {
  extern __shared__ float xw[];  // [kDwT + (k-1)*dil]
  grid_dep_enter();
  const int c = blockIdx.y, b = blockIdx.z, t0 = blockIdx.x * kDwT;
  const int k = a.k, dil = a.dil, span = (k - 1) * dil;
  const float* xr = a.x + ((size_t)b * a.Cin + c) * a.Tin;
  const float al = a.snake_alpha ? a.snake_alpha[c] : 0.0f;
  // xw[i] holds input position t0 + i + xoff - left
  for (int i = threadIdx.x; i < kDwT + span; i += blockDim.x) {
    const int src = t0 + i + a.xoff - a.left;
    float v = 0.0f;
    if (src >= 0 && src < a.Tin) {
      v = xr[src];
      if (a.snake_alpha) v = snake1(v, al);
    }
    xw[i] = v;
  }
  float w[kDwMaxK];
#pragma unroll
  for (int j = 0; j < kDwMaxK; j++) w[j] = j < k ? ldw<BF>(a.w, (size_t)c * k + j) : 0.0f;
  const float bo = a.bias ? a.bias[c] : 0.0f;
  __syncthreads();
  const size_t orow = ((size_t)b * a.Cout + c) * a.Tout;
  for (int i = threadIdx.x; i < kDwT; i += blockDim.x) {
    const int t = t0 + i;
    if (t >= a.Tout) break;
    float acc = bo;
#pragma unroll
    for (int j = 0; j < kDwMaxK; j++)
      if (j < k) acc = fmaf(xw[i + j * dil], w[j], acc);
    if (a.res) acc += a.res[orow + t];
    if (a.tanh_out) acc = tanhf(acc);
    a.y[orow + t] = acc;
  }
}

// Dense causal conv with ONE output channel (the decoder's last conv,
// audio_vae.py:282-292: Snake -> Conv(64 -> 1, k7) -> tanh).  A CTA stages
// the Snake-applied input window of every input channel for kOutT outputs
// in shared memory, then each thread sums its output over channels and taps
// in the (channel, tap) order of conv_kernel (bias, residual, tanh after).
constexpr int kOutT = 128;

template <bool BF>
__global__ void __launch_bounds__(kOutT) conv_out1_kernel(const ConvArgs a) {
  extern __shared__ float win[];  // [Cin][kOutT + span]
  grid_dep_enter();
  const int b = blockIdx.y, t0 = blockIdx.x * kOutT;
  const int k = a.k, dil = a.dil, span = (k - 1) * dil, W = kOutT + span;
  const float* xb = a.x + (size_t)b * a.Cin * a.Tin;
  for (int i = threadIdx.x; i < a.Cin * W; i += blockDim.x) {
    const int c = i / W, r = i - c * W;
    const int src = t0 + r + a.xoff - a.left;
    float v = 0.0f;
    if (src >= 0 && src < a.Tin) {
      v = xb[(size_t)c * a.Tin + src];
      if (a.snake_alpha) v = snake1(v, a.snake_alpha[c]);
    }
    win[i] = v;
  }
  __syncthreads();
  const int t = t0 + threadIdx.x;
  if (t >= a.Tout) return;
  float acc = 0.0f;
  for (int c = 0; c < a.Cin; c++) {
    const float* wr = win + (size_t)c * W + threadIdx.x;
    for (int j = 0; j < k; j++) acc = fmaf(ldw<BF>(a.w, (size_t)c * k + j), wr[j * dil], acc);
  }
  const size_t oi = (size_t)b * a.Tout + t;
  float v = acc + (a.bias ? a.bias[0] : 0.0f);
  if (a.res) v += a.res[oi];
  if (a.tanh_out) v = tanhf(v);
  a.y[oi] = v;
}

__global__ void snake_kernel(const float* x, int C, int T, const float* alpha, float* y,
                             size_t n) {
  grid_dep_enter();
  size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  int c = (int)((i / T) % C);
  y[i] = snake1(x[i], alpha[c]);
}

}  // namespace

cudaError_t launch_conv1d(const ConvArgs& a, cudaStream_t s) {
  if (a.Tout + a.xoff != a.Tin || a.xoff < 0) return cudaErrorInvalidValue;
  if (a.groups != 1) {  // depthwise
    if (a.groups != a.Cin || a.Cin != a.Cout || a.k < 1 || a.k > kDwMaxK || a.dil < 1) return cudaErrorInvalidValue;
    const size_t smem = sizeof(float) * (size_t)(kDwT + (a.k - 1) * a.dil);
    if (smem > 48 * 1024) return cudaErrorInvalidValue;
    dim3 grid((a.Tout + kDwT - 1) / kDwT, a.Cout, a.B);
    if (a.w_bf16)
      CTTS_LK(launch_k(dw_conv_kernel<true>, grid, dim3(256), smem, s, a));
    else
      CTTS_LK(launch_k(dw_conv_kernel<false>, grid, dim3(256), smem, s, a));
    return cudaGetLastError();
  }
  if (conv_tc_supported(a)) return launch_conv_tc(a, a.Tout, 1, 1, s);
  const size_t win = sizeof(float) * (size_t)a.Cin * (kOutT + (a.k - 1) * a.dil);
  if (a.Cout == 1 && win <= 48 * 1024) {
    dim3 g1((a.Tout + kOutT - 1) / kOutT, a.B);
    if (a.w_bf16)
      CTTS_LK(launch_k(conv_out1_kernel<true>, g1, dim3(kOutT), win, s, a));
    else
      CTTS_LK(launch_k(conv_out1_kernel<false>, g1, dim3(kOutT), win, s, a));
    return cudaGetLastError();
  }
  dim3 grid((a.Tout + TT - 1) / TT, (a.Cout + TO - 1) / TO, a.B);
  if (a.w_bf16)
    CTTS_LK(launch_k(conv_kernel<true>, dim3(grid), dim3(256), 0, s, a, a.Tout, 1, 1, 0));
  else
    CTTS_LK(launch_k(conv_kernel<false>, dim3(grid), dim3(256), 0, s, a, a.Tout, 1, 1, 0));
  return cudaGetLastError();
}

// a.w: repacked [stride][Cout][Cin*2] (tap 0 <- x[i-1], tap 1 <- x[i]);
// a.k must be 2, a.dil 1, a.left 1; Tout = Tin * stride.
cudaError_t launch_conv_transpose(const ConvArgs& a, cudaStream_t s) {
  const int Tc = a.Tin - a.xoff;  // input positions that produce output
  if (a.k != 2 || a.xoff < 0 || a.Tout != Tc * a.stride) return cudaErrorInvalidValue;
  if (conv_tc_supported(a)) return launch_conv_tc(a, Tc, a.stride, a.stride, s);
  dim3 grid((Tc + TT - 1) / TT, (a.Cout + TO - 1) / TO, a.B * a.stride);
  long wphase = (long)a.Cout * a.Cin * 2;
  if (a.w_bf16)
    CTTS_LK(launch_k(conv_kernel<true>, dim3(grid), dim3(256), 0, s, a, Tc, a.stride, a.stride, wphase));
  else
    CTTS_LK(launch_k(conv_kernel<false>, dim3(grid), dim3(256), 0, s, a, Tc, a.stride, a.stride, wphase));
  return cudaGetLastError();
}

namespace {
__global__ void stream_ext_kernel(const float* hist_in, const float* x, float* ext, float* hist_out, int H, int T,
                                  size_t rows) {
  grid_dep_enter();
  const size_t row = blockIdx.x;
  if (row >= rows) return;
  const float* hi = hist_in + row * H;
  const float* xi = x + row * T;
  float* e = ext + row * (H + T);
  for (int i = threadIdx.x; i < H + T; i += blockDim.x) e[i] = i < H ? hi[i] : xi[i - H];
  // the last H columns of [hist ++ x]
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    const int src = T + i;
    hist_out[row * H + i] = src < H ? hi[src] : xi[src - H];
  }
}
}  // namespace

cudaError_t launch_stream_ext(const float* hist_in, const float* x, float* ext, float* hist_out, int B, int C,
                              int H, int T, cudaStream_t s) {
  const size_t rows = (size_t)B * C;
  if (!rows || H <= 0 || T <= 0 || hist_in == hist_out) return cudaErrorInvalidValue;
  CTTS_LK(launch_k(stream_ext_kernel, dim3((unsigned)rows), dim3(128), 0, s, hist_in, x, ext, hist_out, H, T, rows));
  return cudaGetLastError();
}

cudaError_t launch_snake(const float* x, int B, int C, int T, const float* alpha, float* y,
                         cudaStream_t s) {
  size_t n = (size_t)B * C * T;
  if (!n) return cudaSuccess;
  CTTS_LK(launch_k(snake_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, s, x, C, T, alpha, y, n));
  return cudaGetLastError();
}

}  // namespace ctts
