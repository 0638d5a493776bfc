// linear.cu -- skinny linear layers on CUDA cores (the decode GEMV path).
//
// Replaces the reference's packed-panel GEMV / small-T SGEMM
// (rust-codec/src/qwen.rs:177-221 linear_gemv, simd.rs:333-387 gemv8,
// gemm.rs:149-221 sgemm_small_t, dit.rs:184-206 linear_rows).  At decode the
// contraction has 1..8 activation rows per weight row, so it is bound by
// streaming W from HBM (or L2): each warp owns RPW weight rows and reads
// them with 16-byte non-allocating loads, the activation tile (up to 8 rows,
// RMSNorm / AdaLN-modulate prologue already applied) sits in shared memory
// and is broadcast to every lane, partial sums are reduced with warp
// shuffles.  The epilogue fuses bias, SiLU / SwiGLU, residual add, AdaLN
// gated residual and the Euler update (y += dt * v).
#include <algorithm>
#include <cstdlib>

#include "common.cuh"
#include "launch_state.h"
#include "kernels.cuh"

namespace ctts {

namespace {

constexpr int kWarps = 4;

template <bool BF16>
struct WVec;
template <>
struct WVec<false> {
  static constexpr int N = 4;
  static CTTS_DEV void load(const void* base, size_t off, float* v) {
    float4 t = ld_stream_f4(reinterpret_cast<const float*>(base) + off);
    v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
  }
};
template <>
struct WVec<true> {
  static constexpr int N = 8;
  static CTTS_DEV void load(const void* base, size_t off, float* v) {
    uint4 t = ld_stream_u4(reinterpret_cast<const uint16_t*>(base) + off);
    v[0] = bf_lo(t.x); v[1] = bf_hi(t.x); v[2] = bf_lo(t.y); v[3] = bf_hi(t.y);
    v[4] = bf_lo(t.z); v[5] = bf_hi(t.z); v[6] = bf_lo(t.w); v[7] = bf_hi(t.w);
  }
};

CTTS_DEV const float* row_in(const float* base, int m, int div, long ld, long ld_outer) {
  return base + (long)(m / div) * ld_outer + (long)(m % div) * ld;
}

template <bool BF16, int MT, int RPW, bool SWIGLU>
__global__ void __launch_bounds__(kWarps * 32) linear_rows_kernel(const LinearArgs a) {
  extern __shared__ __align__(16) float xs[];  // [MT][K]
  constexpr int VEC = WVec<BF16>::N;
  const int K = a.K;
  const int m0 = blockIdx.y * MT;
  const int mt = min(MT, a.M - m0);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;

  grid_dep_enter();
  // ---- prologue: stage the activation tile (RMSNorm + modulate)
  for (int r = warp; r < MT; r += kWarps) {
    float* dst = xs + r * K;
    if (r >= mt) {
      for (int k = lane; k < K; k += 32) dst[k] = 0.0f;
      continue;
    }
    const int m = m0 + r;
    const float* xr = row_in(a.x, m, a.x_div, a.x_ld, a.x_ld_outer);
    const float* md0 = a.mod ? a.mod + (long)(m / a.mod_div) * a.mod_ld : nullptr;
    if ((K & 127) == 0 && K <= 2048 && (reinterpret_cast<uintptr_t>(xr) & 15) == 0) {
      // register-resident row: all loads in flight at once
      float4 v[16];
      const float ss = warp_load_row<16>(xr, K, v);
      const float inv = a.norm_w ? 1.0f / sqrtf(ss / (float)K + a.eps) : 1.0f;
#pragma unroll
      for (int i = 0; i < 16; i++) {
        if (i >= (K >> 7)) break;
        const int k = lane * 4 + 128 * i;
        float e[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
        for (int j = 0; j < 4; j++) {
          if (a.norm_w) e[j] = e[j] * inv * a.norm_w[k + j];
          if (md0) e[j] = e[j] * (1.0f + md0[a.mod_scale + k + j]) + md0[a.mod_shift + k + j];
        }
        *reinterpret_cast<float4*>(dst + k) = make_float4(e[0], e[1], e[2], e[3]);
      }
      continue;
    }
    float inv = 1.0f;
    if (a.norm_w) {
      float ss = 0.0f;
      for (int k = lane; k < K; k += 32) ss = fmaf(xr[k], xr[k], ss);
      ss = warp_sum(ss);
      inv = 1.0f / sqrtf(ss / (float)K + a.eps);
    }
    const float* md = a.mod ? a.mod + (long)(m / a.mod_div) * a.mod_ld : nullptr;
    for (int k = lane; k < K; k += 32) {
      float v = xr[k];
      if (a.norm_w) v = v * inv * a.norm_w[k];
      if (md) v = v * (1.0f + md[a.mod_scale + k]) + md[a.mod_shift + k];
      dst[k] = v;
    }
  }
  __syncthreads();

  const int n0 = (blockIdx.x * kWarps + warp) * RPW;
  if (n0 >= a.N) return;

  float acc[RPW][MT];
  float acc2[SWIGLU ? RPW : 1][MT];
#pragma unroll
  for (int r = 0; r < RPW; r++)
#pragma unroll
    for (int m = 0; m < MT; m++) {
      acc[r][m] = 0.0f;
      if (SWIGLU) acc2[r][m] = 0.0f;
    }

  // SwiGLU weights are stored tile-interleaved (64 gate rows, then the 64
  // matching up rows): gate row n sits at (n/64)*128 + n%64, up at +64.
  int nr[RPW];
#pragma unroll
  for (int r = 0; r < RPW; r++) {
    const int n = min(n0 + r, a.N - 1);
    nr[r] = SWIGLU ? (n >> 6) * 128 + (n & 63) : n;
  }

#pragma unroll 4
  for (int k = lane * VEC; k < K; k += 32 * VEC) {
    float wv[RPW][VEC];
    float wu[SWIGLU ? RPW : 1][VEC];
#pragma unroll
    for (int r = 0; r < RPW; r++) {
      WVec<BF16>::load(a.w, (size_t)nr[r] * K + k, wv[r]);
      if (SWIGLU) WVec<BF16>::load(a.w, (size_t)(nr[r] + 64) * K + k, wu[r]);
    }
#pragma unroll
    for (int m = 0; m < MT; m++) {
      float xv[VEC];
#pragma unroll
      for (int v4 = 0; v4 < VEC; v4 += 4) {
        float4 t = *reinterpret_cast<const float4*>(xs + m * K + k + v4);
        xv[v4] = t.x; xv[v4 + 1] = t.y; xv[v4 + 2] = t.z; xv[v4 + 3] = t.w;
      }
#pragma unroll
      for (int r = 0; r < RPW; r++)
#pragma unroll
        for (int v = 0; v < VEC; v++) {
          acc[r][m] = fmaf(wv[r][v], xv[v], acc[r][m]);
          if (SWIGLU) acc2[r][m] = fmaf(wu[r][v], xv[v], acc2[r][m]);
        }
    }
  }

#pragma unroll
  for (int r = 0; r < RPW; r++)
#pragma unroll
    for (int m = 0; m < MT; m++) {
      acc[r][m] = warp_sum(acc[r][m]);
      if (SWIGLU) acc2[r][m] = warp_sum(acc2[r][m]);
    }

#pragma unroll
  for (int r = 0; r < RPW; r++) {
#pragma unroll
    for (int m = 0; m < MT; m++) {
      if (((r * MT + m) & 31) != lane) continue;
      const int n = n0 + r, mm = m0 + m;
      if (n >= a.N || m >= mt) continue;
      float val = acc[r][m] + (a.bias ? a.bias[SWIGLU ? nr[r] : n] : 0.0f);
      if (SWIGLU) {
        float u = acc2[r][m] + (a.bias ? a.bias[nr[r] + 64] : 0.0f);
        val = silu(val) * u;
      } else if (a.act == 1) {
        val = silu(val);
      }
      float coef = a.gate ? 1.0f + a.gate[(long)(mm / a.gate_div) * a.gate_ld + a.gate_off + n]
                          : a.scale;
      float* yr = const_cast<float*>(row_in(a.y, mm, a.y_div, a.y_ld, a.y_ld_outer));
      float out = coef * val;
      if (a.res) out = row_in(a.res, mm, a.y_div, a.y_ld, a.y_ld_outer)[n] + out;
      yr[n] = out;
    }
  }
}

// Short contractions (K <= 128, fp32 or bf16 weights, no prologue, no
// SwiGLU): the latent-sized projections of a frame (the feedback and the
// DiT condition projections have K = 64).
// The form above splits K over the lanes and shuffle-reduces RPW x MT
// accumulators per warp, which at such K leaves half the lanes idle and
// runs a large unrolled body.  Here a thread owns one output column for MT
// activation rows and walks K in order with fmaf from zero -- the same
// order for every batch size, so a row's result does not depend on the
// batch it runs in; the CTA's NC weight rows are staged transposed in
// shared memory ([K][NC + 1], a warp reads 32 consecutive columns) and its
// activation rows as [MT][K] (broadcast reads).  NC = 128 from 8 rows, 32
// (one warp per CTA, more CTAs) below.  grid (ceil(N / NC), ceil(M / MT)).
template <int MT, int NC, bool BF16>
__global__ void __launch_bounds__(NC) linear_smallk_kernel(const LinearArgs a) {
  constexpr int kSkCols = NC, kSkLd = NC + 1;
  extern __shared__ __align__(16) float sk[];
  const int K = a.K, K4 = K / 4;
  float* xs = sk;           // [MT][K]
  float* wt = sk + MT * K;  // [K][kSkLd]
  const int n0 = blockIdx.x * kSkCols, m0 = blockIdx.y * MT;
  const int mt = min(MT, a.M - m0);
  const int tid = threadIdx.x;
  grid_dep_enter();
  if constexpr (BF16) {  // 8 weights per 16-byte load, widened exactly
    const uint16_t* W = static_cast<const uint16_t*>(a.w);
    const int K8 = K / 8;
    for (int i = tid; i < kSkCols * K8; i += kSkCols) {
      const int n = i / K8, k = (i % K8) * 8;
      uint4 t = make_uint4(0u, 0u, 0u, 0u);
      if (n0 + n < a.N) t = *reinterpret_cast<const uint4*>(W + (size_t)(n0 + n) * K + k);
      const uint32_t u[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
      for (int j = 0; j < 4; j++) {
        wt[(k + 2 * j) * kSkLd + n] = bf_lo(u[j]);
        wt[(k + 2 * j + 1) * kSkLd + n] = bf_hi(u[j]);
      }
    }
  } else {
    const float* W = static_cast<const float*>(a.w);
    for (int i = tid; i < kSkCols * K4; i += kSkCols) {
      const int n = i / K4, k = (i % K4) * 4;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (n0 + n < a.N) v = *reinterpret_cast<const float4*>(W + (size_t)(n0 + n) * K + k);
      wt[(k + 0) * kSkLd + n] = v.x;
      wt[(k + 1) * kSkLd + n] = v.y;
      wt[(k + 2) * kSkLd + n] = v.z;
      wt[(k + 3) * kSkLd + n] = v.w;
    }
  }
  for (int i = tid; i < MT * K; i += kSkCols) {
    const int r = i / K, k = i % K;
    xs[i] = r < mt ? row_in(a.x, m0 + r, a.x_div, a.x_ld, a.x_ld_outer)[k] : 0.0f;
  }
  __syncthreads();
  const int n = n0 + tid;
  if (n >= a.N) return;
  float acc[MT];
#pragma unroll
  for (int m = 0; m < MT; m++) acc[m] = 0.0f;
#pragma unroll 4
  for (int k = 0; k < K; k++) {
    const float w = wt[k * kSkLd + tid];
#pragma unroll
    for (int m = 0; m < MT; m++) acc[m] = fmaf(w, xs[m * K + k], acc[m]);
  }
  const float b = a.bias ? a.bias[n] : 0.0f;
#pragma unroll
  for (int m = 0; m < MT; m++) {
    if (m >= mt) break;
    const int mm = m0 + m;
    float val = acc[m] + b;
    if (a.act == 1) val = silu(val);
    const float coef = a.gate ? 1.0f + a.gate[(long)(mm / a.gate_div) * a.gate_ld + a.gate_off + n] : a.scale;
    float* yr = const_cast<float*>(row_in(a.y, mm, a.y_div, a.y_ld, a.y_ld_outer));
    float out = coef * val;
    if (a.res) out = row_in(a.res, mm, a.y_div, a.y_ld, a.y_ld_outer)[n] + out;
    yr[n] = out;
  }
}

// One warp per row: y = bf16( modulate( RMSNorm(x) ) ), the tensor-core
// path's activation operand.
__global__ void __launch_bounds__(128) prep_bf16_kernel(const PrepArgs a) {
  grid_dep_enter();
  const int row = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= a.M) return;
  const float* xr = a.x + (long)row * a.x_ld;
  const float* md = a.mod ? a.mod + (long)(row / a.mod_div) * a.mod_ld : nullptr;
  uint16_t* yr = a.y + (long)row * a.y_ld;
  if ((a.K & 127) == 0 && a.K <= 2048 && (reinterpret_cast<uintptr_t>(xr) & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(yr) & 7) == 0) {
    float4 v[16];
    const float ss = warp_load_row<16>(xr, a.K, v);
    const float inv = a.norm_w ? 1.0f / sqrtf(ss / (float)a.K + a.eps) : 1.0f;
#pragma unroll
    for (int i = 0; i < 16; i++) {
      if (i >= (a.K >> 7)) break;
      const int k = lane * 4 + 128 * i;
      float e[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
      for (int j = 0; j < 4; j++) {
        if (a.norm_w) e[j] = e[j] * inv * a.norm_w[k + j];
        if (md) e[j] = e[j] * (1.0f + md[a.mod_scale + k + j]) + md[a.mod_shift + k + j];
      }
      uint2 pk;
      pk.x = (uint32_t)f2bf(e[0]) | ((uint32_t)f2bf(e[1]) << 16);
      pk.y = (uint32_t)f2bf(e[2]) | ((uint32_t)f2bf(e[3]) << 16);
      *reinterpret_cast<uint2*>(yr + k) = pk;
    }
    return;
  }
  float inv = 1.0f;
  if (a.norm_w) {
    float ss = 0.0f;
    for (int k = lane; k < a.K; k += 32) ss = fmaf(xr[k], xr[k], ss);
    ss = warp_sum(ss);
    inv = 1.0f / sqrtf(ss / (float)a.K + a.eps);
  }
  for (int k = lane; k < a.K; k += 32) {
    float v = xr[k];
    if (a.norm_w) v = v * inv * a.norm_w[k];
    if (md) v = v * (1.0f + md[a.mod_scale + k]) + md[a.mod_shift + k];
    yr[k] = f2bf(v);
  }
}

template <bool BF16, int MT, int RPW, bool SWIGLU>
cudaError_t launch_t(const LinearArgs& a, cudaStream_t s) {
  auto kern = linear_rows_kernel<BF16, MT, RPW, SWIGLU>;
  size_t smem = (size_t)MT * a.K * sizeof(float);
  static SmemOptIn opt;
  if (cudaError_t e = opt.ensure((const void*)kern, 200 * 1024)) return e;
  dim3 grid((a.N + kWarps * RPW - 1) / (kWarps * RPW), (a.M + MT - 1) / MT);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kWarps * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

int pick_mt(int M) { return M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : 8; }
// a handful of output columns (a stop head: N = 2): one activation row per
// CTA, so the rows spread over the GPU instead of idling most warps of few CTAs
int pick_mt(const LinearArgs& a) { return a.N <= 16 ? 1 : pick_mt(a.M); }

bool smallk(const LinearArgs& a) {
  return a.act != 2 && !a.norm_w && !a.mod && a.K <= 128 && a.K % (a.w_bf16 ? 8 : 4) == 0;
}

template <int MT, int NC, bool BF16>
cudaError_t launch_smallk_t(const LinearArgs& a, cudaStream_t s) {
  const size_t smem = ((size_t)MT * a.K + (size_t)a.K * (NC + 1)) * sizeof(float);
  static SmemOptIn opt;
  if (cudaError_t e = opt.ensure((const void*)linear_smallk_kernel<MT, NC, BF16>, smem)) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((a.N + NC - 1) / NC, (a.M + MT - 1) / MT);
  cfg.blockDim = dim3(NC);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, linear_smallk_kernel<MT, NC, BF16>, a);
}

template <bool BF16>
cudaError_t launch_smallk_b(const LinearArgs& a, cudaStream_t s) {
  switch (pick_mt(a.M)) {
    case 1: return launch_smallk_t<1, 32, BF16>(a, s);
    case 2: return launch_smallk_t<2, 32, BF16>(a, s);
    case 4: return launch_smallk_t<4, 32, BF16>(a, s);
    default: return launch_smallk_t<8, 128, BF16>(a, s);
  }
}

cudaError_t launch_smallk(const LinearArgs& a, cudaStream_t s) {
  return a.w_bf16 ? launch_smallk_b<true>(a, s) : launch_smallk_b<false>(a, s);
}

int pick_rpw(const LinearArgs& a, int mt) {
  int gy = (a.M + mt - 1) / mt;
  for (int rpw : {4, 2}) {
    long ctas = (long)((a.N + kWarps * rpw - 1) / (kWarps * rpw)) * gy;
    if (ctas >= 2 * 148) return rpw;
  }
  return 1;
}

template <bool BF16, bool SW>
cudaError_t dispatch_mt(const LinearArgs& a, cudaStream_t s) {
  int mt = pick_mt(a);
  int rpw = pick_rpw(a, mt);
#define CTTS_L(MT_)                                                     \
  if (mt == MT_) {                                                      \
    if (rpw == 4) return launch_t<BF16, MT_, 4, SW>(a, s);              \
    if (rpw == 2) return launch_t<BF16, MT_, 2, SW>(a, s);              \
    return launch_t<BF16, MT_, 1, SW>(a, s);                            \
  }
  CTTS_L(1) CTTS_L(2) CTTS_L(4) CTTS_L(8)
#undef CTTS_L
  return cudaErrorInvalidValue;
}

}  // namespace

int linear_grid_ctas(const LinearArgs& a) {
  if (smallk(a)) {
    const int mt = pick_mt(a.M), nc = mt < 8 ? 32 : 128;
    return ((a.N + nc - 1) / nc) * ((a.M + mt - 1) / mt);
  }
  int mt = pick_mt(a);
  int rpw = pick_rpw(a, mt);
  return ((a.N + kWarps * rpw - 1) / (kWarps * rpw)) * ((a.M + mt - 1) / mt);
}

bool pdl_enabled() {
  static const bool v = [] {
    const char* e = getenv("CTTS_PDL");
    return !(e && e[0] == '0');
  }();
  return v;
}

cudaError_t launch_prep_bf16(const PrepArgs& a, cudaStream_t s) {
  if (a.M <= 0) return cudaSuccess;
  CTTS_LK(launch_k(prep_bf16_kernel, dim3((a.M + 3) / 4), dim3(128), 0, s, a));
  return cudaGetLastError();
}

cudaError_t launch_linear(const LinearArgs& a, cudaStream_t s) {
  if (a.M <= 0 || a.N <= 0) return cudaSuccess;
  const int vec = a.w_bf16 ? 8 : 4;
  if (a.K <= 0 || a.K % vec != 0 || (size_t)8 * a.K * sizeof(float) > 200 * 1024)
    return cudaErrorInvalidValue;
  const bool sw = a.act == 2;
  if (smallk(a)) return launch_smallk(a, s);
  if (a.w_bf16) return sw ? dispatch_mt<true, true>(a, s) : dispatch_mt<true, false>(a, s);
  return sw ? dispatch_mt<false, true>(a, s) : dispatch_mt<false, false>(a, s);
}

}  // namespace ctts
