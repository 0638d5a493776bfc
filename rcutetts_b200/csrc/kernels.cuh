// kernels.cuh -- launch interfaces of the decode-path kernels (host side).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace ctts {

// ---------------------------------------------------------------- linear
// y[m, n] = epi( sum_k pro(x)[m, k] * W[n, k] )
// Row addressing (x, y and res): row m lives at
//   base + (m / div) * ld_outer + (m % div) * ld
// so a linear can read or write every S-th token of a packed sequence.  The
// default div (kNoDiv) makes it plain row-major: base + m * ld.
constexpr int kNoDiv = 1 << 30;
struct LinearArgs {
  const float* x = nullptr;
  long x_ld = 0, x_ld_outer = 0;
  int x_div = kNoDiv;
  const void* w = nullptr;  // [N (2N for swiglu), K], f32 or bf16 bits
  int w_bf16 = 0;
  const float* bias = nullptr;  // [N (2N)] or null
  float* y = nullptr;
  long y_ld = 0, y_ld_outer = 0;
  int y_div = kNoDiv;
  int M = 0, N = 0, K = 0;
  // prologue: RMSNorm (norm_w != null) then AdaLN modulate (mod != null):
  //   v = v * (1 + mod[b*mod_ld + mod_scale + k]) + mod[b*mod_ld + mod_shift + k], b = m / mod_div
  const float* norm_w = nullptr;
  float eps = 1e-6f;
  const float* mod = nullptr;
  long mod_ld = 0;
  int mod_div = 1, mod_shift = 0, mod_scale = 0;
  // epilogue: val = act(acc + bias); y = (res ? res[m,n] : 0) + coef * val
  //   coef = gate ? 1 + gate[(m / gate_div) * gate_ld + gate_off + n] : scale
  int act = 0;  // 0 none, 1 silu, 2 swiglu (W rows in 128-row groups: 64 gate, 64 up)
  const float* res = nullptr;
  const float* gate = nullptr;
  long gate_ld = 0;
  int gate_div = 1, gate_off = 0;
  float scale = 1.0f;
  int pdl = 0;  // launch with programmatic stream serialization
};

cudaError_t launch_linear(const LinearArgs& a, cudaStream_t s);

// bf16 activation operand for the tensor-core linears:
// y[m, k] = bf16( RMSNorm(x[m]) (norm_w != null) then AdaLN modulate (mod != null) )
struct PrepArgs {
  const float* x = nullptr;
  long x_ld = 0;
  uint16_t* y = nullptr;
  long y_ld = 0;
  int M = 0, K = 0;
  const float* norm_w = nullptr;
  float eps = 1e-6f;
  const float* mod = nullptr;
  long mod_ld = 0;
  int mod_div = 1, mod_shift = 0, mod_scale = 0;
};
cudaError_t launch_prep_bf16(const PrepArgs& a, cudaStream_t s);
// Number of CTAs launch_linear would use (for reporting).
int linear_grid_ctas(const LinearArgs& a);

// ------------------------------------------------------------- LM blocks
struct AttnArgs {
  // qkv rows [rows, (nq + 2*nkv) * hd] (raw projections)
  const float* qkv = nullptr;
  int rows = 0;  // decode: batch; prefill: T
  int prefill_b = -1;  // >=0: all rows belong to utterance prefill_b at pos0 + r
  int pos0 = 0;
  int* pos = nullptr;  // [batch] device positions (== cache length before append)
  int nq = 0, nkv = 0, hd = 0;
  const float* qn = nullptr;  // QK-Norm gains [hd] or null
  const float* kn = nullptr;
  float eps = 1e-6f;
  const float* inv_freq = nullptr;  // [hd/2]
  void* kcache = nullptr;  // this layer: [batch][nkv][cap][hd]
  void* vcache = nullptr;
  int kv_bf16 = 0;
  int cap = 0;
  int batch = 0;
  float* qrot = nullptr;  // [rows, nq*hd] rotated queries
  float* out = nullptr;   // [rows, nq*hd] attention output (fp32) ...
  uint16_t* out_b = nullptr;  // ... or bf16 when set
  float* part = nullptr;  // split partials [batch][nq][nsplit][hd+2]
  int* cnt = nullptr;     // [batch][nkv] split tickets (zero at rest)
  int nsplit = 0, chunk = 0;
  int* err = nullptr;     // device error flag (capacity overflow)
};

cudaError_t launch_qk_rope_append(const AttnArgs& a, cudaStream_t s);
cudaError_t launch_attn_decode(const AttnArgs& a, cudaStream_t s);
cudaError_t launch_attn_prefill(const AttnArgs& a, cudaStream_t s);
cudaError_t launch_advance_pos(int* pos, int batch, cudaStream_t s);

cudaError_t launch_rmsnorm_rows(const float* x, int M, int K, const float* w, float eps,
                                float* y, cudaStream_t s);
cudaError_t launch_embed_gather(const void* table, int table_bf16, int vocab, int H,
                                const int64_t* ids, int n, float* out, int* bad,
                                cudaStream_t s);
cudaError_t launch_rope_inplace(float* x, int M, int heads, int hd, const int* pos,
                                const float* inv_freq, cudaStream_t s);
cudaError_t launch_swiglu(const float* gu, int M, int F, float* out, cudaStream_t s);

// -------------------------------------------------------------- DiT blocks
// attention over each utterance's S-token sequence (bidirectional, RoPE
// positions 0..S-1): qkv [B*S, (nq + 2nkv)*hd] -> out [B*S, nq*hd]
cudaError_t launch_dit_attn(const float* qkv, int B, int S, int nq, int nkv, int hd,
                            const float* inv_freq, float* out, uint16_t* out_b, cudaStream_t s);
// rows r: out[r, :] = SinusoidalPosEmb(t[r]) (dim H)
cudaError_t launch_sin_emb(const float* t, int rows, int H, float* out, cudaStream_t s);
// seq[b, 0, :] = mu[b] + temb + dtemb ; seq[b, 1..P, :] = condh[b*P..]
cudaError_t launch_dit_seq_fill(float* seq, const float* mu, const float* temb,
                                const float* dtemb, const float* condh, int B, int P, int H,
                                cudaStream_t s);
// out[i] = x[i] / scale - bias
cudaError_t launch_affine(const float* x, int n, float scale, float bias, float* out,
                          cudaStream_t s);
// device copy of a small host-computed time grid (passed by value)
struct TGrid {
  static constexpr int kMax = 96;
  int n = 0;
  float t[kMax];
};
cudaError_t launch_fill_tv(float* tv, const TGrid& g, cudaStream_t s);
// x[r, :] += v[:] for r < R
cudaError_t launch_add_rows(float* x, int R, int H, const float* v, cudaStream_t s);
// The tail of one Euler step fused with the head of the next, one CTA per
// utterance: [final RMSNorm -> out_proj -> x += dt*v] (do_out) then
// [in_proj(x) -> seq rows 1+P.., seq row 0 = mu + temb + dtemb, rows
// 1..P = cond_proj(cond)] (fill).
struct DitTailArgs {
  float* seq = nullptr;  // [R, S, H]
  float* x = nullptr;    // [R, P*L] latent, updated in place
  int R = 0, P = 1, H = 0, L = 0;
  const void* out_w = nullptr;  // [L, H]
  const float* out_b = nullptr;
  const void* in_w = nullptr;   // [H, L]
  const float* in_b = nullptr;
  int w_bf16 = 0;
  const float* final_norm = nullptr;
  float eps = 1e-6f;
  float dt = 0.0f;
  int do_out = 0, fill = 0;
  const float* mu = nullptr;     // [R, H]
  const float* temb = nullptr;   // [H] for the step being filled
  const float* dtemb = nullptr;  // [H]
  const float* condh = nullptr;  // [R*P, H]
};
cudaError_t launch_dit_tail(const DitTailArgs& a, cudaStream_t s);
// v = vc + cfg*(vc - vu) ; x += v*dt    (vc = v[0:n], vu = v[n:2n])
cudaError_t launch_cfg_euler(float* x, const float* v2, int n, float cfg, float dt,
                             cudaStream_t s);

// -------------------------------------------------------------- VAE blocks
struct ConvArgs {
  const float* x = nullptr;  // [B, Cin, Tin]
  const void* w = nullptr;   // conv: [Cout, Cin, k]; transposed: see vae.cu
  int w_bf16 = 0;
  const float* bias = nullptr;
  float* y = nullptr;        // [B, Cout, Tout]
  const float* res = nullptr;  // residual added to y (same shape) or null
  const float* snake_alpha = nullptr;  // Snake applied to x on load (per Cin) or null
  int B = 0, Cin = 0, Cout = 0, Tin = 0, Tout = 0, k = 1, dil = 1, left = 0;
  int stride = 1;   // transposed conv stride
  int groups = 1;   // 1 (dense) or Cin == Cout (depthwise); conv1d only
  int tanh_out = 0;
  int xoff = 0;     // output position t reads input position t + xoff + j*dil - left
                    // (streaming: the input carries xoff history columns)
  // bf16 tensor-core path (vae_tc.cu): the weights repacked by repack_conv_tc
  // ([phase][tap][Cin/8][cout_pad][8]); null keeps the CUDA-core kernel
  const void* w_tc = nullptr;
  int cout_pad = 0;
  int* err = nullptr;  // bounded-wait timeouts of the tensor-core path (error 5)
};
cudaError_t launch_conv1d(const ConvArgs& a, cudaStream_t s);
cudaError_t launch_conv_transpose(const ConvArgs& a, cudaStream_t s);

// Arguments of the tensor-core conv kernel (vae_tc.cu).
struct VaeTcArgs {
  const float* x = nullptr;
  const uint16_t* w = nullptr;  // [nphase][k][Cin/8][Cout_pad][8] bf16
  const float *bias = nullptr, *res = nullptr, *alpha = nullptr;
  float* y = nullptr;
  int* err = nullptr;
  int B = 0, Cin = 0, Cout = 0, Cout_pad = 0, Tin = 0, Tout = 0, Tc = 0;
  int k = 1, dil = 1, left = 0, xoff = 0, ostride = 1, nphase = 1, tanh_out = 0;
};
// True when the dense conv `a` can run on the tensor cores (bf16, repacked
// weights set, Cin a multiple of 16, Cout >= 64, (k-1)*dil <= 56, k <= 8).
bool conv_tc_supported(const ConvArgs& a);
// Tc computed positions, output index t*ostride + phase (blockIdx.z = b*nphase + phase).
cudaError_t launch_conv_tc(const ConvArgs& a, int Tc, int ostride, int nphase, cudaStream_t s);
// Repack [nphase][Cout][Cin][k] bf16 conv weights into the tensor-core layout
// [nphase][k][Cin/8][cout_pad][8] (dst zeroed beforehand: rows >= Cout stay 0).
cudaError_t repack_conv_tc(uint16_t* dst, const uint16_t* src, int nphase, int Cout, int Cin, int k, int cout_pad,
                           cudaStream_t s);
cudaError_t launch_snake(const float* x, int B, int C, int T, const float* alpha, float* y,
                         cudaStream_t s);
// Streaming history: ext[b, c, :] = hist_in[b, c, 0:H] ++ x[b, c, 0:T] and
// hist_out[b, c, :] = the last H columns of ext (hist_out != hist_in).
cudaError_t launch_stream_ext(const float* hist_in, const float* x, float* ext, float* hist_out, int B, int C,
                              int H, int T, cudaStream_t s);

}  // namespace ctts
