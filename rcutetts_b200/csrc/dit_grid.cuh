// dit_grid.cuh -- host interface of the grid-persistent DiT Euler loop for
// small batches with fp32 weights (dit_grid.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace ctts {

struct DitGridArgs {
  static constexpr int kMaxNL = 8, kMaxSteps = 16, kMaxRows = 12;
  int R = 0;                      // utterances (3 token rows each: patch 1)
  int NL = 0, steps = 0;
  int H = 0, nq = 0, nkv = 0, hd = 0, F = 0, L = 0;
  float eps = 1e-6f;
  float dts[kMaxSteps];
  float* x = nullptr;             // [R, L] in: x0, out: x after `steps` Euler steps
  const float* mu = nullptr;      // [R, H]
  const float* temb = nullptr;    // [steps, H]
  const float* dtemb = nullptr;   // [H]
  const float* condh = nullptr;   // [R, H]
  const float* ad = nullptr;      // [R, NL*6H] AdaLN or null
  const float* inv_freq = nullptr;  // [hd/2]
  const float* final_norm = nullptr;
  const float *in_w = nullptr, *in_b = nullptr;    // [H, L], [H]
  const float *out_w = nullptr, *out_b = nullptr;  // [L, H], [L]
  const float* wqkv[kMaxNL] = {};  // [(nq+2nkv)*hd, H]
  const float* wo[kMaxNL] = {};    // [H, nq*hd]
  const float* wgu[kMaxNL] = {};   // [2F, H], 64-row gate/up interleave
  const float* wd[kMaxNL] = {};    // [H, F]
  const float* norm1[kMaxNL] = {};
  const float* norm2[kMaxNL] = {};
  // Flag-tagged exchange words (dit_grid_ll_words(), zero at allocation):
  // (tag << 32) | float bits, tag = launch generation and phase.
  unsigned long long* ll = nullptr;
  unsigned* bar = nullptr;        // [0] launch generation, [1] exit count (dit_grid_counters())
  int* err = nullptr;
  // Error-path testing (ctts_debug_inject_wait_fault): polls of an exchange
  // word give up after spin_limit tries (0: the default), and with
  // skip_qkv_cta0 set CTA 0 leaves its QKV outputs unwritten, so the
  // attention phase waits on words no producer writes.
  uint32_t spin_limit = 0;
  int skip_qkv_cta0 = 0;
};

// Counters the launch needs (zero at allocation).
int dit_grid_counters(int NL, int steps);
// 64-bit exchange words the launch needs for up to R utterances.
size_t dit_grid_ll_words(int R, int H, int nq, int nkv, int hd, int F, int L);
// True when the shapes fit the kernel (patch 1, head_dim 64, sizes below
// the shared-memory budget) and a grid of one CTA per SM can be resident.
bool dit_grid_supported(int R, int NL, int steps, int H, int nq, int nkv, int hd, int F, int L);
cudaError_t launch_dit_grid(const DitGridArgs& a, cudaStream_t s);

}  // namespace ctts
