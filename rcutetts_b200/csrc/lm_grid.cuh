// lm_grid.cuh -- host interface of the grid-persistent LM decode step for
// small batches with fp32 weights (lm_grid.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace ctts {

struct LmGridArgs {
  static constexpr int kMaxNL = 24, kMaxRows = 4;
  int R = 0;  // utterances (one new token each); R == the cache's batch
  int NL = 0, H = 0, nq = 0, nkv = 0, hd = 0, F = 0, cap = 0;
  float eps = 1e-6f;
  float* h = nullptr;    // [R, H] residual stream: in the new rows, out the last layer's output
  float* qkv = nullptr;  // [R, (nq + 2 nkv) hd] workspace
  float* part = nullptr;  // [grid CTAs][hd + 2] attention partials (lm_grid_part_floats())
  float* act = nullptr;  // [R, F] workspace
  float* out = nullptr;  // [R, H] final RMSNorm of h
  const float* final_norm = nullptr;
  int* pos = nullptr;    // [R] cache lengths; every one advanced by one at the end
  const float* inv_freq = nullptr;  // [hd / 2] RoPE
  float* kcache = nullptr;  // fp32, layer l at + l * layer_elems: [R][nkv][cap][hd]
  float* vcache = nullptr;
  size_t layer_elems = 0;
  const float* wqkv[kMaxNL] = {};  // [(nq + 2 nkv) hd, H]
  const float* wo[kMaxNL] = {};    // [H, nq hd]
  const float* wgu[kMaxNL] = {};   // [2F, H], 64-row gate/up interleave
  const float* wd[kMaxNL] = {};    // [H, F]
  const float* norm1[kMaxNL] = {};
  const float* norm2[kMaxNL] = {};
  const float* qn[kMaxNL] = {};    // QK-Norm gains [hd] or null
  const float* kn[kMaxNL] = {};
  unsigned* bar = nullptr;  // barrier counters, zero at rest (lm_grid_counters())
  int* err = nullptr;       // 1: a position outside the cache; 4: a barrier or copy wait gave up
};

// Barrier counters one launch needs (all zero between launches).
int lm_grid_counters(int NL);
// Floats of the attention-partial workspace one launch needs.
size_t lm_grid_part_floats(int hd);
// True when the shapes fit the kernel's shared memory and a grid of one CTA
// per SM can be resident (cooperative launch).
bool lm_grid_supported(int R, int NL, int H, int nq, int nkv, int hd, int F);
cudaError_t launch_lm_grid(const LmGridArgs& a, cudaStream_t s);

}  // namespace ctts
