// dit_cluster.cuh -- host interface of the cluster-resident DiT Euler loop
// (dit_cluster.cu).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ctts {

// Shapes the kernel is specialised for (the benchmark DiT head: hidden 512,
// 8 heads of 64, SwiGLU 1536, patch 1 -> 3 tokens per utterance, latent 64).
struct DitClusterShape {
  static constexpr int kC = 16;     // CTAs per thread-block cluster
  static constexpr int kH = 512;    // hidden
  static constexpr int kF = 1536;   // SwiGLU width
  static constexpr int kNH = 8;     // heads (MHA)
  static constexpr int kHD = 64;    // head dim
  static constexpr int kL = 64;     // latent
  static constexpr int kU = 10;     // utterances per cluster
  static constexpr int kMaxNL = 4;  // layers
  static constexpr int kMaxSteps = 16;
};

// Weights repacked so that CTA c of a cluster streams one contiguous slice
// per GEMM: QKV rows [c*96, c*96+96) of layer l are q, k, v of head c/2 for
// dims {16(c%2)..+15, 32+16(c%2)..+15}; gate/up rows [c*192, +192) are gate
// then up of SwiGLU columns [96c, 96c+96) (both pre-tiled in 64-column K
// blocks); o-proj and down are split over K: CTA c's blocks hold all 512
// output rows against its own input columns (o-proj: the 32 attention dims
// CTA c produces; down: SwiGLU columns [96c, 96c+96)), as 256-row x
// 32-column blocks [CTA][K atom][half].  All bf16, layers stacked.
struct DitClusterW {
  uint16_t *qkv = nullptr, *o = nullptr, *gu = nullptr, *dn = nullptr;
  float* norms = nullptr;  // [NL][2][H]: norm1, norm2
  CUtensorMap tm_qkv, tm_o, tm_gu, tm_dn;
  int NL = 0;
};

struct DitClusterArgs {
  int R = 0;          // utterances
  int NL = 0, steps = 0;
  int adaln = 0;
  float eps = 1e-6f;
  float dts[DitClusterShape::kMaxSteps];
  float* x = nullptr;             // [R, L] in: x0, out: x after `steps` Euler steps
  const float* mu = nullptr;      // [R, H]
  const float* temb = nullptr;    // [steps, H]
  const float* dtemb = nullptr;   // [H]
  const float* condh = nullptr;   // [R, H]
  const float* ad = nullptr;      // [R, NL*6H] AdaLN (shift1, scale1, gate1, shift2, scale2, gate2)
  const float* norms = nullptr;   // [NL][2][H]
  const float* fnorm = nullptr;   // [H]
  const uint16_t* out_w = nullptr;  // [L, H] bf16
  const float* out_b = nullptr;     // [L] or null
  const uint16_t* in_w = nullptr;   // [H, L] bf16
  const float* in_b = nullptr;      // [H] or null
  const float* inv_freq = nullptr;  // [HD/2]
  int* err = nullptr;
};

// Device error word value when an owner's sum of split-K partials (each
// exchanged as fp16) is not finite: a partial outside the fp16 range or a
// non-finite input.  The run's output is invalid; the caller reruns on the
// fp32-partial launch chain.
constexpr int kDitClusterErrRange = 5;

// Dynamic shared memory of one CTA for NL layers.
size_t dit_cluster_smem(int NL);
// Clusters of kC CTAs that fit on this GPU at once (0: the kernel cannot run).
int dit_cluster_max_active();
// Packs the layer weights (wqkv [1536,512] as stored, wgu [3072,512] in
// 64-row gate/up interleave, wo [512,512], wd [512,1536]) into W and builds
// its tensor maps.  Allocates W's buffers on the first call and repacks into
// the same buffers afterwards.  Synchronous.
cudaError_t dit_cluster_pack(DitClusterW& W, int NL, const void* const* wqkv, const void* const* wo,
                             const void* const* wgu, const void* const* wd, const float* const* norm1,
                             const float* const* norm2);
void dit_cluster_free(DitClusterW& W);
cudaError_t launch_dit_cluster(const DitClusterW& W, const DitClusterArgs& a, cudaStream_t s);

}  // namespace ctts
