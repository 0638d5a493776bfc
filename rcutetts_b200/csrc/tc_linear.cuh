// tc_linear.cuh -- host interface of the tcgen05 bf16 linear (tc_linear.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

namespace ctts {

// Epilogue and per-launch state (filled by launch_tc_linear from TcCall).
struct TcArgs {
  int M = 0, N = 0;         // activation rows, weight rows (2x outputs for swiglu)
  int m0 = 0, MT = 0;       // first row / rows per MMA tile (MMA N)
  int kblocks = 0, splitk = 1, stages = 1, tmem_cols = 32;
  const float* bias = nullptr;  // [N]
  int act = 0;                  // 0 none, 2 swiglu (W rows tile-interleaved: 64 gate, 64 up)
  float* y = nullptr;           // fp32 output [M, y_ld] ...
  uint16_t* yb = nullptr;       // ... or bf16 output
  long y_ld = 0;
  const float* res = nullptr;   // fp32 residual [M, y_ld]
  const float* gate = nullptr;  // AdaLN gate: coef = 1 + gate[(m/gate_div)*gate_ld + gate_off + col]
  long gate_ld = 0;
  int gate_div = 1, gate_off = 0;
  float scale = 1.0f;           // coef when gate is null
  // RMSNorm folded into the GEMM: the B operand holds bf16(x * gain) and the
  // accumulator of row m is scaled by 1/sqrt(sum_t rs_ssp[t*rs_ld + m] / rs_k
  // + rs_eps), the row's sum of squares given as rs_nt partials.
  const float* rs_ssp = nullptr;
  long rs_ld = 0;
  int rs_nt = 0;
  float rs_k = 1.0f, rs_eps = 0.0f;
  // Producer side of that fold (fp32 output, no SwiGLU): also write
  // yb2 = bf16(out * g2[col]) with leading dimension y_ld, and this tile's
  // partial sum of squares of each output row to ssp[tile*ssp_ld + m].
  uint16_t* yb2 = nullptr;
  const float* g2 = nullptr;
  float* ssp = nullptr;
  long ssp_ld = 0;
  float* part = nullptr;        // split-K partial tiles
  int* counters = nullptr;      // per-tile tickets (zero at rest)
  int* err = nullptr;           // device error flag
};

struct TcPlan {
  int MT = 0, mtiles = 0, ntiles = 0, kblocks = 0, splitk = 1, stages = 1, tmem_cols = 32;
  size_t smem = 0;
};

// One call: Y = epi(X[M,K] . W[N,K]^T); X, W bf16 row-major (K % 64 == 0,
// 16-byte aligned rows).
struct TcCall {
  const uint16_t* x = nullptr;
  const uint16_t* w = nullptr;
  int M = 0, N = 0, K = 0;
  TcArgs epi;  // bias / act / y / yb / y_ld / res / gate* / scale
  float* part = nullptr;
  size_t part_floats = 0;
  int* counters = nullptr;
  int counter_count = 0;
  int* err = nullptr;
  int pdl = 0;
  int max_splitk = 64;
};

TcPlan tc_plan(int M, int N, int K, int num_sms, int max_splitk = 64);
int tc_num_sms();
size_t tc_scratch_floats(const TcPlan& p);
cudaError_t launch_tc_linear(const TcCall& c, cudaStream_t s);

}  // namespace ctts
