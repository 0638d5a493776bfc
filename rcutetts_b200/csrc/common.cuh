// common.cuh -- shared device helpers for the sm_100a decode-path kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#define CTTS_DEV __device__ __forceinline__

namespace ctts {

// bf16 weights are stored as raw uint16 bit patterns; widening is exact
// (the same shift the reference's bf16_to_f32 does, simd.rs:283-319).
CTTS_DEV float bf2f(uint16_t u) { return __uint_as_float(((uint32_t)u) << 16); }
CTTS_DEV float bf_lo(uint32_t u) { return __uint_as_float(u << 16); }
CTTS_DEV float bf_hi(uint32_t u) { return __uint_as_float(u & 0xFFFF0000u); }

// round-to-nearest-even f32 -> bf16 bits (NaN kept quiet)
CTTS_DEV uint16_t f2bf(float f) {
  uint32_t u = __float_as_uint(f);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x7FFFFFu)) return (uint16_t)((u >> 16) | 0x40);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

CTTS_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

CTTS_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

CTTS_DEV float silu(float g) { return g / (1.0f + expf(-g)); }

// Programmatic dependent launch: a kernel launched with the
// programmatic-stream-serialization attribute may start while its
// predecessor drains; it must call grid_dep_wait() before touching the
// predecessor's outputs.  Both are no-ops for a normal launch.
CTTS_DEV void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
CTTS_DEV void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" :::); }
// The usual entry of a kernel in the chain: inputs of the predecessor are
// complete after this, and the successor may begin its own prologue.
CTTS_DEV void grid_dep_enter() {
  grid_dep_wait();
  grid_dep_launch();
}

// 16-byte loads that bypass L1 allocation for streamed weights.
CTTS_DEV float4 ld_stream_f4(const float* p) {
  float4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
               : "l"(p));
  return r;
}
CTTS_DEV uint4 ld_stream_u4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// A warp loads one fp32 row of K elements (K % 128 == 0, K <= 128*MAXV)
// into registers with every float4 load issued before any use: lane holds
// v[i] = x[lane*4 + 128*i .. +3].  Returns the sum of squares (warp total).
template <int MAXV>
CTTS_DEV float warp_load_row(const float* x, int K, float4* v) {
  const int lane = threadIdx.x & 31;
  const int nv = K >> 7;
#pragma unroll
  for (int i = 0; i < MAXV; i++)
    if (i < nv) v[i] = *reinterpret_cast<const float4*>(x + lane * 4 + 128 * i);
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < MAXV; i++)
    if (i < nv) {
      ss = fmaf(v[i].x, v[i].x, ss);
      ss = fmaf(v[i].y, v[i].y, ss);
      ss = fmaf(v[i].z, v[i].z, ss);
      ss = fmaf(v[i].w, v[i].w, ss);
    }
  return warp_sum(ss);
}

#define CTTS_LK(x)                        \
  do {                                    \
    cudaError_t _e = (x);                 \
    if (_e != cudaSuccess) return _e;     \
  } while (0)

// Host: launch with the programmatic-stream-serialization attribute (PDL)
// unless it is switched off (CTTS_PDL=0).
bool pdl_enabled();

template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                            Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

}  // namespace ctts
