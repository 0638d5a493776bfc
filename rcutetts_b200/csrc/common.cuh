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

}  // namespace ctts
