// vae_tc.cu -- dense causal Conv1d and per-phase ConvTranspose1d of the VAE
// decoder on the tcgen05 tensor cores (bf16 operands, fp32 accumulate in
// TMEM): the bf16 path of launch_conv1d / launch_conv_transpose.
//
// Implicit GEMM (conv.rs:53-115 with snake.rs:26-36 applied to the input,
// decode.rs:39-80 for the transposed conv):
//   y[o, t*ostride + ph] = bias[o] (+ res) + sum_{j<k} sum_c W_j[o, c] * xs[c, t + xoff + j*dil - left]
//   xs = Snake(x) (x when no alpha), zero outside [0, Tin)
// A CTA owns 256 output channels (two M = 128 MMAs, accumulators in TMEM
// columns [0, 256) and [256, 512)) x 256 output positions (MMA N = 256) of
// one utterance and phase.  The reduction runs over 16-channel stages
// through a 3-slot shared-memory ring:
//  * weights (A): the load-time repack w_tc [phase][tap][Cin/8][Cout_pad][8]
//    makes every (tap, 8-channel chunk) a contiguous run of 16-byte rows, so
//    a stage is 2k bulk copies of up to 4 KB into the no-swizzle K-major
//    layout [tap][chunk][256 rows][16 B];
//  * activations (B): the window of 256 + (k-1)*dil input positions of the
//    stage's 16 channels, Snake applied and rounded to bf16 by four
//    producer warps while loading (two such groups take alternate stages),
//    stored [chunk][row][16 B]; tap j reads
//    rows [j*dil, j*dil + 256) of it -- a row offset of the descriptor's
//    start address -- so the window is loaded once for all k taps.
// Epilogue (warps 4..7, TMEM lane quadrant = warp & 3): bias, residual,
// tanh, the transposed conv's interleave (output index t*ostride + ph).
//
// Every wait is bounded; on timeout the CTA records error 5 in `err`, the
// other roles give up at their next wait, in-flight MMAs are drained before
// TMEM is released.
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"
#include "launch_state.h"
#include "tc_ptx.cuh"

namespace ctts {

namespace {

constexpr int kVT = 256;              // output positions per CTA (MMA N)
constexpr int kVO = 256;              // output channels per CTA (2 x M = 128)
constexpr int kVStages = 3;           // ring slots
constexpr int kVMaxHalo = 56;         // (k - 1) * dilation supported
constexpr int kVMaxK = 8;             // taps supported
constexpr int kVThreads = 320;        // warp 0 weights, warp 1 MMA, warps 2..9 activations
constexpr int kVProd = 256;           // activation producer threads
constexpr int kVProd0 = 64;           // first producer thread
constexpr int kVGroup = 128;          // producer threads per stage (two groups, alternate stages)
constexpr int kVItems = 5;            // 16-byte chunks per producer thread and stage (2 x 312 rows max)
constexpr int kVMaxCin = 1024;        // input channels (Snake table in shared memory)
constexpr size_t kVMinSmem = 120 * 1024;  // one CTA per SM: its 512 TMEM columns

static_assert(kVItems * kVGroup >= 2 * (kVT + kVMaxHalo + 7), "producer items cover the window");

struct VLay {
  uint32_t rows, a_bytes, b_bytes, stage;
  size_t total;
};
__host__ __device__ inline VLay vlay(int k, int halo) {
  VLay L;
  L.rows = (uint32_t)((kVT + halo + 7) & ~7);
  L.a_bytes = (uint32_t)k * 2u * (uint32_t)kVO * 16u;  // [tap][chunk][256 rows][16 B]
  L.b_bytes = 2u * L.rows * 16u;                       // [chunk][rows][16 B]
  L.stage = L.a_bytes + L.b_bytes;
  L.total = (size_t)kVStages * L.stage + 8 * (2 * kVStages + 2) + 16 + 8 * (size_t)kVMaxCin;
  return L;
}

// K-major operand without swizzle: 8-row x 16-byte core matrices stored as
// 128 contiguous bytes, K-adjacent core matrices `lbo` bytes apart,
// M/N-adjacent 8-row groups `sbo` bytes apart; version 1, layout type 0.
CTTS_DEV uint64_t desc_nosw(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1u << 46;
  return d;
}

CTTS_DEV void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

CTTS_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Bounded wait that gives up early once another role has aborted.
CTTS_DEV bool vwait(uint64_t* bar, uint32_t parity, volatile int* abort) {
  const uint32_t ad = smem_u32(bar);
  for (uint32_t it = 0; it < kWaitLimit; ++it) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(ad), "r"(parity)
        : "memory");
    if (done) return true;
    if ((it & 1023u) == 1023u && *abort) return false;
  }
  return false;
}

// Snake (snake.rs:26-36) with the per-channel 1/(alpha + 1e-9) precomputed;
// the sine is the hardware approximation: the result is rounded to bf16
// for the MMA, whose rounding error (2^-9 relative) dominates its error.
CTTS_DEV float snake_fast(float v, float al, float inv) {
  const float s = __sinf(v * al);
  return v + inv * (s * s);
}

// two floats -> packed bf16x2 (round to nearest even), lo in the low half
CTTS_DEV uint32_t pack_bf2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

__global__ void __launch_bounds__(kVThreads, 1) vae_tc_conv_kernel(const VaeTcArgs a) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  // aligned by an offset into the shared array (not through an integer
  // cast), so the compiler keeps every access through it in shared space
  uint8_t* smem = smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u);
  const int halo = (a.k - 1) * a.dil;
  const VLay L = vlay(a.k, halo);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)kVStages * L.stage);
  uint64_t* empty = full + kVStages;
  uint64_t* done = empty + kVStages;
  uint64_t* fin = done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(fin + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float2* snk = reinterpret_cast<float2*>(smem + (size_t)kVStages * L.stage + 8 * (2 * kVStages + 2) + 16);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t0 = blockIdx.x * kVT, o0 = blockIdx.y * kVO;
  const int b = blockIdx.z / a.nphase, ph = blockIdx.z % a.nphase;
  const int nm = min(2, (a.Cout_pad - o0) / 128);  // M tiles of this CTA (1 or 2)
  const int C8 = a.Cin / 8, nst = a.Cin / 16;
  const uint32_t sbase = smem_u32(smem);

  if (tid == 0) {
    for (int s = 0; s < kVStages; s++) {
      mbar_init(&full[s], 1 + kVGroup);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    mbar_init(fin, 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // per-channel Snake parameters: (alpha, 1 / (alpha + 1e-9))
  if (a.alpha)
    for (int c = tid; c < a.Cin; c += blockDim.x) {
      const float al = a.alpha[c];
      snk[c] = make_float2(al, 1.0f / (al + 1e-9f));
    }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  const uint16_t* wph = a.w + (size_t)ph * a.k * C8 * a.Cout_pad * 8;
  const uint32_t rows_bytes = (uint32_t)nm * 128u * 16u;
  // weights of stage s into its slot (arrive + expected bytes on full)
  auto issue_a = [&](int s) {
    const int slot = s % kVStages;
    const uint32_t dst = sbase + (uint32_t)slot * L.stage;
    mbar_expect_tx(&full[slot], (uint32_t)a.k * 2u * rows_bytes);
    for (int j = 0; j < a.k; j++)
      for (int kc = 0; kc < 2; kc++) {
        const uint16_t* src = wph + (((size_t)j * C8 + (size_t)(2 * s + kc)) * a.Cout_pad + o0) * 8;
        bulk_g2s(dst + (uint32_t)(j * 2 + kc) * (uint32_t)(kVO * 16), src, rows_bytes, &full[slot]);
      }
  };
  // the weights do not depend on the previous kernel: the first stages are
  // fetched before waiting on it (programmatic dependent launch)
  const int pre = min(nst, kVStages);
  if (tid == 0)
    for (int s = 0; s < pre; s++) issue_a(s);
  grid_dep_wait();
  grid_dep_launch();

  bool ok = true;
  if (tid == 0) {
    // ---- weight loader
    for (int s = pre; s < nst && ok; s++) {
      const int slot = s % kVStages;
      if (!vwait(&empty[slot], ((s / kVStages) - 1) & 1, abort)) {
        ok = false;
        break;
      }
      issue_a(s);
    }
  } else if (tid == 32) {
    // ---- MMA issuer: per stage, k taps x nm M tiles of M=128, N=256, K=16
    const uint32_t idesc = umma_idesc(kVT);
    const uint32_t blbo = L.rows * 16u;
    for (int s = 0; s < nst && ok; s++) {
      const int slot = s % kVStages;
      if (!vwait(&full[slot], (s / kVStages) & 1, abort)) {
        ok = false;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t sa = sbase + (uint32_t)slot * L.stage;
      const uint32_t sb = sa + L.a_bytes;
      for (int j = 0; j < a.k; j++) {
        const uint64_t bd = desc_nosw(sb + (uint32_t)(j * a.dil) * 16u, blbo, 128u);
        for (int m = 0; m < nm; m++) {
          const uint64_t ad = desc_nosw(sa + (uint32_t)(j * 2) * (uint32_t)(kVO * 16) + (uint32_t)(m * 128 * 16),
                                        (uint32_t)(kVO * 16), 128u);
          umma_bf16(tmem + (uint32_t)(m * kVT), ad, bd, idesc, (s > 0 || j > 0) ? 1u : 0u);
        }
      }
      umma_commit(&empty[slot]);
    }
    if (ok) umma_commit(done);
    // every MMA issued has completed before TMEM can be released
    umma_commit(fin);
    vwait(fin, 0, abort);
  } else if (tid >= kVProd0) {
    // ---- activation producers: Snake(x) window -> bf16 [chunk][row][16 B].
    // Two groups of 128 threads take alternate stages, so two windows are
    // in flight; each thread issues every load of its stage before any
    // Snake arithmetic (the staging is bound by global-load latency).
    const int p = tid - kVProd0;
    const int grp = p / kVGroup, q = p % kVGroup;
    const int rows = (int)L.rows, span = kVT + halo;
    const float* xb = a.x + (size_t)b * a.Cin * a.Tin;
    const int base_t = t0 + a.xoff - a.left;
    for (int s = grp; s < nst && ok; s += 2) {
      const int slot = s % kVStages;
      if (s >= kVStages && !vwait(&empty[slot], ((s / kVStages) - 1) & 1, abort)) {
        ok = false;
        break;
      }
      const uint32_t bst = sbase + (uint32_t)slot * L.stage + L.a_bytes;
      float v[kVItems][8];
#pragma unroll
      for (int it = 0; it < kVItems; it++) {
        const int item = q + it * kVGroup;
        const int kc = item / rows, r = item - kc * rows;
        const int src = base_t + r;
        const bool ld = item < 2 * rows && r < span && src >= 0 && src < a.Tin;
        const float* xc = xb + (size_t)(16 * s + 8 * kc) * a.Tin + src;
#pragma unroll
        for (int e = 0; e < 8; e++) v[it][e] = ld ? __ldg(xc + (size_t)e * a.Tin) : 0.0f;
      }
#pragma unroll
      for (int it = 0; it < kVItems; it++) {
        const int item = q + it * kVGroup;
        if (item >= 2 * rows) break;
        const int kc = item / rows, r = item - kc * rows;
        const int src = base_t + r;
        if (a.alpha && r < span && src >= 0 && src < a.Tin) {
          const float2* sk = snk + 16 * s + 8 * kc;
#pragma unroll
          for (int e = 0; e < 8; e++) {
            const float2 t = sk[e];
            v[it][e] = snake_fast(v[it][e], t.x, t.y);
          }
        }
        const uint32_t w0 = pack_bf2(v[it][0], v[it][1]);
        const uint32_t w1 = pack_bf2(v[it][2], v[it][3]);
        const uint32_t w2 = pack_bf2(v[it][4], v[it][5]);
        const uint32_t w3 = pack_bf2(v[it][6], v[it][7]);
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(bst + (uint32_t)(kc * rows + r) * 16u),
                     "r"(w0), "r"(w1), "r"(w2), "r"(w3)
                     : "memory");
      }
      // the writes above are read by the tensor cores (async proxy)
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive(&full[slot]);
    }
  }
  if (!ok) {
    if (!*abort) {
      *abort = 1;
      if (a.err) atomicExch(a.err, 5);
    }
  }

  // ---- epilogue: warps 4..7 (TMEM lanes 32q..32q+31, q = warp & 3)
  if (warp >= 4 && warp < 8) {
    const bool have = __all_sync(0xffffffffu, !*abort && vwait(done, 0, abort));
    if (!have && !*abort) {
      *abort = 1;
      if (a.err) atomicExch(a.err, 5);
    }
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const int q = warp & 3;
    const bool vec = a.ostride == 1 && (a.Tout & 3) == 0;
    for (int m = 0; m < nm && have; m++) {
      const int o = o0 + m * 128 + q * 32 + lane;
      const bool ov = o < a.Cout;
      const float bo = (ov && a.bias) ? __ldg(a.bias + o) : 0.0f;
      const size_t orow = ((size_t)b * a.Cout + (ov ? o : 0)) * a.Tout;
      for (int cc = 0; cc < kVT / 16; cc++) {
        uint32_t r[16];
        tmem_ld16_nowait(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(m * kVT + cc * 16), r);
        tmem_wait();
        const int tb = t0 + cc * 16;
        if (!ov || tb >= a.Tc) continue;
        float val[16];
#pragma unroll
        for (int i = 0; i < 16; i++) val[i] = __uint_as_float(r[i]) + bo;
        if (vec && tb + 16 <= a.Tc) {
          float* yp = a.y + orow + tb;
          if (a.res) {
            const float4* rp = reinterpret_cast<const float4*>(a.res + orow + tb);
#pragma unroll
            for (int i = 0; i < 4; i++) {
              const float4 rv = rp[i];
              val[4 * i] += rv.x;
              val[4 * i + 1] += rv.y;
              val[4 * i + 2] += rv.z;
              val[4 * i + 3] += rv.w;
            }
          }
          if (a.tanh_out) {
#pragma unroll
            for (int i = 0; i < 16; i++) val[i] = tanhf(val[i]);
          }
#pragma unroll
          for (int i = 0; i < 4; i++)
            reinterpret_cast<float4*>(yp)[i] = make_float4(val[4 * i], val[4 * i + 1], val[4 * i + 2], val[4 * i + 3]);
        } else {
#pragma unroll
          for (int i = 0; i < 16; i++) {
            const int t = tb + i;
            if (t >= a.Tc) break;
            const size_t oi = orow + (size_t)t * a.ostride + ph;
            float v = val[i];
            if (a.res) v += a.res[oi];
            if (a.tanh_out) v = tanhf(v);
            a.y[oi] = v;
          }
        }
      }
    }
  }

  __syncwarp();
  __syncthreads();
  if (*abort) {
    // let bulk copies already in flight land before the CTA leaves
    long long c0, c1;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(c0));
    do {
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(c1));
    } while (c1 - c0 < 200000);
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
}

// dst[ph][j][c8][o][e] = src[((ph * Cout + o) * Cin + 8 c8 + e) * k + j]
// (rows o >= Cout stay zero: the buffer is zeroed at allocation)
__global__ void repack_conv_tc_kernel(uint16_t* dst, const uint16_t* src, int nphase, int Cout, int Cin, int k,
                                      int cout_pad) {
  const size_t n = (size_t)nphase * Cout * Cin * k;
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int j = (int)(i % k);
  const size_t r = i / k;
  const int c = (int)(r % Cin);
  const size_t r2 = r / Cin;
  const int o = (int)(r2 % Cout);
  const int ph = (int)(r2 / Cout);
  const size_t d = ((((size_t)ph * k + j) * (Cin / 8) + c / 8) * cout_pad + o) * 8 + (c & 7);
  dst[d] = src[i];
}

}  // namespace

bool conv_tc_supported(const ConvArgs& a) {
  return a.w_bf16 && a.w_tc && a.groups == 1 && a.Cin % 16 == 0 && a.Cin >= 16 && a.Cin <= kVMaxCin &&
         a.Cout >= 64 && a.k >= 1 &&
         a.k <= kVMaxK && (a.k - 1) * a.dil <= kVMaxHalo && a.cout_pad >= a.Cout && a.cout_pad % 128 == 0;
}

cudaError_t launch_conv_tc(const ConvArgs& a, int Tc, int ostride, int nphase, cudaStream_t s) {
  if (!conv_tc_supported(a) || Tc <= 0 || (reinterpret_cast<uintptr_t>(a.w_tc) & 15)) return cudaErrorInvalidValue;
  const VLay L = vlay(a.k, (a.k - 1) * a.dil);
  const size_t smem = std::max(L.total + 128, kVMinSmem);
  static SmemOptIn opt;
  if (cudaError_t e = opt.ensure((const void*)vae_tc_conv_kernel, smem)) return e;
  VaeTcArgs t;
  t.x = a.x; t.w = static_cast<const uint16_t*>(a.w_tc); t.bias = a.bias; t.res = a.res; t.y = a.y;
  t.alpha = a.snake_alpha; t.err = a.err;
  t.B = a.B; t.Cin = a.Cin; t.Cout = a.Cout; t.Cout_pad = a.cout_pad; t.Tin = a.Tin; t.Tout = a.Tout; t.Tc = Tc;
  t.k = a.k; t.dil = a.dil; t.left = a.left; t.xoff = a.xoff; t.ostride = ostride; t.nphase = nphase;
  t.tanh_out = a.tanh_out;
  dim3 grid((unsigned)((Tc + kVT - 1) / kVT), (unsigned)((a.Cout + kVO - 1) / kVO), (unsigned)(a.B * nphase));
  CTTS_LK(launch_k(vae_tc_conv_kernel, grid, dim3(kVThreads), smem, s, t));
  return cudaGetLastError();
}

cudaError_t repack_conv_tc(uint16_t* dst, const uint16_t* src, int nphase, int Cout, int Cin, int k, int cout_pad,
                           cudaStream_t s) {
  if (Cin % 8 != 0 || cout_pad < Cout) return cudaErrorInvalidValue;
  const size_t n = (size_t)nphase * Cout * Cin * k;
  repack_conv_tc_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(dst, src, nphase, Cout, Cin, k, cout_pad);
  return cudaGetLastError();
}

}  // namespace ctts
