// dit_cluster.cu -- the whole DiT Euler loop of one frame (every step, every
// layer, the output/feedback tail) as ONE kernel launch on thread-block
// clusters of 16 CTAs.
//
// Replaces the per-step launch chain of dit.rs:775-814 predict_cached /
// euler_sample (in_proj + seq fill, per layer RMSNorm+AdaLN -> QKV ->
// 3-token RoPE attention -> o-proj + gated residual -> RMSNorm+AdaLN ->
// SwiGLU -> down + gated residual, final norm -> out_proj -> x += dt*v).
//
// Layout.  A cluster owns kU = 10 utterances (30 token rows: row 3u+s is
// token s of utterance u) for the whole frame.  CTA c of the cluster owns
// hidden columns [32c, 32c+32) of the residual stream (fp32, in shared
// memory for all steps).  Every GEMM is a tcgen05.mma chain with the
// activations as A (rows 0..29 valid; the descriptor's 8-row groups beyond
// the fourth read the following shared memory and land in accumulator
// lanes that are never read), a weight slice as B streamed by TMA through
// a 4-slot ring that runs ahead of the activations across layers and steps
// (the weights do not depend on them), the accumulator in TMEM:
//  * QKV and gate/up are split over N: CTA c computes 96 QKV columns (half
//    of head c/2) and 192 gate/up columns (SwiGLU columns [96c, 96c+96))
//    from the all-gathered normed operand (K = 512);
//  * o-proj and down are split over K: CTA c multiplies its own 32
//    attention dims / 96 SwiGLU columns by all 512 output rows (N = 2 x 256
//    MMAs), and the partials (accumulated in fp32, exchanged as fp16: an
//    11-bit significand, 4x finer than the bf16 operands of these GEMMs)
//    are reduce-scattered: each owner sums the 16 partials of its 32
//    columns in fp32, in CTA order (deterministic).
//
// Exchange.  A operands are stored K-major with the 64-byte swizzle as one
// contiguous slice per CTA ([32-column atom][row group][8 rows x 64 B]), so
// the all-gathers end with the compute warps writing their own slice in
// place and pushing it to the 15 peers with one bulk copy each
// (cp.async.bulk shared::cta -> shared::cluster), completing on the peer's
// mbarrier; the per-step out_proj partials and the new latent go the same
// way from small staging buffers.  The other per-layer exchanges leave
// straight from the compute threads' registers as remote stores that
// complete on the receiver's mbarrier (st.async ... mbarrier::complete_tx),
// a warp's 32 stores filling one contiguous span: each thread its row's
// fp16 split-K partials into the 16 owners' partial blocks (the
// reduce-scatter), warp 0 its row statistics and attention score partials.
// Every mbarrier is armed with its phase's byte count
// (arrive.expect_tx) by its waiter right after the previous phase
// completed, which by the stage order is before any peer can push for that
// phase; consecutive stages never share an mbarrier.  Stages that feed a
// GEMM (A barriers, two arrivals: the arm and this CTA's own slice) are
// waited by the MMA thread, the others (B barriers, reduce-scatter) by the
// compute warps.  RMSNorm row sums are reduced from the 16 per-CTA partials
// in CTA order (deterministic), attention scores from the two half-head
// partials in order, out_proj over the 16 column slices in order.  AdaLN
// slices of the next layer are prefetched by bulk copies from global
// memory into a second buffer.
//
// Roles (512 threads): warps 0, 4, 8, 12 = compute (lane = token row; TMEM
// lanes 0..31, columns split over the four), warp 1 = MMA issuer (lane 0)
// and TMEM owner, warp 2 = TMA producer (lane 0).  Every wait is bounded;
// on timeout the CTA records an error code, tells its peers to stop, waits
// (bounded) for its own copies and MMAs in flight, and leaves through a
// final cluster barrier.
#include <algorithm>
#include <cstdio>
#include <mutex>
#include <vector>

#include <cuda_fp16.h>

#include "dit_cluster.cuh"
#include "launch_state.h"
#include "tc_ptx.cuh"

namespace ctts {

namespace {

using Sh = DitClusterShape;
constexpr int kC = Sh::kC, kH = Sh::kH, kF = Sh::kF, kHD = Sh::kHD, kL = Sh::kL, kU = Sh::kU;
constexpr int kNT = 512;               // threads per CTA: 16 warps, compute warps 0, 4, 8, 12
constexpr int kRows = 3 * kU;          // 30 token rows per cluster
constexpr int kGrp = (kRows + 7) / 8;  // 4 groups of 8 rows (32 row slots)
constexpr int kOwn = kH / kC;          // 32 hidden columns per CTA
constexpr int kActOwn = kF / kC;       // 96 SwiGLU columns per CTA
constexpr int kQkvN = 3 * kHD / 2;     // 96: q, k, v of half a head
constexpr int kGuN = 2 * kActOwn;      // 192: gate + up
// A operands: K-major, no swizzle, one contiguous slice per CTA: slice =
// [row group g][8-column core kc][8 rows x 16 bytes], so a CTA's share of an
// operand is one block it can push to its peers with a single bulk copy.
constexpr uint32_t kSlice = kGrp * (kOwn / 8) * 128;      // 2 KB: 32 columns
constexpr uint32_t kActSlice = kGrp * (kActOwn / 8) * 128;  // 6 KB: 96 columns
constexpr uint32_t kXA = 0;                              // norm outputs, K = 512 (all-gathered)
constexpr uint32_t kATT = kXA + kC * kSlice;             // own attention slice (o-proj A, K = 32)
constexpr uint32_t kSWI = kATT + kSlice;                 // own SwiGLU slice (down A, K = 96)
constexpr uint32_t kPART = kSWI + kActSlice;             // split-K partials from every CTA (o-proj / down)
constexpr uint32_t kPartBytes = 32 * kOwn * 2;           // 2 KB: [4 column chunks][32 rows][8 halves]
constexpr uint32_t kRING = kPART + kC * kPartBytes;      // weight ring
constexpr uint32_t kSlotBytes = kGuN * 128;              // 24 KB: one 192-row, 64-wide K block
constexpr int kSlots = 4;
constexpr uint32_t kF32 = kRING + kSlots * kSlotBytes;
constexpr int kTmemCols = 512;                           // split-K accumulators span all 512 outputs
// split-K weight blocks (o-proj, down): 256 output rows x 32 K columns,
// 64-byte swizzle, 16 KB per ring slot
constexpr uint32_t kHalfBlk = 256 * 64;
static_assert(kRING % 1024 == 0 && kATT % 512 == 0 && kSWI % 512 == 0 && kPART % 16 == 0,
              "operand alignment");
constexpr int kSeqLd = kOwn + 1;
constexpr int kAdLd = 6 * kOwn + 4;  // 196: 16-byte rows, 2-way banks at most
// fp32 area, float offsets from kF32 (exchange buffers 16-byte aligned)
constexpr int oSEQ = 0;                          // [32][33] residual stream, own columns
constexpr int oSSR = 1056;                       // [16][32] row sum-of-squares partials, by source CTA
constexpr int oSCR = oSSR + kC * 32;             // [2][3][32] attention score partials, by half, key token, row
constexpr int oVR = oSCR + 2 * 32 * 3;           // [16][10][4] out_proj partials of my 4 latent columns, by source
constexpr int oVRO = oVR + kC * kU * 4;          // [16][10][4] my partials, by owner
constexpr int oXS = oVRO + kC * kU * 4;          // [16][10][4] latent x, by owner: x[u][4c+i]
constexpr int oXO = oXS + kC * kU * 4;           // [10][4] my updated latent columns
constexpr int oXN = oXO + kU * 4;                // [10][32] final-normed x rows, own columns
constexpr int oMU = oXN + kU * kOwn;             // [10][32] mu
constexpr int oCH = oMU + kU * kOwn;             // [10][32] cond_proj rows
constexpr int oDT = oCH + kU * kOwn;             // [32] delta-time embedding
constexpr int oINB = oDT + kOwn;                 // [32] in_proj bias
constexpr int oFN = oINB + kOwn;                 // [32] final norm
constexpr int oOUTB = oFN + kOwn;                // [4] out_proj bias of my latent columns (+4 pad)
constexpr int oRCS = oOUTB + 8;                  // [3 positions][cos 16, sin 16] RoPE of my dims
constexpr int oTEMB = oRCS + 96;                 // [steps][32] time embeddings
constexpr int oNRM = oTEMB + Sh::kMaxSteps * kOwn;  // [NL][2][32] norm1, norm2
__host__ __device__ constexpr int oAD(int NL) { return oNRM + NL * 2 * kOwn; }  // [2][10][196] AdaLN, by layer parity
__host__ __device__ constexpr int oPSC(int NL) { return oAD(NL) + 2 * kU * kAdLd; }  // [4][32][3] score partials
__host__ __device__ constexpr int oPSS(int NL) { return oPSC(NL) + 4 * 32 * 3; }     // [4][32] row ss partials
__host__ __device__ constexpr int f32_floats(int NL) { return oPSS(NL) + 4 * 32; }
static_assert(oSSR >= 32 * kSeqLd && oSSR % 4 == 0 && oSCR % 4 == 0 && oVR % 4 == 0 && oXS % 4 == 0 &&
                  oXO % 4 == 0 && oVRO % 4 == 0 && oNRM % 4 == 0,
              "exchange buffers must be 16-byte aligned");

// byte offsets of the bf16 tail tables and the barriers
struct Lay {
  uint32_t outw, inw, bar;
  size_t total;
};
__host__ __device__ inline Lay lay(int NL) {
  Lay L;
  const uint32_t f32_end = kF32 + (uint32_t)f32_floats(NL) * 4u;
  L.outw = (f32_end + 15u) & ~15u;          // [32 own cols][64 latent] out_proj slice (transposed)
  L.inw = L.outw + kOwn * kL * 2;           // [64 latent][32 own cols] in_proj slice (transposed)
  L.bar = (L.inw + kOwn * kL * 2 + 15u) & ~15u;
  L.total = (size_t)L.bar + 16 * 8 + 16;    // 16 mbarriers, TMEM slot, abort flag
  return L;
}

// mbarrier indices
constexpr int bFULL = 0, bEMPTY = kSlots, bMMA = 2 * kSlots, bFIN = bMMA + 1, bA = bFIN + 1, bB = bA + 2,
              bAD = bB + 2, bRS = bAD + 1;
static_assert(bRS < 16, "16 mbarrier slots");

// Optional stage timeline (build with -DCTTS_DIT_TRACE): CTA 0 records
// (event, %globaltimer) pairs of its compute warp (row 0) and MMA thread.
#ifdef CTTS_DIT_TRACE
__device__ long long g_dit_trace[2][8192];
__device__ int g_dit_trace_n[2];
CTTS_DEV void dtrace(int role, int ev, int& n) {
  if (blockIdx.x != 0) return;
  long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  if (n < 4095) {
    g_dit_trace[role][2 * n] = ev;
    g_dit_trace[role][2 * n + 1] = t;
    n++;
    g_dit_trace_n[role] = n;
  }
}
#define DTRACE(role, ev) \
  if (lane == 0) dtrace(role, ev, tr_n)
#else
#define DTRACE(role, ev)
#endif

// per-GEMM geometry.  QKV (0) and gate/up (2): the CTA's weight slice is
// the MMA N (96 / 192 rows), 64-wide K blocks pre-tiled as
// [layer][CTA][K block][N rows][64] (128-byte swizzle), kbps K blocks per
// ring slot.  o-proj (1) and down (3) are split over K: the CTA multiplies
// its own 32 attention dims / 96 SwiGLU columns by all 512 output rows, in
// blocks of 256 rows x 32 K columns (64-byte swizzle) pre-tiled as
// [layer][CTA][K atom][half][256][32]; nblk ring slots per GEMM.
struct Gemm {
  int nblk, kbps;
  uint32_t bytes;  // per ring slot
};
CTTS_DEV Gemm gemm(int g) {
  switch (g) {
    case 0: return {kH / 64 / 2, 2, 2u * kQkvN * 128u};
    case 1: return {2, 1, kHalfBlk};
    case 2: return {kH / 64, 1, kGuN * 128u};
    default: return {6, 1, kHalfBlk};
  }
}
// bytes a CTA receives from its 15 peers for the A stage of GEMM g (the
// split-K GEMMs read only this CTA's own slice)
CTTS_DEV uint32_t a_bytes(int g) { return (g == 0 || g == 2) ? (uint32_t)(kC - 1) * kSlice : 0u; }

// Bytes of B stage b (all senders, self included).  Order: the first fill,
// then per Euler step [scores, row stats, row stats] per layer, out_proj
// partials, new x, next fill.
constexpr uint32_t kSsBytes = kC * 128, kScBytes = 2 * 384, kVrBytes = kC * kU * 16;
CTTS_DEV uint32_t b_bytes(int b, int NL) {
  if (b == 0) return kSsBytes;
  const int per = 3 * NL + 3, rem = (b - 1) % per;
  if (rem < 3 * NL) return rem % 3 == 0 ? kScBytes : kSsBytes;
  return rem == 3 * NL + 2 ? kSsBytes : kVrBytes;
}

// Bounded waits that give up early once this CTA is aborting.
CTTS_DEV bool wait_cluster(uint32_t bar, uint32_t parity, const volatile uint32_t* abort) {
  for (uint32_t it = 0; it < kWaitLimit; ++it) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    if (done) return true;
    if ((it & 255u) == 255u && *abort) return false;
  }
  return false;
}
CTTS_DEV bool wait_local(uint32_t bar, uint32_t parity, const volatile uint32_t* abort) {
  for (uint32_t it = 0; it < kWaitLimit; ++it) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    if (done) return true;
    if ((it & 255u) == 255u && *abort) return false;
  }
  return false;
}

// arrive (one of the phase's arrivals) and raise its expected bytes
CTTS_DEV void arm(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
CTTS_DEV void arrive_local(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
// bulk copy of `bytes` from this CTA's shared memory into CTA `rank`'s, at
// the same offsets, completing on that CTA's mbarrier at `bar`
CTTS_DEV void push(uint32_t dst, uint32_t src, uint32_t bytes, uint32_t bar, uint32_t rank) {
  asm volatile(
      "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          mapa_shared(dst, rank)),
      "r"(src), "r"(bytes), "r"(mapa_shared(bar, rank))
      : "memory");
}
// remote stores from registers into CTA `rank`'s shared memory at the same
// offset, completing (their bytes) on that CTA's mbarrier at `bar`: they
// leave straight from the thread, not through the CTA's bulk-copy queue
CTTS_DEV void sta_v4(uint32_t dst, uint32_t x, uint32_t y, uint32_t z, uint32_t w, uint32_t bar, uint32_t rank) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
                   mapa_shared(dst, rank)),
               "r"(x), "r"(y), "r"(z), "r"(w), "r"(mapa_shared(bar, rank))
               : "memory");
}
CTTS_DEV void sta_f32(uint32_t dst, float v, uint32_t bar, uint32_t rank) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(
                   mapa_shared(dst, rank)),
               "r"(__float_as_uint(v)), "r"(mapa_shared(bar, rank))
               : "memory");
}
CTTS_DEV void st_rc_u32(uint32_t a, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(a), "r"(v) : "memory");
}
CTTS_DEV uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
CTTS_DEV void st_u4(uint8_t* p, uint32_t x, uint32_t y, uint32_t z, uint32_t w) {
  *reinterpret_cast<uint4*>(p) = make_uint4(x, y, z, w);
}

// Byte offset of the 16-byte chunk holding columns [8kc, 8kc+8) of row r
// inside a slice: [32-column atom][8-row group][8 rows x 64 B, 64-byte
// swizzle (chunk ^= (row >> 1) & 3)], so a 32-column slice is 2 KB and the
// 16 row groups one M=128 MMA reads are 8 KB of contiguous shared memory.
CTTS_DEV uint32_t slice_off(int r, int kc) {
  const int rr = r & 7;
  return (uint32_t)(kc >> 2) * (kGrp * 512u) + (uint32_t)(r >> 3) * 512u + (uint32_t)rr * 64u +
         ((uint32_t)((kc & 3) ^ ((rr >> 1) & 3)) << 4);
}

// UMMA descriptor of a K-major operand with 64-byte swizzle: SBO = 512
// bytes between 8-row groups, LBO unused (1), version 1, layout type 4.
CTTS_DEV uint64_t desc_sw64(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1u << 16;
  d |= (uint64_t)(512u >> 4) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)4u << 61;
  return d;
}

CTTS_DEV uint32_t pack_bf(float a, float b) { return (uint32_t)f2bf(a) | ((uint32_t)f2bf(b) << 16); }

// SiLU through the identity g * sigmoid(g) = (g/2) * (1 + tanh(g/2)): one
// hardware tanh (tanh.approx, absolute error near 2^-11) instead of an
// exponential and a reciprocal.  The SwiGLU stage of 3072 elements per CTA
// is bound by the special-function unit of the compute warps' single SM
// sub-partition; the error stays below the bf16 rounding of the operand.
CTTS_DEV float silu_tanh(float g) {
  const float h = 0.5f * g;
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(h));
  return fmaf(h, t, h);
}

__global__ void __launch_bounds__(kNT, 1)
    dit_cluster_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmO,
                       const __grid_constant__ CUtensorMap tmG, const __grid_constant__ CUtensorMap tmD,
                       const DitClusterArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // aligned by an offset into the shared array (not through an integer
  // cast), so the compiler keeps every access through it in shared space
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int NL = a.NL, steps = a.steps;
  const Lay LY = lay(NL);
  const uint32_t sb = smem_u32(smem);
  float* F = reinterpret_cast<float*>(smem + kF32);
  const uint32_t fb = sb + kF32;  // byte address of F
  uint16_t* outw_t = reinterpret_cast<uint16_t*>(smem + LY.outw);
  uint16_t* inw_t = reinterpret_cast<uint16_t*>(smem + LY.inw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + LY.bar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + LY.bar + 128);
  volatile uint32_t* abort = reinterpret_cast<volatile uint32_t*>(smem + LY.bar + 132);
  auto bar = [&](int i) { return sb + LY.bar + 8u * (uint32_t)i; };

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = (int)cluster_rank();
  const int U0 = (int)(blockIdx.x / kC) * kU;
#ifdef CTTS_DIT_TRACE
  int tr_n = 0;
#endif
  const int nvalid = max(0, min(kU, a.R - U0));

  if (tid == 0) {
    for (int i = 0; i < kSlots; i++) {
      mbar_init(&bars[bFULL + i], 1);
      mbar_init(&bars[bEMPTY + i], 1);
    }
    mbar_init(&bars[bMMA], 1);
    mbar_init(&bars[bFIN], 1);
    mbar_init(&bars[bAD], 1);
    // A stages: the MMA thread's arm + this CTA's own slice; B stages: the
    // compute warp's arm (every sender, itself included, pushes bytes)
    for (int i = 0; i < 2; i++) {
      mbar_init(&bars[bA + i], 2);
      mbar_init(&bars[bB + i], 1);
    }
    mbar_init(&bars[bRS], 1);
    *abort = 0u;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    arm(bar(bA + 0), a_bytes(0));
    arm(bar(bA + 1), a_bytes(1));
    arm(bar(bB + 0), b_bytes(0, NL));
    arm(bar(bB + 1), b_bytes(1, NL));
    arm(bar(bRS), kC * kPartBytes);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  // the weights do not depend on earlier kernels: the producer fills the
  // ring before the programmatic-launch wait
  const CUtensorMap* maps[4] = {&tmQ, &tmO, &tmG, &tmD};
  uint32_t pit = 0;  // producer: ring slots filled so far
  int pst = 0, pl = 0, pg = 0, pkb = 0;  // producer position
  bool pdone = false;
  auto produce_one = [&]() {
    const Gemm G = gemm(pg);
    const int slot = (int)(pit % kSlots);
    const uint32_t dst = sb + kRING + (uint32_t)slot * kSlotBytes;
    mbar_expect_tx(&bars[bFULL + slot], G.bytes);
    // first row of this slot's box in the tiled matrix
    int y;
    if (pg == 0) y = ((pl * kC + c) * (kH / 64) + pkb * G.kbps) * kQkvN;
    else if (pg == 2) y = ((pl * kC + c) * (kH / 64) + pkb) * kGuN;
    else y = ((pl * kC + c) * G.nblk + pkb) * 256;
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            dst),
        "l"(reinterpret_cast<uint64_t>(maps[pg])), "r"(0), "r"(y), "r"(bar(bFULL + slot))
        : "memory");
    pit++;
    if (++pkb >= G.nblk) {
      pkb = 0;
      if (++pg == 4) {
        pg = 0;
        if (++pl == NL) {
          pl = 0;
          if (++pst == steps) pdone = true;
        }
      }
    }
  };
  if (warp == 2 && lane == 0)
    while (!pdone && pit < (uint32_t)kSlots) produce_one();
  grid_dep_wait();

  // ---- per-CTA constants (every thread)
  const int adld = NL * 6 * kH;
  for (int i = tid; i < kC * kU * 4; i += kNT) {  // xs[q][u][i] = x[u][4q + i]
    const int q = i / (kU * 4), u = (i / 4) % kU, k = 4 * q + (i & 3);
    F[oXS + i] = (u < nvalid) ? a.x[(size_t)(U0 + u) * kL + k] : 0.0f;
  }
  for (int i = tid; i < kU * kOwn; i += kNT) {
    const int u = i / kOwn, j = i % kOwn;
    const bool ok = u < nvalid;
    F[oMU + i] = ok ? a.mu[(size_t)(U0 + u) * kH + c * kOwn + j] : 0.0f;
    F[oCH + i] = ok ? a.condh[(size_t)(U0 + u) * kH + c * kOwn + j] : 0.0f;
  }
  for (int i = tid; i < 32 * kSeqLd; i += kNT) F[oSEQ + i] = 0.0f;
  for (int j = tid; j < kOwn; j += kNT) {
    F[oDT + j] = a.dtemb[c * kOwn + j];
    F[oINB + j] = a.in_b ? a.in_b[c * kOwn + j] : 0.0f;
    F[oFN + j] = a.fnorm[c * kOwn + j];
  }
  if (tid < 4) F[oOUTB + tid] = a.out_b ? a.out_b[4 * c + tid] : 0.0f;
  if (tid < 48) {  // the three token positions' rotations, computed once
    const int sp = tid / 16, j = tid % 16;
    float sn, cs;
    sincosf((float)sp * a.inv_freq[16 * (c & 1) + j], &sn, &cs);
    F[oRCS + sp * 32 + j] = cs;
    F[oRCS + sp * 32 + 16 + j] = sn;
  }
  for (int i = tid; i < steps * kOwn; i += kNT) F[oTEMB + i] = a.temb[(size_t)(i / kOwn) * kH + c * kOwn + i % kOwn];
  for (int i = tid; i < NL * 2 * kOwn; i += kNT)
    F[oNRM + i] = a.norms[(size_t)(i / kOwn) * kH + c * kOwn + i % kOwn];
  // AdaLN slices of layer 0 in buffer 0; invalid utterances stay zero in both
  for (int i = tid; i < 2 * kU * kAdLd; i += kNT) {
    const int buf = i / (kU * kAdLd), u = (i / kAdLd) % kU, e = i % kAdLd;
    float v = 0.0f;
    if (buf == 0 && a.adaln && u < nvalid && e < 6 * kOwn)
      v = a.ad[(size_t)(U0 + u) * adld + (size_t)(e / kOwn) * kH + c * kOwn + e % kOwn];
    F[oAD(NL) + i] = v;
  }
  for (int i = tid; i < kOwn * kL; i += kNT) {
    const int j = i / kL, o = i % kL;  // outw_t[j][o] = out_w[o][32c + j]
    outw_t[i] = a.out_w[(size_t)o * kH + c * kOwn + j];
    const int ii = i / kOwn, jj = i % kOwn;  // inw_t[i][j] = in_w[32c + j][i]
    inw_t[i] = a.in_w[(size_t)(c * kOwn + jj) * kL + ii];
  }
  // the async proxy (bulk copies into the AdaLN buffers) sees the zeros
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  __syncthreads();
  grid_dep_launch();
  // every CTA's barriers exist and are armed before any peer pushes
  cluster_sync();

  const float eps = a.eps;
  bool ok = true;
  auto fail = [&](int code) {
    if (!*abort) {
      *abort = 1u;
      if (a.err) atomicExch(a.err, code);
      for (int d = 0; d < kC; d++) st_rc_u32(mapa_shared(sb + LY.bar + 132, (uint32_t)d), 1u);
    }
  };

  if (warp == 2) {
    // ================= TMA producer (weights)
    if (lane == 0) {
      while (!pdone) {
        const int slot = (int)(pit % kSlots);
        if (!wait_local(bar(bEMPTY + slot), ((pit / kSlots) - 1) & 1, abort)) {
          fail(3);
          break;
        }
        produce_one();
      }
      // drain: the last fills of every slot have landed
      const uint32_t n0 = pit > (uint32_t)kSlots ? pit - kSlots : 0;
      for (uint32_t i = n0; i < pit; i++) wait_local(bar(bFULL + (int)(i % kSlots)), (i / kSlots) & 1, abort);
    }
  } else if (warp == 1) {
    // ================= MMA issuer
    if (lane == 0) {
      uint32_t it = 0, aph = 0;
      for (int st = 0; st < steps && ok; st++)
        for (int l = 0; l < NL && ok; l++)
          for (int g = 0; g < 4 && ok; g++) {
            const Gemm G = gemm(g);
            const uint32_t ab = bar(bA + (int)(aph & 1));
            if (!wait_cluster(ab, (aph >> 1) & 1, abort)) {
              ok = false;
              break;
            }
            arm(ab, a_bytes((g + 2) & 3));  // this barrier's next stage
            aph++;
            DTRACE(1, 5);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            if (g == 1 || g == 3) {
              // split-K: this CTA's own slice (one / three 32-column atoms)
              // times 256-row weight blocks, accumulators D[:, 256 h + n]
              const uint32_t idesc = umma_idesc(256);
              const uint32_t abase = sb + (g == 1 ? kATT : kSWI);
              for (int blk = 0; blk < G.nblk && ok; blk++) {
                const int slot = (int)(it % kSlots);
                if (!wait_local(bar(bFULL + slot), (it / kSlots) & 1, abort)) {
                  ok = false;
                  break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                DTRACE(1, 8);
                const int atom = blk >> 1, half = blk & 1;
                const uint64_t ad = desc_sw64(abase + (uint32_t)atom * 2048u);
                const uint64_t bd = desc_sw64(sb + kRING + (uint32_t)slot * kSlotBytes);
                const uint32_t dcol = tmem + 256u * (uint32_t)half;
                umma_bf16(dcol, ad, bd, idesc, atom ? 1u : 0u);
                umma_bf16(dcol, ad + 2, bd + 2, idesc, 1u);
                umma_commit(&bars[bEMPTY + slot]);
                it++;
              }
              if (ok) umma_commit(&bars[bMMA]);
              DTRACE(1, 6);
              continue;
            }
            const int GN = g == 0 ? kQkvN : kGuN;
            const int nkb = kH / 64;
            const uint32_t idesc = umma_idesc(GN);
            const uint32_t abase = sb + kXA;
            // Both operands advance by constant descriptor steps (address >> 4
            // in the low bits): the A operand's 32-column atoms are 2 KB apart
            // in column order for every GEMM (one atom per 32-column slice,
            // three per 96-column slice), so K step ks sits at atom ks / 2,
            // +32 bytes for odd ks; a weight K block is G.N rows of 128 bytes.
            uint64_t ad = desc_sw64(abase);
            const uint64_t bstep = (uint64_t)(GN * 8);
            for (int kb0 = 0; kb0 < nkb && ok; kb0 += G.kbps) {
              const int slot = (int)(it % kSlots);
              if (!wait_local(bar(bFULL + slot), (it / kSlots) & 1, abort)) {
                ok = false;
                break;
              }
              asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
              DTRACE(1, 8);
              const int n = G.kbps;
              uint64_t bd = umma_desc(sb + kRING + (uint32_t)slot * kSlotBytes);
              for (int q = 0; q < n; q++) {
                umma_bf16(tmem, ad, bd, idesc, (kb0 | q) ? 1u : 0u);
                umma_bf16(tmem, ad + 2, bd + 2, idesc, 1u);
                umma_bf16(tmem, ad + 128, bd + 4, idesc, 1u);
                umma_bf16(tmem, ad + 130, bd + 6, idesc, 1u);
                ad += 256;
                bd += bstep;
              }
              umma_commit(&bars[bEMPTY + slot]);
              it++;
            }
            if (ok) umma_commit(&bars[bMMA]);
            DTRACE(1, 6);
          }
      if (!ok) fail(3);
      // every MMA this thread issued has completed before TMEM is freed
      umma_commit(&bars[bFIN]);
      wait_local(bar(bFIN), 0, abort);
    }
  } else if ((warp & 3) == 0) {
    // ================= compute warps 0, 4, 8, 12 (cw = 0..3): lane = token
    // row (TMEM lanes 0..31, which warps 0 mod 4 may read).  Every stage
    // splits its columns over the four warps; warp 0 alone waits on the
    // exchange/MMA barriers, combines the per-warp row partials in warp
    // order (deterministic), pushes to the peers and runs the per-step
    // tail.  All four warps pass the same named barriers in the same order,
    // with `ok` made uniform at each of them.
    const int cw = warp >> 2;
    const int r = lane, u = r / 3, s = r % 3;
    const bool rv = r < kRows;
    float* seq = F + oSEQ;
    float* ssr = F + oSSR;
    float* scr = F + oSCR;
    float* vr = F + oVR;
    float* xs = F + oXS;
    float* xn = F + oXN;
    float* nrm = F + oNRM;
    float* psc = F + oPSC(NL);  // [4 warps][32 rows][3] score partials
    float* pss = F + oPSS(NL);  // [4 warps][32 rows] sum-of-squares partials
    volatile uint32_t* cok = reinterpret_cast<volatile uint32_t*>(smem + LY.bar + 136);
    uint32_t bph = 0, aph = 0, gph = 0, nsync = 0;
    auto cbar = [&]() { asm volatile("bar.sync 1, 128;" ::: "memory"); };
    // warp 0's `ok` to all compute warps (two slots: a slow reader of one
    // sync never sees the next sync's value)
    auto sync_ok = [&]() {
      if (cw == 0 && lane == 0) cok[nsync & 1] = ok ? 1u : 0u;
      cbar();
      ok = cok[nsync & 1] != 0u;
      nsync++;
    };
    // B stage (warp 0) from a staging buffer: its writes visible to the
    // bulk copies, lane d pushes to CTA d; then wait and re-arm for two
    // stages later
    auto pushB = [&](uint32_t src_off, uint32_t dst_off, uint32_t bytes) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      DTRACE(0, 7);
      const uint32_t bb = bar(bB + (int)(bph & 1));
      if (lane < kC) push(sb + dst_off, sb + src_off, bytes, bb, (uint32_t)lane);
    };
    auto waitB = [&]() {
      const uint32_t bb = bar(bB + (int)(bph & 1));
      if (ok && !wait_cluster(bb, (bph >> 1) & 1, abort)) ok = false;
      if (lane == 0) arm(bb, b_bytes((int)bph + 2, NL));
      bph++;
      __syncwarp();
      DTRACE(0, 3);
    };
    // A stage (all compute warps): this CTA's slice, written in place by the
    // four warps, to the 15 peers (warp 0 pushes; a contiguous 2 KB block
    // per peer as one bulk copy -- the slice's 64-byte row stride would
    // scatter per-thread remote stores)
    auto postA = [&](uint32_t slice_addr, uint32_t bytes) {
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      cbar();
      if (cw == 0) {
        DTRACE(0, 7);
        const uint32_t ab = bar(bA + (int)(aph & 1));
        if (lane == 0) arrive_local(ab);
        if (bytes && lane < kC && lane != c) push(slice_addr, slice_addr, bytes, ab, (uint32_t)lane);
        __syncwarp();
        DTRACE(0, 1);
      }
      aph++;
    };
    // accumulator complete (warp 0 waits, all warps then read TMEM)
    auto wait_mma = [&]() {
      if (cw == 0 && ok && !wait_local(bar(bMMA), gph & 1, abort)) ok = false;
      gph++;
      sync_ok();
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      if (cw == 0) DTRACE(0, 4);
    };
    // warp 0: this CTA's partial of row r's sum of squares -> ssr[c][r] of
    // every CTA (itself included), by remote stores
    auto push_row_stat = [&](float v) {
      DTRACE(0, 7);
      const uint32_t bb = bar(bB + (int)(bph & 1));
      const uint32_t dst = fb + (uint32_t)(oSSR + c * 32 + r) * 4u;
#pragma unroll 4
      for (int i = 0; i < kC; i++) sta_f32(dst, v, bb, (uint32_t)((c + i) & (kC - 1)));
    };
    // the per-warp row partials pss[cw][r] summed in warp order -> every
    // CTA's ssr[c] (warp 0), then all warps see the 16 CTAs' sums
    auto ss_combine_push = [&]() {
      if (cw == 0) DTRACE(0, 13);
      cbar();
      if (cw == 0) {
        DTRACE(0, 14);
        push_row_stat(((pss[r] + pss[32 + r]) + pss[64 + r]) + pss[96 + r]);
        waitB();
      }
      sync_ok();
    };
    auto row_inv = [&](int row) {
      float ss = 0.0f;
#pragma unroll
      for (int q = 0; q < kC; q++) ss += ssr[q * 32 + row];
      return 1.0f / sqrtf(ss / (float)kH + eps);
    };
    // RMSNorm (+ AdaLN modulate) of own columns [8cw, 8cw+8) -> chunk cw of
    // my slice of the K=512 operand
    auto norm_slice = [&](const float* adb, int l, int which) {
      const float inv = row_inv(r);
      const float* nw = nrm + (l * 2 + which) * kOwn;
      const float* md = adb + min(u, kU - 1) * kAdLd + which * 3 * kOwn;  // shift, scale
      uint32_t pk[4];
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        const int j = 8 * cw + e;
        float e0 = seq[r * kSeqLd + j] * inv * nw[j], e1 = seq[r * kSeqLd + j + 1] * inv * nw[j + 1];
        if (a.adaln) {
          e0 = e0 * (1.0f + md[kOwn + j]) + md[j];
          e1 = e1 * (1.0f + md[kOwn + j + 1]) + md[j + 1];
        }
        pk[e >> 1] = pack_bf(e0, e1);
      }
      st_u4(smem + kXA + c * kSlice + slice_off(r, cw), pk[0], pk[1], pk[2], pk[3]);
      postA(sb + kXA + c * kSlice, kSlice);
    };
    // Split-K reduce-scatter.  The accumulator holds this CTA's partial of
    // all 512 outputs for its 32 rows; warp cw sends columns
    // [128cw, 128cw + 128) -- owner CTAs 4cw..4cw+3 -- as fp16 (11-bit
    // significand, 4x finer than the bf16 operands of these GEMMs), each
    // lane its row, by remote stores into the owner's partial block of this
    // CTA ([4 column chunks][32 rows][8 halves]) that complete on the
    // owner's bRS.  Warp 0 waits for all 16 blocks of the phase.
    uint32_t rsph = 0;
    auto rs_exchange = [&]() {
      // 16-column halves through two register buffers: the TMEM load of
      // half i + 1 is in flight while half i is converted and sent
      const uint32_t dst = sb + kPART + (uint32_t)c * kPartBytes + (uint32_t)r * 16u;
      const uint32_t rb = bar(bRS);
      auto stage_half = [&](const uint32_t* v, int i) {
        const uint32_t d = (uint32_t)(4 * cw + (i >> 1));
#pragma unroll
        for (int q = 0; q < 2; q++) {
          uint32_t h[4];
#pragma unroll
          for (int e = 0; e < 4; e++) {
            const __half2 p2 = __floats2half2_rn(__uint_as_float(v[8 * q + 2 * e]), __uint_as_float(v[8 * q + 2 * e + 1]));
            h[e] = *reinterpret_cast<const uint32_t*>(&p2);
          }
          sta_v4(dst + (uint32_t)(2 * (i & 1) + q) * 512u, h[0], h[1], h[2], h[3], rb, d);
        }
      };
      auto half_addr = [&](int i) { return tmem + 32u * (uint32_t)(4 * cw + (i >> 1)) + 16u * (uint32_t)(i & 1); };
      uint32_t va[16], vb[16];
      tmem_ld16_nowait(half_addr(0), va);
#pragma unroll
      for (int i = 0; i < 8; i += 2) {
        tmem_wait16(va);
        tmem_ld16_nowait(half_addr(i + 1), vb);
        stage_half(va, i);
        tmem_wait16(vb);
        if (i + 2 < 8) tmem_ld16_nowait(half_addr(i + 2), va);
        stage_half(vb, i + 1);
      }
      if (cw == 0) {
        DTRACE(0, 9);
        if (ok && !wait_cluster(rb, rsph & 1, abort)) ok = false;
        if (lane == 0) arm(rb, kC * kPartBytes);  // the next exchange's bytes
        __syncwarp();
        DTRACE(0, 11);
      }
      rsph++;
      sync_ok();
      if (cw == 0) DTRACE(0, 12);
    };
    // gated residual update of own columns [8cw, 8cw+8) from the 16 split-K
    // partials (summed in CTA order: deterministic), and their sum of
    // squares -> pss[cw]
    auto resid_rs = [&](const float* adb, int gate_k) {
      float p = 0.0f;
      if (rv) {
        // own columns [8cw, 8cw+8) are chunk cw of every source's block
        const uint8_t* part = smem + kPART + (uint32_t)cw * 512u + (uint32_t)r * 16u;
        float acc[8];
#pragma unroll
        for (int e = 0; e < 8; e++) acc[e] = 0.0f;
#pragma unroll 4
        for (int q2 = 0; q2 < kC; q2++) {
          const uint4 w4 = *reinterpret_cast<const uint4*>(part + q2 * kPartBytes);
          const uint32_t w[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
          for (int e = 0; e < 4; e++) {
            // fp32 += fp16 in one instruction (the fp16 value converts
            // exactly; one rounding, as with a convert and an add)
            asm("{\n\t.reg .f16 lo, hi;\n\t"
                "mov.b32 {lo, hi}, %2;\n\t"
                "add.rn.f32.f16 %0, lo, %0;\n\t"
                "add.rn.f32.f16 %1, hi, %1;\n\t}"
                : "+f"(acc[2 * e]), "+f"(acc[2 * e + 1])
                : "r"(w[e]));
          }
        }
        if (cw == 0) DTRACE(0, 15);
        // a partial outside the fp16 range (or a non-finite input) leaves a
        // non-finite sum: flagged for the host, which reruns in fp32
        bool fin = true;
#pragma unroll
        for (int e = 0; e < 8; e++) fin = fin && fabsf(acc[e]) <= 3.40282347e38f;
        if (!fin && a.err) atomicCAS(a.err, 0, kDitClusterErrRange);
        const float* gt = adb + u * kAdLd + gate_k * kOwn;
#pragma unroll
        for (int e = 0; e < 8; e++) {
          const int j = 8 * cw + e;
          const float coef = a.adaln ? 1.0f + gt[j] : 1.0f;
          const float nv = seq[r * kSeqLd + j] + coef * acc[e];
          seq[r * kSeqLd + j] = nv;
          p = fmaf(nv, nv, p);
        }
        if (cw == 0) DTRACE(0, 16);
      } else {
#pragma unroll
        for (int e = 0; e < 8; e++) p = fmaf(seq[r * kSeqLd + 8 * cw + e], seq[r * kSeqLd + 8 * cw + e], p);
      }
      pss[cw * 32 + r] = p;
    };
    // seq rows of step stn: [mu + temb + dtemb; cond; in_proj(x)] (warp 0,
    // lane = column), then the rows' sums of squares to every CTA
    auto fill = [&](int stn) {
      // all compute warps: lane = own column, warp cw the utterances cw,
      // cw + 4, cw + 8; in_proj's dot products of a warp's utterances advance
      // together (independent chains), each in latent order
      const int j = lane;
      float acc[3] = {0.0f, 0.0f, 0.0f};
#pragma unroll 4
      for (int i4 = 0; i4 < kL / 4; i4++) {
        float w4[4];
#pragma unroll
        for (int e = 0; e < 4; e++) w4[e] = bf2f(inw_t[(4 * i4 + e) * kOwn + j]);
#pragma unroll
        for (int k = 0; k < 3; k++) {
          const int uu = cw + 4 * k;
          if (uu < kU) {
            const float4 xv = *reinterpret_cast<const float4*>(&xs[(i4 * kU + uu) * 4]);
            acc[k] = fmaf(w4[0], xv.x, acc[k]);
            acc[k] = fmaf(w4[1], xv.y, acc[k]);
            acc[k] = fmaf(w4[2], xv.z, acc[k]);
            acc[k] = fmaf(w4[3], xv.w, acc[k]);
          }
        }
      }
#pragma unroll
      for (int k = 0; k < 3; k++) {
        const int uu = cw + 4 * k;
        if (uu < kU) {
          seq[(3 * uu) * kSeqLd + j] = (F[oMU + uu * kOwn + j] + F[oTEMB + stn * kOwn + j]) + F[oDT + j];
          seq[(3 * uu + 1) * kSeqLd + j] = F[oCH + uu * kOwn + j];
          seq[(3 * uu + 2) * kSeqLd + j] = acc[k] + F[oINB + j];
        }
      }
      cbar();
      // warp 0: the rows' sums of squares to every CTA
      if (cw == 0) {
        float p = 0.0f;
#pragma unroll 8
        for (int jj = 0; jj < kOwn; jj++) p = fmaf(seq[r * kSeqLd + jj], seq[r * kSeqLd + jj], p);
        push_row_stat(p);
        waitB();
      }
    };

    fill(0);
    sync_ok();
    for (int st = 0; st < steps && ok; st++) {
      for (int l = 0; l < NL && ok; l++) {
        const int LG = st * NL + l;  // layer count so far
        const float* adb = F + oAD(NL) + (LG & 1) * kU * kAdLd;
        if (a.adaln && LG > 0) {
          // this layer's slices (prefetched one layer ago)
          if (cw == 0 && ok && !wait_local(bar(bAD), (LG - 1) & 1, abort)) ok = false;
          sync_ok();
          if (!ok) break;
        }
        // S1: norm1 -> my operand slice -> peers
        norm_slice(adb, l, 0);
        if (a.adaln && cw == 0) {
          // the next layer's AdaLN slices into the other buffer, one 128-byte
          // copy per (utterance, part)
          if (LG + 1 < steps * NL) {
            const int ln = (LG + 1) % NL;
            const uint32_t dst = fb + (uint32_t)(oAD(NL) + ((LG + 1) & 1) * kU * kAdLd) * 4u;
            if (lane == 0) arm(bar(bAD), (uint32_t)(nvalid * 6 * 128));
            __syncwarp();
            if (lane < nvalid)
              for (int k = 0; k < 6; k++)
                asm volatile(
                    "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], 128, [%2];" ::"r"(
                        dst + (uint32_t)(lane * kAdLd + k * kOwn) * 4u),
                    "l"((uint64_t)__cvta_generic_to_global(a.ad + (size_t)(U0 + lane) * adld + (size_t)ln * 6 * kH +
                                                          k * kH + c * kOwn)),
                    "r"(bar(bAD))
                    : "memory");
          }
        }
        // S2: QKV accumulator -> RoPE -> half-head score partials -> partner.
        // Warp cw rotates dims {4cw..4cw+3} with their pairs {+16} and holds
        // v dims [8cw, 8cw+8) for the P.V of S3.
        wait_mma();
        if (!ok) break;
        float q[8], k[8], v[8];
        {
          uint32_t t0[4], t1[4], t2[4], t3[4], t4[8];
          tmem_ld4_nowait(tmem + 4 * cw, t0);
          tmem_ld4_nowait(tmem + 16 + 4 * cw, t1);
          tmem_ld4_nowait(tmem + 32 + 4 * cw, t2);
          tmem_ld4_nowait(tmem + 48 + 4 * cw, t3);
          tmem_ld8_nowait(tmem + 64 + 8 * cw, t4);
          tmem_wait();
#pragma unroll
          for (int i = 0; i < 4; i++) {
            q[i] = __uint_as_float(t0[i]);
            q[i + 4] = __uint_as_float(t1[i]);
            k[i] = __uint_as_float(t2[i]);
            k[i + 4] = __uint_as_float(t3[i]);
          }
#pragma unroll
          for (int i = 0; i < 8; i++) v[i] = __uint_as_float(t4[i]);
        }
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const int j = 4 * cw + i;
          const float cs = F[oRCS + s * 32 + j], sn = F[oRCS + s * 32 + 16 + j];
          float a1 = q[i], a2 = q[i + 4];
          q[i] = a1 * cs - a2 * sn;
          q[i + 4] = a1 * sn + a2 * cs;
          a1 = k[i];
          a2 = k[i + 4];
          k[i] = a1 * cs - a2 * sn;
          k[i + 4] = a1 * sn + a2 * cs;
        }
#pragma unroll
        for (int jt = 0; jt < 3; jt++) {
          const int src = min(3 * u + jt, 31);
          float d = 0.0f;
#pragma unroll
          for (int i = 0; i < 8; i++) d = fmaf(q[i], __shfl_sync(0xffffffffu, k[i], src), d);
          psc[(cw * 32 + r) * 3 + jt] = d;
        }
        cbar();
        if (cw == 0) {
          // my half-head score partials -> scr[c & 1] of this CTA and its
          // partner (the other half of the head)
          DTRACE(0, 7);
          const uint32_t bb = bar(bB + (int)(bph & 1));
          const uint32_t dst = fb + (uint32_t)(oSCR + (c & 1) * 96 + r) * 4u;
#pragma unroll
          for (int jt = 0; jt < 3; jt++) {
            const float v = ((psc[r * 3 + jt] + psc[(32 + r) * 3 + jt]) + psc[(64 + r) * 3 + jt]) +
                            psc[(96 + r) * 3 + jt];
            sta_f32(dst + 128u * (uint32_t)jt, v, bb, (uint32_t)c);
            sta_f32(dst + 128u * (uint32_t)jt, v, bb, (uint32_t)(c ^ 1));
          }
          waitB();
        }
        sync_ok();
        if (!ok) break;
        // S3: softmax over the utterance's 3 tokens, P.V on dims [8cw, 8cw+8)
        // -> chunk cw of my attention slice
        {
          float sc[3], m = -INFINITY;
          const float scale = 1.0f / sqrtf((float)kHD);
#pragma unroll
          for (int jt = 0; jt < 3; jt++) {
            sc[jt] = (scr[jt * 32 + r] + scr[96 + jt * 32 + r]) * scale;
            m = fmaxf(m, sc[jt]);
          }
          float lsum = 0.0f;
#pragma unroll
          for (int jt = 0; jt < 3; jt++) {
            sc[jt] = expf(sc[jt] - m);
            lsum += sc[jt];
          }
          const float inv = 1.0f / lsum;
          float o[8];
#pragma unroll
          for (int i = 0; i < 8; i++) o[i] = 0.0f;
#pragma unroll
          for (int jt = 0; jt < 3; jt++) {
            const int src = min(3 * u + jt, 31);
            const float p = sc[jt] * inv;
#pragma unroll
            for (int i = 0; i < 8; i++) o[i] = fmaf(p, __shfl_sync(0xffffffffu, v[i], src), o[i]);
          }
          // the o-proj is split over K: this slice (the CTA's 32 attention
          // dims) is the whole A operand of its partial product
          st_u4(smem + kATT + slice_off(r, cw), pack_bf(o[0], o[1]), pack_bf(o[2], o[3]), pack_bf(o[4], o[5]),
                pack_bf(o[6], o[7]));
          postA(sb + kATT, 0);
        }
        // S4: o-proj partials -> owners; the 16 partials of my columns ->
        // gated residual -> row statistics
        wait_mma();
        if (!ok) break;
        rs_exchange();
        if (!ok) break;
        resid_rs(adb, 2);
        ss_combine_push();
        if (!ok) break;
        // S5: norm2 -> operand
        norm_slice(adb, l, 1);
        // S6: gate/up accumulator -> SwiGLU of columns [24cw, 24cw+24) ->
        // chunks 3cw..3cw+2 of my slice of the K=1536 operand
        wait_mma();
        if (!ok) break;
        {
          uint8_t* sl = smem + kSWI;
          // chunk t = 8 gate + 8 up columns in one 16-register buffer; the
          // TMEM loads of chunk t + 1 are in flight while chunk t is computed
          auto load_chunk = [&](int t, uint32_t* c) {
            tmem_ld8_nowait(tmem + 24 * cw + 8 * t, c);
            tmem_ld8_nowait(tmem + kActOwn + 24 * cw + 8 * t, c + 8);
          };
          auto swiglu_chunk = [&](const uint32_t* c, int t) {
            uint32_t pk[4];
#pragma unroll
            for (int e = 0; e < 8; e += 2) {
              const float g0 = __uint_as_float(c[e]), g1 = __uint_as_float(c[e + 1]);
              pk[e >> 1] = pack_bf(silu_tanh(g0) * __uint_as_float(c[8 + e]), silu_tanh(g1) * __uint_as_float(c[8 + e + 1]));
            }
            st_u4(sl + slice_off(r, 3 * cw + t), pk[0], pk[1], pk[2], pk[3]);
          };
          uint32_t ca[16], cb[16];
          load_chunk(0, ca);
          tmem_wait16(ca);
          load_chunk(1, cb);
          swiglu_chunk(ca, 0);
          tmem_wait16(cb);
          load_chunk(2, ca);
          swiglu_chunk(cb, 1);
          tmem_wait16(ca);
          swiglu_chunk(ca, 2);
          postA(sb + kSWI, 0);
        }
        // S7: down partials -> owners -> gated residual -> row statistics
        wait_mma();
        if (!ok) break;
        rs_exchange();
        if (!ok) break;
        resid_rs(adb, 5);
        ss_combine_push();
      }
      if (!ok) break;
      // T1: final norm of the x rows (row 3u + 2 of utterance u; lane = own
      // column, warp cw the utterances cw, cw + 4, cw + 8), then the out_proj
      // partial over the own columns (warp cw latent outputs [16cw, 16cw+16),
      // half-warp h utterances [5h, 5h+5), each sum in column order), 4
      // latent columns to each owner CTA
#pragma unroll
      for (int k = 0; k < 3; k++) {
        const int uu = cw + 4 * k;
        if (uu < kU) {
          const float inv = row_inv(3 * uu + 2);
          xn[uu * kOwn + lane] = seq[(3 * uu + 2) * kSeqLd + lane] * inv * F[oFN + lane];
        }
      }
      cbar();
      {
        const int o = 16 * cw + (lane & 15), u5 = 5 * (lane >> 4);
        float ac[5];
#pragma unroll
        for (int k = 0; k < 5; k++) ac[k] = 0.0f;
#pragma unroll 4
        for (int j = 0; j < kOwn; j++) {
          const float w = bf2f(outw_t[j * kL + o]);
#pragma unroll
          for (int k = 0; k < 5; k++) ac[k] = fmaf(w, xn[(u5 + k) * kOwn + j], ac[k]);
        }
        // owner of latent column o is CTA o/4; vro[owner][uu][o%4]
#pragma unroll
        for (int k = 0; k < 5; k++) F[oVRO + ((o >> 2) * kU + u5 + k) * 4 + (o & 3)] = ac[k];
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      cbar();
      if (cw == 0) {
        {
          const uint32_t bb = bar(bB + (int)(bph & 1));
          if (lane < kC)
            push(sb + kF32 + (oVR + c * kU * 4) * 4, sb + kF32 + (oVRO + lane * kU * 4) * 4, kU * 16, bb,
                 (uint32_t)lane);
        }
        waitB();
        if (ok) {
          // T2: my 4 latent columns: reduce the 16 partials in order, Euler update
          for (int e = lane; e < kU * 4; e += 32) {
            const int uu = e >> 2, i = e & 3;
            float acc = 0.0f;
#pragma unroll
            for (int q2 = 0; q2 < kC; q2++) acc += vr[(q2 * kU + uu) * 4 + i];
            const float xnew = xs[(c * kU + uu) * 4 + i] + a.dts[st] * (acc + F[oOUTB + i]);
            if (st + 1 == steps) {
              if (uu < nvalid) a.x[(size_t)(U0 + uu) * kL + 4 * c + i] = xnew;
            } else {
              F[oXO + e] = xnew;
            }
          }
          if (st + 1 < steps) {
            pushB(kF32 + oXO * 4, kF32 + (oXS + c * kU * 4) * 4, kU * 16);
            waitB();
          }
        }
      }
      sync_ok();
      if (ok && st + 1 < steps) {
        // T3: the next step's sequence
        fill(st + 1);
        sync_ok();
      }
    }
    if (cw == 0 && !ok) fail(3);
  }

  __syncwarp();
  __syncthreads();
  if (*abort) {
    // let bulk copies already in flight land before any CTA leaves
    long long t0, t1;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    do {
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t1));
    } while (t1 - t0 < 200000);
  }
  // no CTA leaves while a peer may still write into its shared memory
  cluster_sync();
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
}

// Pre-tiling: src [blocks*N rows, K] (row-major slices of N rows) ->
// dst [blocks][K/64][N][64], one 128-byte row per 8 threads.
__global__ void tile_kernel(uint16_t* dst, const uint16_t* src, int N, int K) {
  const size_t t = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int nkb = K / 64;
  const size_t row = t >> 3;  // dst row
  const int part = (int)(t & 7);
  const size_t blk = row / ((size_t)nkb * N);
  const int kb = (int)((row / N) % nkb), n = (int)(row % N);
  const uint4* s = reinterpret_cast<const uint4*>(src + (blk * N + n) * K + kb * 64) + part;
  reinterpret_cast<uint4*>(dst + row * 64)[part] = *s;
}

// Split-K weight blocks: dst[blk][r][k] (256 rows x 32 columns per block,
// blocks ordered [CTA c][atom a][half h]) = W[256 h + r][col(c, 32 a + k)]
// for W [512 rows, K] row-major; col() = the CTA's K columns: the o-proj's
// attention dims of CTA c (perm[32 c + k]) or the down projection's SwiGLU
// columns 96 c + k (perm null, 3 atoms per CTA).
__global__ void splitk_blocks_kernel(uint16_t* dst, const uint16_t* W, int K, int atoms, const int* perm) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const size_t n = (size_t)kC * atoms * 2 * 256 * 32;
  if (i >= n) return;
  const int k = (int)(i % 32), r = (int)((i / 32) % 256);
  const size_t blk = i / (32 * 256);
  const int h = (int)(blk % 2), a_ = (int)((blk / 2) % atoms), cc = (int)(blk / (2 * atoms));
  const int kk = cc * atoms * 32 + a_ * 32 + k;
  const int col = perm ? perm[kk] : kk;
  dst[i] = W[(size_t)(256 * h + r) * K + col];
}

// dst row i (K bf16 elements) = src row idx[i]
__global__ void gather_rows_kernel(uint16_t* dst, const uint16_t* src, const int* idx, int K) {
  const int i = blockIdx.x;
  const uint4* s = reinterpret_cast<const uint4*>(src + (size_t)idx[i] * K);
  uint4* d = reinterpret_cast<uint4*>(dst + (size_t)i * K);
  for (int t = threadIdx.x; t < K / 8; t += blockDim.x) d[t] = s[t];
}

// 2D bf16 tensor [rows, 32] (64-byte rows), box [256 rows, 32], 64-byte
// swizzle: the split-K weight blocks.
bool make_map_sw64(CUtensorMap* m, const void* base, int rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {32, (cuuint64_t)rows};
  cuuint64_t strides[1] = {64};
  cuuint32_t box[2] = {32, 256};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

cudaError_t set_attrs(size_t smem) {
  static SmemOptIn opt;
  return opt.ensure((const void*)dit_cluster_kernel, smem, /*nonportable_cluster=*/true);
}

cudaLaunchConfig_t make_cfg(int nclusters, size_t smem, cudaStream_t s, cudaLaunchAttribute* attr, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kC * nclusters, 1, 1);
  cfg.blockDim = dim3(kNT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kC;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  return cfg;
}

}  // namespace

size_t dit_cluster_smem(int NL) { return lay(NL).total + 1024; }

int dit_cluster_max_active() {
  const size_t smem = dit_cluster_smem(Sh::kMaxNL);
  if (smem > 227 * 1024) return 0;
  if (set_attrs(smem) != cudaSuccess) return 0;
  cudaLaunchAttribute attr[2];
  cudaLaunchConfig_t cfg = make_cfg(1, smem, nullptr, attr, false);
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, dit_cluster_kernel, &cfg) != cudaSuccess) {
    (void)cudaGetLastError();
    return 0;
  }
  return n;
}

cudaError_t dit_cluster_pack(DitClusterW& W, int NL, const void* const* wqkv, const void* const* wo,
                             const void* const* wgu, const void* const* wd, const float* const* norm1,
                             const float* const* norm2) {
  if (NL <= 0 || NL > Sh::kMaxNL) return cudaErrorInvalidValue;
  W.NL = NL;
  const size_t nq = (size_t)NL * kC * kQkvN * kH, no = (size_t)NL * kH * kH;
  const size_t ng = (size_t)NL * kC * kGuN * kH, nd = (size_t)NL * kH * kF;
  cudaError_t e;
  // a repack (new weights uploaded) reuses the buffers: the addresses, and
  // the tensor maps built from them, stay what earlier launches captured
  if (!W.qkv) {
    if ((e = cudaMalloc(&W.qkv, nq * 2)) != cudaSuccess) return e;
    if ((e = cudaMalloc(&W.o, no * 2)) != cudaSuccess) return e;
    if ((e = cudaMalloc(&W.gu, ng * 2)) != cudaSuccess) return e;
    if ((e = cudaMalloc(&W.dn, nd * 2)) != cudaSuccess) return e;
    if ((e = cudaMalloc(&W.norms, sizeof(float) * NL * 2 * kH)) != cudaSuccess) return e;
  }
  // row maps
  std::vector<int> iq(kC * kQkvN), ig(kC * kGuN), iid(kH);
  for (int c = 0; c < kC; c++) {
    const int h = c >> 1, hf = c & 1;
    for (int i = 0; i < kQkvN; i++) {
      const int part = i / 32, j = i % 32;
      const int dim = j < 16 ? 16 * hf + j : 32 + 16 * hf + (j - 16);
      iq[c * kQkvN + i] = part * kH + h * kHD + dim;
    }
    for (int i = 0; i < kGuN; i++) {
      const int n = kActOwn * c + (i % kActOwn);
      ig[c * kGuN + i] = (n >> 6) * 128 + (i >= kActOwn ? 64 : 0) + (n & 63);
    }
  }
  for (int i = 0; i < kH; i++) iid[i] = i;
  std::vector<int> pcol(kH);  // o-proj column 32c + j <- attention dim of CTA c
  for (int c = 0; c < kC; c++)
    for (int j = 0; j < kOwn; j++) {
      const int h = c >> 1, hf = c & 1;
      pcol[c * kOwn + j] = h * kHD + (j < 16 ? 16 * hf + j : 32 + 16 * hf + (j - 16));
    }
  int* didx = nullptr;
  const size_t nidx = iq.size() + ig.size() + iid.size() + pcol.size();
  if ((e = cudaMalloc(&didx, nidx * sizeof(int))) != cudaSuccess) return e;
  std::vector<int> all;
  all.insert(all.end(), iq.begin(), iq.end());
  all.insert(all.end(), ig.begin(), ig.end());
  all.insert(all.end(), iid.begin(), iid.end());
  all.insert(all.end(), pcol.begin(), pcol.end());
  e = cudaMemcpy(didx, all.data(), nidx * sizeof(int), cudaMemcpyHostToDevice);
  const int* dq = didx;
  const int* dg = didx + iq.size();
  const int* di = dg + ig.size();
  const int* dp = di + iid.size();
  for (int l = 0; l < NL && e == cudaSuccess; l++) {
    gather_rows_kernel<<<kC * kQkvN, 64>>>(W.qkv + (size_t)l * kC * kQkvN * kH,
                                           static_cast<const uint16_t*>(wqkv[l]), dq, kH);
    const unsigned nob = (unsigned)(((size_t)kC * 1 * 2 * 256 * 32 + 255) / 256);
    splitk_blocks_kernel<<<nob, 256>>>(W.o + (size_t)l * kH * kH, static_cast<const uint16_t*>(wo[l]), kH, 1, dp);
    gather_rows_kernel<<<kC * kGuN, 64>>>(W.gu + (size_t)l * kC * kGuN * kH,
                                          static_cast<const uint16_t*>(wgu[l]), dg, kH);
    const unsigned ndb = (unsigned)(((size_t)kC * 3 * 2 * 256 * 32 + 255) / 256);
    splitk_blocks_kernel<<<ndb, 256>>>(W.dn + (size_t)l * kH * kF, static_cast<const uint16_t*>(wd[l]), kF, 3,
                                       nullptr);
    e = cudaGetLastError();
    if (e == cudaSuccess)
      e = cudaMemcpy(W.norms + (size_t)(l * 2) * kH, norm1[l], sizeof(float) * kH, cudaMemcpyDeviceToDevice);
    if (e == cudaSuccess)
      e = cudaMemcpy(W.norms + (size_t)(l * 2 + 1) * kH, norm2[l], sizeof(float) * kH, cudaMemcpyDeviceToDevice);
  }
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaFree(didx);
  if (e != cudaSuccess) return e;
  // pre-tile every packed matrix in place (through a scratch copy)
  uint16_t* tmp = nullptr;
  if ((e = cudaMalloc(&tmp, std::max(std::max(nq, no), std::max(ng, nd)) * 2)) != cudaSuccess) return e;
  struct T {
    uint16_t* p;
    size_t n;
    int N, K;
  } mats[2] = {{W.qkv, nq, kQkvN, kH}, {W.gu, ng, kGuN, kH}};  // o / down are blocked already
  for (auto& m : mats) {
    if (e == cudaSuccess) e = cudaMemcpy(tmp, m.p, m.n * 2, cudaMemcpyDeviceToDevice);
    if (e == cudaSuccess) {
      const size_t threads = m.n / 64 * 8;
      tile_kernel<<<(unsigned)((threads + 255) / 256), 256>>>(m.p, tmp, m.N, m.K);
      e = cudaGetLastError();
    }
  }
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaFree(tmp);
  if (e != cudaSuccess) return e;
  if (!make_map(&W.tm_qkv, W.qkv, (int)(nq / 64), 64, 2 * kQkvN) || !make_map_sw64(&W.tm_o, W.o, (int)(no / 32)) ||
      !make_map(&W.tm_gu, W.gu, (int)(ng / 64), 64, kGuN) || !make_map_sw64(&W.tm_dn, W.dn, (int)(nd / 32)))
    return cudaErrorInvalidPitchValue;
  return cudaSuccess;
}

void dit_cluster_free(DitClusterW& W) {
  cudaFree(W.qkv);
  cudaFree(W.o);
  cudaFree(W.gu);
  cudaFree(W.dn);
  cudaFree(W.norms);
  W = DitClusterW();
}

cudaError_t launch_dit_cluster(const DitClusterW& W, const DitClusterArgs& a, cudaStream_t s) {
  if (a.R <= 0) return cudaSuccess;
  if (a.NL != W.NL || a.steps <= 0 || a.steps > Sh::kMaxSteps) return cudaErrorInvalidValue;
  const size_t smem = dit_cluster_smem(a.NL);
  cudaError_t e = set_attrs(dit_cluster_smem(Sh::kMaxNL));
  if (e != cudaSuccess) return e;
  cudaLaunchAttribute attr[2];
  cudaLaunchConfig_t cfg = make_cfg((a.R + kU - 1) / kU, smem, s, attr, pdl_enabled());
  e = cudaLaunchKernelEx(&cfg, dit_cluster_kernel, W.tm_qkv, W.tm_o, W.tm_gu, W.tm_dn, a);
  if (e != cudaSuccess) (void)cudaGetLastError();
  return e;
}

}  // namespace ctts

#ifdef CTTS_DIT_TRACE
// Copies the recorded timeline out (role 0 compute, 1 MMA) and resets it.
extern "C" __attribute__((visibility("default"))) int ctts_dit_trace(long long* out0, int* n0, long long* out1,
                                                                     int* n1) {
  int n[2];
  cudaMemcpyFromSymbol(n, ctts::g_dit_trace_n, sizeof(n));
  cudaMemcpyFromSymbol(out0, ctts::g_dit_trace, sizeof(long long) * 8192, 0);
  cudaMemcpyFromSymbol(out1, ctts::g_dit_trace, sizeof(long long) * 8192, sizeof(long long) * 8192);
  *n0 = n[0];
  *n1 = n[1];
  n[0] = ctts::dit_cluster_max_active();
  fprintf(stderr, "dit_cluster_max_active=%d\n", n[0]);
  int z[2] = {0, 0};
  return cudaMemcpyToSymbol(ctts::g_dit_trace_n, z, sizeof(z)) == cudaSuccess ? 0 : -2;
}
#endif
