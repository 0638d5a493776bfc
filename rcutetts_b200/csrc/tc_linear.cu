// tc_linear.cu -- bf16 linear layers on the 5th-generation tensor cores
// (tcgen05.mma with the accumulator in TMEM, operands staged by TMA).
//
// Replaces the packed SGEMM for batched decode (gemm.rs:45-291 sgemm_bias,
// simd.rs:256-270 micro_8x8) when weights are bf16 and the batch has >= 16
// rows.  Swap-AB: the weight matrix W[N, K] is the MMA's A operand (128
// weight rows per CTA on the MMA M side) and the activations X[M, K] the B
// operand (the batch on the MMA N side, 16..256), so D[n, m] = sum_k W[n,k]
// X[m,k] lives in TMEM with one weight row per TMEM lane.
//
// Pipeline per CTA (128 threads): thread 0 issues TMA loads of 64-wide K
// blocks of W and X into an S-stage shared-memory ring (128-byte swizzle),
// thread 32 issues four K=16 MMAs per block and commits each stage back to
// the producer, then all four warps read the accumulator with tcgen05.ld
// (warp w owns TMEM lanes 32w..32w+31).  The K range is split over
// `splitk` CTAs per 128-row tile when the tile count alone cannot fill the
// GPU; partial tiles go to a scratch buffer and the last CTA of a tile (an
// atomic ticket) sums them in split order -- deterministic -- and runs the
// epilogue: bias, SwiGLU (tile rows 0..63 gate, 64..127 up), AdaLN gate,
// residual, fp32 or bf16 output.
//
// Every wait on an mbarrier is bounded; on timeout the CTA records an error
// code, skips the rest of its work, releases its TMEM and returns.
#include <cuda.h>

#include <cstdlib>

#include "common.cuh"
#include "launch_state.h"
#include "tc_linear.cuh"
#include "tc_ptx.cuh"

namespace ctts {

namespace {

// Optional phase timeline (build with -DCTTS_TC_TRACE): thread 0 of the
// first CTA of the grid records %globaltimer per event and launch.
#ifdef CTTS_TC_TRACE
// Consecutive launches overlap (programmatic dependent launch): the launch
// number is taken atomically once, at event 0 (after its timestamp); later
// events store into their own slot without waiting on memory.
constexpr int kTcTraceLaunches = 256, kTcTraceEvents = 16;
__device__ long long g_tc_trace[kTcTraceLaunches * kTcTraceEvents];
__device__ int g_tc_launch;
CTTS_DEV void tc_trace(int ev) {
  if (blockIdx.x != 0 || blockIdx.y != 0 || threadIdx.x != 0) return;
  __shared__ int lid;
  long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  if (ev == 0) lid = atomicAdd(&g_tc_launch, 1);
  if (lid < kTcTraceLaunches && ev < kTcTraceEvents) g_tc_trace[lid * kTcTraceEvents + ev] = t;
}
#define TC_TRACE(ev) tc_trace(ev)
#else
#define TC_TRACE(ev)
#endif

constexpr int kBK = 64;            // K elements per stage (128 bytes of bf16)
constexpr int kTileN = 128;        // weight rows per CTA (MMA M)
// Epilogue of four adjacent output columns of row m, y = res + coef * val
// (coef = 1 + AdaLN gate, or `scale`), split in two halves so a thread can
// issue the global loads of several output units before any of their stores.
struct Epi4 {
  float g[4], r[4];
};
CTTS_DEV void epi_fetch(const TcArgs& a, int m, int col, int n, Epi4& e) {
  const long yo = (long)m * a.y_ld + col;
  const float* gp = a.gate ? a.gate + (long)(m / a.gate_div) * a.gate_ld + a.gate_off + col : nullptr;
  if (n == 4 && (yo & 3) == 0 && (!gp || ((reinterpret_cast<uintptr_t>(gp) & 15) == 0))) {
    float4 gv = gp ? *reinterpret_cast<const float4*>(gp) : make_float4(0.f, 0.f, 0.f, 0.f);
    float4 rv = a.res ? *reinterpret_cast<const float4*>(a.res + yo) : make_float4(0.f, 0.f, 0.f, 0.f);
    e.g[0] = gv.x; e.g[1] = gv.y; e.g[2] = gv.z; e.g[3] = gv.w;
    e.r[0] = rv.x; e.r[1] = rv.y; e.r[2] = rv.z; e.r[3] = rv.w;
  } else {
#pragma unroll
    for (int j = 0; j < 4; j++) {
      e.g[j] = (gp && j < n) ? gp[j] : 0.0f;
      e.r[j] = (a.res && j < n) ? a.res[yo + j] : 0.0f;
    }
  }
}
// The next RMSNorm's gains for four output columns (zero where n < 4).
CTTS_DEV float4 epi_gains(const TcArgs& a, int col, int n) {
  if (!a.yb2) return make_float4(0.f, 0.f, 0.f, 0.f);
  if (n == 4 && (reinterpret_cast<uintptr_t>(a.g2 + col) & 15) == 0) return *reinterpret_cast<const float4*>(a.g2 + col);
  return make_float4(n > 0 ? a.g2[col] : 0.f, n > 1 ? a.g2[col + 1] : 0.f, n > 2 ? a.g2[col + 2] : 0.f,
                     n > 3 ? a.g2[col + 3] : 0.f);
}
// 1/rms of activation row m from the folded-norm partial sums (1 without).
// The first 16 partials are requested together (one round trip to L2 for
// the usual widths) and summed in tile order like the rest.
CTTS_DEV float epi_rinv(const TcArgs& a, int m) {
  if (!a.rs_ssp) return 1.0f;
  constexpr int kBatch = 16;
  float v[kBatch];
#pragma unroll
  for (int t = 0; t < kBatch; t++) v[t] = t < a.rs_nt ? a.rs_ssp[(long)t * a.rs_ld + m] : 0.0f;
  float ss = 0.0f;
#pragma unroll
  for (int t = 0; t < kBatch; t++)
    if (t < a.rs_nt) ss += v[t];
  for (int t = kBatch; t < a.rs_nt; t++) ss += a.rs_ssp[(long)t * a.rs_ld + m];
  return 1.0f / sqrtf(ss / a.rs_k + a.rs_eps);
}
CTTS_DEV void epi_store(const TcArgs& a, int m, int col, int n, const float* val, const Epi4& e, const float4& g,
                        float* out) {
  const long yo = (long)m * a.y_ld + col;
#pragma unroll
  for (int j = 0; j < 4; j++) out[j] = e.r[j] + (a.gate ? 1.0f + e.g[j] : a.scale) * val[j];
  if (a.yb2) {  // the next RMSNorm's operand, gain applied, scale folded downstream
    if (n == 4 && (yo & 3) == 0) {
      uint2 pk;
      pk.x = (uint32_t)f2bf(out[0] * g.x) | ((uint32_t)f2bf(out[1] * g.y) << 16);
      pk.y = (uint32_t)f2bf(out[2] * g.z) | ((uint32_t)f2bf(out[3] * g.w) << 16);
      *reinterpret_cast<uint2*>(a.yb2 + yo) = pk;
    } else {
      const float gg[4] = {g.x, g.y, g.z, g.w};
      for (int j = 0; j < n; j++) a.yb2[yo + j] = f2bf(out[j] * gg[j]);
    }
  }
  if (n == 4 && (yo & 3) == 0) {
    if (a.yb) {
      uint2 pk;
      pk.x = (uint32_t)f2bf(out[0]) | ((uint32_t)f2bf(out[1]) << 16);
      pk.y = (uint32_t)f2bf(out[2]) | ((uint32_t)f2bf(out[3]) << 16);
      *reinterpret_cast<uint2*>(a.yb + yo) = pk;
    } else {
      *reinterpret_cast<float4*>(a.y + yo) = make_float4(out[0], out[1], out[2], out[3]);
    }
    return;
  }
  for (int j = 0; j < n; j++) {
    if (a.yb)
      a.yb[yo + j] = f2bf(out[j]);
    else
      a.y[yo + j] = out[j];
  }
}

// SW: the SwiGLU epilogue (act 2); SPLIT: K split over a cluster (else the
// CTA's own accumulator is the whole sum).  The epilogue runs several
// rounds of output units per thread for wide tiles (a 64-row tile of a
// 12288-column AdaLN projection: 8), so its dead paths are compiled out.
template <bool SW, bool SPLIT>
__global__ void __launch_bounds__(128)
    tc_linear_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                     const TcArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  TC_TRACE(0);
  // 1024-byte alignment for the swizzled tiles, by an offset into the
  // shared array (not through an integer cast), so the compiler keeps every
  // access through it in shared space
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int S = a.stages;
  const int bbytes = a.MT * 128;
  const size_t stage_bytes = 16384 + (size_t)bbytes;
  // barriers sit after both the stage ring and the epilogue exchange area
  const size_t xch_bytes = (size_t)a.MT * kTileN * 4;  // fp32 partial tile (phase 1)
  const size_t region = (size_t)S * stage_bytes > xch_bytes ? (size_t)S * stage_bytes : xch_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + ((region + 15) & ~size_t(15)));
  uint64_t* full = bars;
  uint64_t* empty = bars + S;
  uint64_t* done = bars + 2 * S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 1);
  int* flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tile = blockIdx.x, split = blockIdx.y;
  const int n0 = tile * kTileN;
  const int kb0 = (int)(((long)split * a.kblocks) / a.splitk);
  const int kb1 = (int)(((long)(split + 1) * a.kblocks) / a.splitk);
  const int nk = kb1 - kb0;
  const uint32_t ncols = a.tmem_cols;

  if (tid == 0) {
    for (int s = 0; s < S; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    *flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(ncols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  TC_TRACE(1);

  // Weights do not depend on the previous kernel: their first stages are
  // fetched before waiting on it (programmatic dependent launch), the
  // activation tiles only after.
  const int pre = nk < S ? nk : S;
  if (tid == 0) {
    for (int i = 0; i < pre; i++) {
      uint8_t* sa = smem + (size_t)i * stage_bytes;
      mbar_add_tx(&full[i], 16384u);
      tma_load_2d(sa, &tmW, (kb0 + i) * kBK, n0, &full[i]);
    }
  }
  grid_dep_wait();
  grid_dep_launch();
  TC_TRACE(2);

  bool ok = true;
  if (tid == 0) {  // ---- TMA producer
    for (int i = 0; i < nk && ok; i++) {
      const int s = i % S;
      uint8_t* sa = smem + (size_t)s * stage_bytes;
      if (i >= S) {
        ok = mbar_wait(&empty[s], ((i / S) - 1) & 1);
        if (!ok) break;
        mbar_expect_tx(&full[s], (uint32_t)stage_bytes);
        tma_load_2d(sa, &tmW, (kb0 + i) * kBK, n0, &full[s]);
      } else {
        mbar_expect_tx(&full[s], (uint32_t)(stage_bytes - 16384));
      }
      tma_load_2d(sa + 16384, &tmX, (kb0 + i) * kBK, a.m0, &full[s]);
    }
  } else if (tid == 32) {  // ---- MMA issuer
    const uint32_t idesc = umma_idesc(a.MT);
    for (int i = 0; i < nk && ok; i++) {
      const int s = i % S;
      ok = mbar_wait(&full[s], (i / S) & 1);
      if (!ok) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t sa = smem_u32(smem + (size_t)s * stage_bytes);
      const uint32_t sb = sa + 16384;
#pragma unroll
      for (int kk = 0; kk < kBK / 16; kk++)
        umma_bf16(tmem, umma_desc(sa + kk * 32), umma_desc(sb + kk * 32), idesc, (i > 0 || kk > 0) ? 1u : 0u);
      umma_commit(&empty[s]);
    }
    if (ok) umma_commit(done);
  }
  if (!ok) atomicExch(flag, 1);
  __syncwarp();

  // ---- epilogue operands that do not depend on the accumulator (residual,
  // AdaLN gate, next-norm gains, folded-norm row scale) of this thread's
  // first round of output units, fetched while the MMAs run.  Output unit u
  // of this CTA = row m_lo + u / groups, four columns at (u % groups) * 4.
  const int mcount = min(a.MT, a.M - a.m0);
  const int rows_per = (mcount + a.splitk - 1) / a.splitk;
  const int m_lo = split * rows_per, m_hi = min(mcount, m_lo + rows_per);
  constexpr bool sw = SW;
  constexpr int groups = sw ? 16 : 32;
  constexpr int gshift = sw ? 4 : 5;  // log2(groups)
  const int nunits = max(0, m_hi - m_lo) * groups;
  constexpr int kU = 2;
  auto unit_geom = [&](int u, int& em, int& ec, int& en) {
    const int m = m_lo + (u >> gshift), c = (u & (groups - 1)) * 4;
    em = a.m0 + m;
    ec = sw ? tile * 64 + c : n0 + c;
    en = u < nunits ? (sw ? 4 : max(0, min(4, a.N - (n0 + c)))) : 0;
  };
  // the operands of round r + 1 are requested at the start of round r
  auto fetch_round = [&](int u0, Epi4* ep, float* rinv, float4* g) {
#pragma unroll
    for (int q = 0; q < kU; q++) {
      int em, ec, en;
      unit_geom(u0 + q * 128, em, ec, en);
      rinv[q] = 1.0f;
      g[q] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (en > 0) {
        epi_fetch(a, em, ec, en, ep[q]);
        rinv[q] = epi_rinv(a, em);
        g[q] = epi_gains(a, ec, en);
      }
    }
  };
  Epi4 cur_ep[kU];
  float cur_rinv[kU];
  float4 cur_g[kU];
  fetch_round(tid, cur_ep, cur_rinv, cur_g);
  // a thread's column group is the same in every round (the round and unit
  // strides are multiples of the group count): its bias, loaded once
  const int cb = (tid % groups) * 4;
  float bias_g[4], bias_u[4];
#pragma unroll
  for (int j = 0; j < 4; j++) {
    bias_g[j] = (a.bias && (sw || n0 + cb + j < a.N)) ? a.bias[n0 + cb + j] : 0.0f;
    bias_u[j] = (a.bias && sw) ? a.bias[n0 + 64 + cb + j] : 0.0f;
  }

  // ---- epilogue: every warp waits for the accumulator
  bool have = mbar_wait(done, 0);
  TC_TRACE(3);
  if (!have) atomicExch(flag, 1);
  __syncthreads();
  const bool failed = *flag != 0;
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");

  const int r = warp * 32 + lane;  // TMEM lane = W row within the tile
  const uint32_t tl = tmem + ((uint32_t)(warp * 32) << 16);
  // ---- phase 1: accumulator -> this CTA's partial tile in shared memory
  // (the stage ring is free once every MMA has completed): part[m][128].
  float* part = reinterpret_cast<float*>(smem);
  if (!failed) {
    // four 16-column loads in flight per wait
    for (int c0 = 0; c0 < a.MT; c0 += 64) {
      uint32_t v[4][16];
#pragma unroll
      for (int q = 0; q < 4; q++)
        if (c0 + 16 * q < a.MT) tmem_ld16_nowait(tl + c0 + 16 * q, v[q]);
      tmem_wait();
#pragma unroll
      for (int q = 0; q < 4; q++)
        if (c0 + 16 * q < a.MT)
#pragma unroll
          for (int j = 0; j < 16; j++) part[(c0 + 16 * q + j) * kTileN + r] = __uint_as_float(v[q][j]);
    }
  }
  TC_TRACE(4);
  // every split of this tile (one cluster) has its partial in shared memory
  cluster_sync();
  TC_TRACE(5);

  // ---- phase 2: CTA `split` reduces rows [m_lo, m_hi) of the tile over all
  // splits, in split order (deterministic), reading peers over DSMEM, and
  // runs the epilogue on float4 column groups.
  // a failed peer leaves a garbage partial: lane s reads split s's flag
  const uint32_t peer_flag =
      (SPLIT && lane < a.splitk) ? ld_dsmem_u32(mapa_shared(smem_u32(flag), (uint32_t)lane)) : 0u;
  const bool any_failed = failed || __any_sync(0xffffffffu, peer_flag != 0u);
  if (!any_failed) {
    const uint32_t my_base = smem_u32(part);
    // kU output units per thread per round: every DSMEM partial of the round
    // is requested before the first sum, and the epilogue's global loads of
    // the round are issued before its stores (prefetched for round one).
    for (int u0 = tid; u0 < nunits; u0 += 128 * kU) {
      Epi4 nxt_ep[kU];
      float nxt_rinv[kU];
      float4 nxt_g[kU];
      fetch_round(u0 + 128 * kU, nxt_ep, nxt_rinv, nxt_g);
      float acc[kU][4], accu[kU][4];
#pragma unroll
      for (int q = 0; q < kU; q++) {
        const int u = u0 + q * 128;
        float4 tg[8], tu[8];
        const int m = m_lo + (u >> gshift), c = (u & (groups - 1)) * 4;
        const uint32_t off = (uint32_t)(m * kTileN + c) * 4u;
#pragma unroll
        for (int s0 = 0; s0 < (SPLIT ? 8 : 1); s0++) {
          if (u < nunits && s0 < a.splitk) {
            if (!SPLIT || s0 == split) {  // this CTA's own partial: a local read
              tg[s0] = *reinterpret_cast<const float4*>(part + m * kTileN + c);
              if (sw) tu[s0] = *reinterpret_cast<const float4*>(part + m * kTileN + c + 64);
            } else {
              const uint32_t remote = mapa_shared(my_base + off, (uint32_t)s0);
              tg[s0] = ld_dsmem_f4(remote);
              if (sw) tu[s0] = ld_dsmem_f4(remote + 64u * 4u);
            }
          }
        }
#pragma unroll
        for (int j = 0; j < 4; j++) acc[q][j] = accu[q][j] = 0.0f;
#pragma unroll
        for (int s0 = 0; s0 < (SPLIT ? 8 : 1); s0++) {
          if (u < nunits && s0 < a.splitk) {
            acc[q][0] += tg[s0].x; acc[q][1] += tg[s0].y; acc[q][2] += tg[s0].z; acc[q][3] += tg[s0].w;
            if (sw) {
              accu[q][0] += tu[s0].x; accu[q][1] += tu[s0].y; accu[q][2] += tu[s0].z; accu[q][3] += tu[s0].w;
            }
          }
        }
      }
      if (u0 == tid) TC_TRACE(8);
      // epilogue with the operands fetched a round ago (during the
      // mainloop for round one)
      int em[kU], ec[kU], en[kU];
#pragma unroll
      for (int q = 0; q < kU; q++) unit_geom(u0 + q * 128, em[q], ec[q], en[q]);
#pragma unroll
      for (int q = 0; q < kU; q++) {
        const int u = u0 + q * 128;
        float sq = 0.0f;
        if (en[q] > 0) {  // rinv: folded RMSNorm of activation row em[q]
          const float rinv = cur_rinv[q];
          float val[4], out[4];
#pragma unroll
          for (int j = 0; j < 4; j++) {
            if (sw)
              val[j] = silu(acc[q][j] * rinv + bias_g[j]) * (accu[q][j] * rinv + bias_u[j]);
            else
              val[j] = acc[q][j] * rinv + (j < en[q] ? bias_g[j] : 0.0f);
          }
          epi_store(a, em[q], ec[q], en[q], val, cur_ep[q], cur_g[q], out);
          for (int j = 0; j < en[q]; j++) sq = fmaf(out[j], out[j], sq);
        }
        // one warp covers one output row of the tile (32 groups of 4
        // columns): its sum of squares over the tile's columns
        if (a.ssp) {
          sq = warp_sum(sq);
          if (lane == 0 && u < nunits) a.ssp[(long)tile * a.ssp_ld + em[q]] = sq;
        }
      }
#pragma unroll
      for (int q = 0; q < kU; q++) {
        cur_ep[q] = nxt_ep[q];
        cur_rinv[q] = nxt_rinv[q];
        cur_g[q] = nxt_g[q];
      }
    }
  } else if (tid == 0 && a.err) {
    atomicExch(a.err, 2);
  }
  TC_TRACE(6);
  // no CTA leaves while a peer may still read its shared memory
  cluster_sync();
  TC_TRACE(7);

  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols));
}

// ---------------------------------------------------------- host helpers

}  // namespace


EncodeTiledFn encode_fn() {
  static const EncodeTiledFn fn = [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<EncodeTiledFn>(p);
    (void)cudaGetLastError();
    return EncodeTiledFn(nullptr);
  }();
  return fn;
}

// 2D bf16 tensor [rows, cols] (cols contiguous), box [box_rows, 64], SW128.
bool make_map(CUtensorMap* m, const void* base, int rows, int cols, int box_rows) {
  constexpr int kBK = 64;
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}


int tc_num_sms() {
  const int n = device_sms();
  return n > 0 ? n : 148;
}

TcPlan tc_plan(int M, int N, int K, int num_sms, int max_splitk) {
  TcPlan p;
  p.MT = ((std::min(M, 256) + 15) / 16) * 16;
  p.mtiles = (M + p.MT - 1) / p.MT;
  p.ntiles = (N + kTileN - 1) / kTileN;
  p.kblocks = K / kBK;
  // the K splits of one tile form a thread-block cluster (<= 8, portable);
  // aim for about one wave of CTAs.  CTTS_TC_MAX_SPLITK caps the split.
  static const int env_cap = [] {
    const char* e = getenv("CTTS_TC_MAX_SPLITK");
    return e ? std::max(1, atoi(e)) : 8;
  }();
  max_splitk = std::min(max_splitk, env_cap);
  // a power of two, one CTA per SM; where that leaves the K unsplit (tiles
  // beyond the SM count: a tile's epilogue then covers all its rows, e.g. 8
  // rounds for the 96 tiles of the DiT's AdaLN projection), two CTAs per SM
  // and a split of 2 when the tile's partial (MT x 128 floats) leaves room
  // (a larger split of tiles that already split measured slower)
  const int ctas_per_split = p.ntiles * p.mtiles;
  const int per_sm = (num_sms / ctas_per_split < 2 && p.MT <= 128) ? 2 : 1;
  int sk = std::max(1, std::min(std::min(std::min(per_sm * num_sms / ctas_per_split, p.kblocks), max_splitk), 8));
  while (sk & (sk - 1)) sk &= sk - 1;
  p.splitk = sk;
  const int kb_per = (p.kblocks + p.splitk - 1) / p.splitk;
  const size_t stage = 16384 + (size_t)p.MT * 128;
  // a grid beyond one CTA per SM keeps two CTAs per SM resident
  const size_t budget = ctas_per_split * p.splitk > num_sms ? 100 * 1024 : 200 * 1024;
  p.stages = std::max(1, std::min(kb_per, (int)(budget / stage)));
  p.stages = std::min(p.stages, 8);
  size_t pipe = (size_t)p.stages * stage;
  size_t xch = (size_t)p.MT * kTileN * 4;
  p.smem = ((std::max(pipe, xch) + 15) & ~size_t(15)) + 1024 /*align*/ + 8 * (2 * p.stages + 1) + 16;
  int cols = 32;
  while (cols < p.MT) cols <<= 1;
  p.tmem_cols = cols;
  return p;
}

size_t tc_scratch_floats(const TcPlan& p) {
  (void)p;
  return 0;  // split-K partials stay in the cluster's shared memory
}

cudaError_t launch_tc_linear(const TcCall& c, cudaStream_t s) {
  if (c.K % kBK != 0 || c.M <= 0 || c.N <= 0) return cudaErrorInvalidValue;
  // row statistics need one warp per output row (no SwiGLU column pairing)
  if ((c.epi.ssp || c.epi.yb2) && (c.epi.act == 2 || c.epi.yb || !c.epi.y)) return cudaErrorInvalidValue;
  if (c.epi.yb2 && !c.epi.g2) return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(c.w) & 15) || (reinterpret_cast<uintptr_t>(c.x) & 15))
    return cudaErrorInvalidValue;
  TcPlan p = tc_plan(c.M, c.N, c.K, tc_num_sms(), c.max_splitk);
  const bool sw = c.epi.act == 2, ksplit = p.splitk > 1;
  auto kern = sw ? (ksplit ? tc_linear_kernel<true, true> : tc_linear_kernel<true, false>)
                 : (ksplit ? tc_linear_kernel<false, true> : tc_linear_kernel<false, false>);
  static SmemOptIn opts[4];  // dynamic smem opt-in per device and instance (static smem is tiny)
  if (cudaError_t e = opts[(sw ? 2 : 0) + (ksplit ? 1 : 0)].ensure((const void*)kern, p.smem)) return e;
  CUtensorMap tmW, tmX;
  // distinct codes for the tensor-map failures (diagnostics)
  if (!encode_fn()) return cudaErrorNotSupported;
  if (!make_map(&tmW, c.w, c.N, c.K, kTileN)) return cudaErrorInvalidPitchValue;
  if (!make_map(&tmX, c.x, c.M, c.K, p.MT)) return cudaErrorInvalidPitchValue;
  for (int mt = 0; mt < p.mtiles; mt++) {
    TcArgs a = c.epi;
    a.M = c.M;
    a.N = c.N;
    a.m0 = mt * p.MT;
    a.MT = p.MT;
    a.kblocks = p.kblocks;
    a.splitk = p.splitk;
    a.stages = p.stages;
    a.tmem_cols = p.tmem_cols;
    a.err = c.err;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.ntiles, p.splitk, 1);
    cfg.blockDim = dim3(128);
    cfg.dynamicSmemBytes = p.smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = p.splitk;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tmW, tmX, a);
    if (e != cudaSuccess) {
      (void)cudaGetLastError();
      return e;
    }
  }
  return cudaSuccess;
}

}  // namespace ctts

#ifdef CTTS_TC_TRACE
// Copies the recorded timeline out ([launch][event] timestamps, 0 = not
// recorded; *n = launches) and resets it.
extern "C" __attribute__((visibility("default"))) int ctts_tc_trace(long long* out, int* n) {
  cudaMemcpyFromSymbol(n, ctts::g_tc_launch, sizeof(int));
  if (*n > ctts::kTcTraceLaunches) *n = ctts::kTcTraceLaunches;
  cudaMemcpyFromSymbol(out, ctts::g_tc_trace, sizeof(ctts::g_tc_trace));
  static long long zeros[ctts::kTcTraceLaunches * ctts::kTcTraceEvents] = {};
  cudaMemcpyToSymbol(ctts::g_tc_trace, zeros, sizeof(zeros));
  int z = 0;
  return cudaMemcpyToSymbol(ctts::g_tc_launch, &z, sizeof(int)) == cudaSuccess ? 0 : -2;
}
#endif
