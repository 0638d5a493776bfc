// attention.cu -- LM attention blocks and small LM ops.
//
// qk_rope_append: QK-Norm + NeoX RoPE of the new q/k rows and the KV-cache
//   append for prefill rows (qwen.rs:255-272).
// attn_step: the whole decode-step attention of a layer in one launch --
//   query QK-Norm + RoPE, KV append of the new row, GQA attention over each
//   utterance's ragged cache (qwen.rs:323-362), split over the sequence so
//   a batch of one still fills the GPU, splits merged by the last CTA.
// attn_split: the batched decode step: each (utterance, KV head) is split
//   over the keys into a thread-block cluster of CTAs whose partial softmax
//   states merge over distributed shared memory (one wave for the batch).
// attn_prefill: causal attention of T new rows against the cache
//   (qwen.rs:273-297).
#include "common.cuh"
#include "kernels.cuh"
#include "launch_state.h"
#include "tc_ptx.cuh"

namespace ctts {

namespace {

constexpr int kMaxG = 8;     // query heads per KV head handled by one CTA
constexpr int kMaxHd = 128;  // head_dim upper bound (hd/32 values per lane)

template <bool BF>
CTTS_DEV float ld_kv(const void* base, size_t i) {
  if (BF) return bf2f(reinterpret_cast<const uint16_t*>(base)[i]);
  return reinterpret_cast<const float*>(base)[i];
}
template <bool BF>
CTTS_DEV void st_kv(void* base, size_t i, float v) {
  if (BF)
    reinterpret_cast<uint16_t*>(base)[i] = f2bf(v);
  else
    reinterpret_cast<float*>(base)[i] = v;
}

// one warp per (row, head); grid (rows, ceil((nq + 2nkv)/4)), 128 threads
template <bool BF>
__global__ void __launch_bounds__(128) qk_rope_append_kernel(const AttnArgs a) {
  grid_dep_enter();
  const int row = blockIdx.x;
  const int head = blockIdx.y * 4 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int nq = a.nq, nkv = a.nkv, hd = a.hd;
  if (head >= nq + 2 * nkv) return;
  const int b = a.prefill_b >= 0 ? a.prefill_b : row;
  const int pos = a.prefill_b >= 0 ? a.pos0 + row : a.pos[row];
  if (pos < 0 || pos >= a.cap) {
    if (lane == 0 && a.err) atomicExch(a.err, 1);
    return;
  }
  const int per = hd / 32;  // values per lane (2 for hd=64)
  const int width = (nq + 2 * nkv) * hd;
  const float* src = a.qkv + (size_t)row * width + head * hd;
  float v[kMaxHd / 32];
#pragma unroll
  for (int j = 0; j < kMaxHd / 32; j++) v[j] = j < per ? src[lane + 32 * j] : 0.0f;

  if (head >= nq + nkv) {  // V row -> cache
    const int kh = head - nq - nkv;
    size_t base = (((size_t)b * nkv + kh) * a.cap + pos) * hd;
#pragma unroll
    for (int j = 0; j < kMaxHd / 32; j++)
      if (j < per) st_kv<BF>(a.vcache, base + lane + 32 * j, v[j]);
    return;
  }
  const bool is_q = head < nq;
  const float* g = is_q ? a.qn : a.kn;
  if (g) {
    float ss = 0.0f;
#pragma unroll
    for (int j = 0; j < kMaxHd / 32; j++) ss = fmaf(v[j], v[j], ss);
    ss = warp_sum(ss);
    float inv = 1.0f / sqrtf(ss / (float)hd + a.eps);
#pragma unroll
    for (int j = 0; j < kMaxHd / 32; j++)
      if (j < per) v[j] = v[j] * inv * g[lane + 32 * j];
  }
  // rotate-half: element i pairs with i + hd/2; with hd/2 a multiple of 32
  // both live in this lane (j and j + per/2).
  float o[kMaxHd / 32];
  const int half = per / 2;
#pragma unroll
  for (int j = 0; j < kMaxHd / 64; j++) {
    if (j >= half) break;
    int i = lane + 32 * j;
    float ang = (float)pos * a.inv_freq[i];
    float sn, cs;
    sincosf(ang, &sn, &cs);
    float x1 = v[j], x2 = v[j + half];
    o[j] = x1 * cs - x2 * sn;
    o[j + half] = x1 * sn + x2 * cs;
  }
  if (is_q) {
    float* dst = a.qrot + (size_t)row * nq * hd + head * hd;
#pragma unroll
    for (int j = 0; j < kMaxHd / 32; j++)
      if (j < per) dst[lane + 32 * j] = o[j];
  } else {
    const int kh = head - nq;
    size_t base = (((size_t)b * nkv + kh) * a.cap + pos) * hd;
#pragma unroll
    for (int j = 0; j < kMaxHd / 32; j++)
      if (j < per) st_kv<BF>(a.kcache, base + lane + 32 * j, o[j]);
  }
}

// Fused decode step of one layer's attention (qwen.rs:323-362): QK-Norm +
// NeoX RoPE of the step's queries, the KV-cache append of the new key/value
// row, GQA attention over each utterance's ragged cache and the merge of
// the sequence splits -- one launch.
//
// grid (nsplit, nkv, batch), 128 threads.  CTA (split, kv head, utterance)
// owns keys [split*chunk, +chunk) of that utterance.  The cached rows of
// the range are contiguous in the cache ([b][kv head][cap][hd]), so one bulk
// copy each brings K and V into shared memory, issued before the wait on the
// previous kernel (they were written frames ago).  The CTA whose range
// holds the new position also normalises/rotates the new key, rounds it to
// the cache type and writes it to the cache and to its shared tile.  Every
// query head of the group is scored against the tile (K/V read once per
// group), the online-softmax partial [m, l, acc[hd]] goes to global memory,
// and the last CTA of the (utterance, kv head) -- an atomic ticket --
// merges the splits in split order (deterministic) and writes the output.
template <bool BF, int HD>
__global__ void __launch_bounds__(128) attn_step_kernel(const AttnArgs a) {
  constexpr int ES = BF ? 2 : 4;
  constexpr int ROWB = HD * ES;     // bytes of one cache row
  constexpr int NC = ROWB / 16;     // 16-byte chunks per row
  constexpr int VPC = 16 / ES;      // values per chunk
  constexpr int PER = HD / 32;      // values per lane of a head vector
  constexpr int HP = HD / 2;        // dim pairs
  constexpr int PARTS = 128 / HP;   // key partitions of the P.V pass
  extern __shared__ __align__(128) uint8_t kv_smem[];
  __shared__ __align__(16) float qs[kMaxG][HD];
  __shared__ float ps[kMaxG][128];
  __shared__ float red[kMaxG][4];
  __shared__ float stat[kMaxG][2];
  __shared__ __align__(16) float accs[PARTS][kMaxG][HD];
  __shared__ __align__(8) uint64_t bar;
  __shared__ int s_last;

  const int split = blockIdx.x, kh = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nq = a.nq, nkv = a.nkv, G = nq / nkv, chunk = a.chunk;
  uint8_t* Ks = kv_smem;
  uint8_t* Vs = kv_smem + (size_t)chunk * ROWB;
  const uint32_t bar_a = static_cast<uint32_t>(__cvta_generic_to_shared(&bar));

  const int pos = a.pos[b];
  const bool bad = pos < 0 || pos >= a.cap;
  const int n = bad ? 0 : pos + 1;  // keys incl. the row appended this step
  const int r0 = split * chunk, r1 = min(r0 + chunk, n);
  const int nrows = max(0, r1 - r0);
  const int ncached = max(0, min(r1, pos) - r0);  // rows already in the cache
  const size_t row0 = ((size_t)b * nkv + kh) * a.cap;  // cache row of key 0
  // the barrier is initialised before any thread can wait on it or any
  // copy can complete on it
  if (tid == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar_a));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (tid == 0) {
    if (ncached > 0) {
      const uint32_t bytes = (uint32_t)ncached * ROWB;
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar_a), "r"(2 * bytes)
                   : "memory");
      const uint8_t* ksrc = reinterpret_cast<const uint8_t*>(a.kcache) + (row0 + r0) * ROWB;
      const uint8_t* vsrc = reinterpret_cast<const uint8_t*>(a.vcache) + (row0 + r0) * ROWB;
      asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                       static_cast<uint32_t>(__cvta_generic_to_shared(Ks))),
                   "l"(ksrc), "r"(bytes), "r"(bar_a)
                   : "memory");
      asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                       static_cast<uint32_t>(__cvta_generic_to_shared(Vs))),
                   "l"(vsrc), "r"(bytes), "r"(bar_a)
                   : "memory");
    }
  }
  grid_dep_enter();
  if (bad && split == 0 && tid == 0 && a.err) atomicExch(a.err, 1);

  // ---- queries (and the new key/value row in its split): one warp per job
  const bool has_new = !bad && pos >= r0 && pos < r1;
  const int width = (nq + 2 * nkv) * HD;
  const float* src_row = a.qkv + (size_t)b * width;
  const int jobs = nrows > 0 ? G + (has_new ? 2 : 0) : 0;
  for (int job = warp; job < jobs; job += 4) {
    const bool is_q = job < G, is_v = job == G + 1;
    const int head = is_q ? kh * G + job : (is_v ? nq + nkv + kh : nq + kh);
    const float* src = src_row + head * HD;
    float v[PER];
#pragma unroll
    for (int j = 0; j < PER; j++) v[j] = src[lane + 32 * j];
    if (!is_v) {
      const float* gn = is_q ? a.qn : a.kn;
      if (gn) {
        float ss = 0.0f;
#pragma unroll
        for (int j = 0; j < PER; j++) ss = fmaf(v[j], v[j], ss);
        ss = warp_sum(ss);
        const float inv = 1.0f / sqrtf(ss / (float)HD + a.eps);
#pragma unroll
        for (int j = 0; j < PER; j++) v[j] = v[j] * inv * gn[lane + 32 * j];
      }
      // rotate-half: element i pairs with i + HD/2 (same lane, j + PER/2)
#pragma unroll
      for (int j = 0; j < PER / 2; j++) {
        const int i = lane + 32 * j;
        float sn, cs;
        sincosf((float)pos * a.inv_freq[i], &sn, &cs);
        const float x1 = v[j], x2 = v[j + PER / 2];
        v[j] = x1 * cs - x2 * sn;
        v[j + PER / 2] = x1 * sn + x2 * cs;
      }
    }
    if (is_q) {
#pragma unroll
      for (int j = 0; j < PER; j++) qs[job][lane + 32 * j] = v[j];
    } else {
      void* cache = is_v ? a.vcache : a.kcache;
      uint8_t* tile = (is_v ? Vs : Ks) + (size_t)(pos - r0) * ROWB;
#pragma unroll
      for (int j = 0; j < PER; j++) {
        const int d = lane + 32 * j;
        if constexpr (BF) {
          const uint16_t hb = f2bf(v[j]);
          reinterpret_cast<uint16_t*>(cache)[(row0 + pos) * HD + d] = hb;
          reinterpret_cast<uint16_t*>(tile)[d] = hb;
        } else {
          reinterpret_cast<float*>(cache)[(row0 + pos) * HD + d] = v[j];
          reinterpret_cast<float*>(tile)[d] = v[j];
        }
      }
    }
  }
  if (ncached > 0) {
    bool ok = false;
    for (uint32_t it = 0; it < (1u << 24) && !ok; ++it) {
      uint32_t done;
      asm volatile(
          "{\n\t.reg .pred p;\n\t"
          "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0;\n\t"
          "selp.u32 %0, 1, 0, p;\n\t}"
          : "=r"(done)
          : "r"(bar_a)
          : "memory");
      ok = done != 0;
    }
    if (!ok && a.err) atomicExch(a.err, 3);
  }
  __syncthreads();

  if (nrows > 0) {
    // ---- scores: one key per thread; the 16-byte chunks of a row are
    // visited in a per-thread rotated order (no bank conflicts)
    const float scale = 1.0f / sqrtf((float)HD);
    float sc[kMaxG];
#pragma unroll
    for (int g = 0; g < kMaxG; g++) sc[g] = -INFINITY;
    if (tid < nrows) {
#pragma unroll
      for (int g = 0; g < kMaxG; g++) sc[g] = 0.0f;
      const uint8_t* krow = Ks + (size_t)tid * ROWB;
#pragma unroll 4
      for (int cc = 0; cc < NC; cc++) {
        const int c = (cc + tid) % NC;
        const uint4 t = *reinterpret_cast<const uint4*>(krow + c * 16);
        float kv[VPC];
        if constexpr (BF) {
          kv[0] = bf_lo(t.x); kv[1] = bf_hi(t.x); kv[2] = bf_lo(t.y); kv[3] = bf_hi(t.y);
          kv[4] = bf_lo(t.z); kv[5] = bf_hi(t.z); kv[6] = bf_lo(t.w); kv[7] = bf_hi(t.w);
        } else {
          kv[0] = __uint_as_float(t.x); kv[1] = __uint_as_float(t.y);
          kv[2] = __uint_as_float(t.z); kv[3] = __uint_as_float(t.w);
        }
#pragma unroll
        for (int g = 0; g < kMaxG; g++) {
          if (g >= G) break;
          const float* q = qs[g] + c * VPC;
#pragma unroll
          for (int e = 0; e < VPC; e++) sc[g] = fmaf(q[e], kv[e], sc[g]);
        }
      }
#pragma unroll
      for (int g = 0; g < kMaxG; g++) sc[g] *= scale;
    }
    // ---- softmax statistics of the split
#pragma unroll
    for (int g = 0; g < kMaxG; g++) {
      if (g >= G) break;
      const float m = warp_max(sc[g]);
      if (lane == 0) red[g][warp] = m;
    }
    __syncthreads();
    if (tid < G) stat[tid][0] = fmaxf(fmaxf(red[tid][0], red[tid][1]), fmaxf(red[tid][2], red[tid][3]));
    __syncthreads();
#pragma unroll
    for (int g = 0; g < kMaxG; g++) {
      if (g >= G) break;
      const float p = tid < nrows ? expf(sc[g] - stat[g][0]) : 0.0f;
      ps[g][tid] = p;
      const float l = warp_sum(p);
      if (lane == 0) red[g][warp] = l;
    }
    __syncthreads();
    if (tid < G) stat[tid][1] = red[tid][0] + red[tid][1] + red[tid][2] + red[tid][3];
    // ---- P.V: thread -> (dim pair, key partition)
    const int dp = tid % HP, pp = tid / HP;
    float acc[kMaxG][2];
#pragma unroll
    for (int g = 0; g < kMaxG; g++) acc[g][0] = acc[g][1] = 0.0f;
    for (int j = pp; j < nrows; j += PARTS) {
      float v0, v1;
      if constexpr (BF) {
        const uint32_t t = reinterpret_cast<const uint32_t*>(Vs + (size_t)j * ROWB)[dp];
        v0 = bf_lo(t);
        v1 = bf_hi(t);
      } else {
        const float2 t = reinterpret_cast<const float2*>(Vs + (size_t)j * ROWB)[dp];
        v0 = t.x;
        v1 = t.y;
      }
#pragma unroll
      for (int g = 0; g < kMaxG; g++) {
        if (g >= G) break;
        const float p = ps[g][j];
        acc[g][0] = fmaf(p, v0, acc[g][0]);
        acc[g][1] = fmaf(p, v1, acc[g][1]);
      }
    }
#pragma unroll
    for (int g = 0; g < kMaxG; g++) {
      if (g >= G) break;
      accs[pp][g][2 * dp] = acc[g][0];
      accs[pp][g][2 * dp + 1] = acc[g][1];
    }
    __syncthreads();
    // ---- partial [m, l, acc[HD]] per query head, partitions summed in order
    const size_t pstride = (size_t)a.nsplit * (HD + 2);
    float* pbase = a.part + (((size_t)b * nq + kh * G) * a.nsplit + split) * (HD + 2);
    for (int i = tid; i < G * HD; i += 128) {
      const int g = i / HD, d = i % HD;
      float t = 0.0f;
#pragma unroll
      for (int q = 0; q < PARTS; q++) t += accs[q][g][d];
      pbase[g * pstride + 2 + d] = t;
    }
    if (tid < G) {
      pbase[tid * pstride] = stat[tid][0];
      pbase[tid * pstride + 1] = stat[tid][1];
    }
  }
  // ---- ticket: the last CTA of (utterance, kv head) merges the splits
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    int* cnt = a.cnt + (size_t)b * nkv + kh;
    const int t = atomicAdd(cnt, 1);
    s_last = t == a.nsplit - 1;
    if (s_last) *cnt = 0;  // ready for the next launch
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const int nsa = (n + chunk - 1) / chunk;  // splits that hold keys
  for (int i = tid; i < G * HD; i += 128) {
    const int g = i / HD, d = i % HD, h = kh * G + g;
    const float* pb = a.part + ((size_t)b * nq + h) * a.nsplit * (HD + 2);
    float M = -INFINITY;
    for (int s2 = 0; s2 < nsa; s2++) M = fmaxf(M, __ldcg(pb + (size_t)s2 * (HD + 2)));
    float L = 0.0f, acc = 0.0f;
    for (int s2 = 0; s2 < nsa; s2++) {
      const float* q = pb + (size_t)s2 * (HD + 2);
      const float w = expf(__ldcg(q) - M);
      L = fmaf(__ldcg(q + 1), w, L);
      acc = fmaf(__ldcg(q + 2 + d), w, acc);
    }
    const float o = nsa > 0 ? acc / L : 0.0f;
    const size_t oi = (size_t)b * nq * HD + (size_t)h * HD + d;
    if (a.out_b)
      a.out_b[oi] = f2bf(o);
    else
      a.out[oi] = o;
  }
}

// Optional phase timeline (build with -DCTTS_ATT_TRACE): thread 0 of the
// first CTA of every decode-attention launch records %globaltimer per event.
#ifdef CTTS_ATT_TRACE
// The launch number is taken atomically once, at event 0 (after its
// timestamp); later events store into their own [launch][event] slot.
constexpr int kAttTraceLaunches = 128, kAttTraceEvents = 16;
__device__ long long g_att_trace[kAttTraceLaunches * kAttTraceEvents];
__device__ int g_att_launch;
CTTS_DEV void att_trace(int ev) {
  if (blockIdx.x != 0 || blockIdx.y != 0 || blockIdx.z != 0 || threadIdx.x != 0) return;
  __shared__ int lid;
  long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  if (ev == 0) lid = atomicAdd(&g_att_launch, 1);
  if (lid < kAttTraceLaunches && ev < kAttTraceEvents) g_att_trace[lid * kAttTraceEvents + ev] = t;
}
#define ATT_TRACE(ev) att_trace(ev)
#else
#define ATT_TRACE(ev)
#endif

// Large-batch form of the same decode step: one CTA per (kv head,
// utterance) walks the utterance's keys in 128-key stages through a
// two-stage ring of bulk copies (the copy of stage s+2 is issued as soon as
// stage s is consumed) with an online softmax, so there is no split merge
// and the grid is one wave.  Each warp owns 16 keys of every stage and keeps
// its own softmax state in registers (one block barrier per stage); the 8
// warp states merge once at the end, in warp order.  The new key/value row is kept in shared memory
// and placed into its stage's tile once that stage's copy has landed.
// grid (nkv, batch), 256 threads, dynamic smem 2 stages x (K, V) x 128 rows.
template <bool BF, int HD, int GM>
__global__ void __launch_bounds__(256) attn_loop_kernel(const AttnArgs a) {
  constexpr int ES = BF ? 2 : 4;
  constexpr int ROWB = HD * ES;
  constexpr int NC = ROWB / 16;
  constexpr int VPC = 16 / ES;
  constexpr int PER = HD / 32;
  constexpr int C = 128;             // keys per stage
  constexpr int NT = 256;
  constexpr int NW = NT / 32;
  constexpr int KPW = C / NW;        // keys of a stage per warp
  constexpr int KPI = 32 / NC;       // keys per warp pass: NC lanes per key, one 16-byte chunk each
  constexpr int NIT = KPW / KPI;     // passes over the warp's keys
  constexpr int DPL = HD / 32;       // V dims per lane in the P.V pass
  static_assert(NC == 8 || NC == 16, "one key row is 8 or 16 chunks of 16 bytes");
  extern __shared__ __align__(128) uint8_t kv_smem[];  // [2][K|V][C][ROWB]
  __shared__ __align__(16) float qs[kMaxG][HD];
  __shared__ __align__(16) uint8_t newrow[2][ROWB];  // new K, V row in the cache type
  __shared__ float wpart[NW][GM][HD + 2];            // per-warp [m, l, acc[HD]]
  __shared__ __align__(8) uint64_t bars[2];
  ATT_TRACE(0);

  const int kh = blockIdx.x, b = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nq = a.nq, nkv = a.nkv, G = nq / nkv;
  const int pos = a.pos[b];
  const bool bad = pos < 0 || pos >= a.cap;
  const int n = bad ? 0 : pos + 1;
  const int nst = (n + C - 1) / C;
  const size_t row0 = ((size_t)b * nkv + kh) * a.cap;
  auto tile = [&](int buf, int kv) { return kv_smem + ((size_t)(buf * 2 + kv) * C) * ROWB; };
  auto bar_a = [&](int i) { return static_cast<uint32_t>(__cvta_generic_to_shared(&bars[i])); };
  // rows of stage st already in the cache (the new row at `pos` is not)
  auto cached = [&](int st) { return max(0, min(st * C + C, pos) - st * C); };
  auto issue = [&](int st) {  // thread 0
    const int rows = cached(st);
    if (rows <= 0) return;
    const int buf = st & 1;
    const uint32_t bytes = (uint32_t)rows * ROWB;
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar_a(buf)), "r"(2 * bytes)
                 : "memory");
#pragma unroll
    for (int kv = 0; kv < 2; kv++) {
      const uint8_t* src = reinterpret_cast<const uint8_t*>(kv ? a.vcache : a.kcache) + (row0 + (size_t)st * C) * ROWB;
      asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                       static_cast<uint32_t>(__cvta_generic_to_shared(tile(buf, kv)))),
                   "l"(src), "r"(bytes), "r"(bar_a(buf))
                   : "memory");
    }
  };
  if (tid == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar_a(0)));
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar_a(1)));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (tid == 0 && !bad) {  // cached rows were written frames ago
    issue(0);
    if (nst > 1) issue(1);
  }
  ATT_TRACE(1);
  grid_dep_enter();
  ATT_TRACE(2);
  if (bad && kh == 0 && tid == 0 && a.err) atomicExch(a.err, 1);

  // ---- queries and the new key/value row: one warp per job
  const int width = (nq + 2 * nkv) * HD;
  const float* src_row = a.qkv + (size_t)b * width;
  const int jobs = bad ? 0 : G + 2;
  for (int job = warp; job < jobs; job += NW) {
    const bool is_q = job < G, is_v = job == G + 1;
    const int head = is_q ? kh * G + job : (is_v ? nq + nkv + kh : nq + kh);
    const float* src = src_row + head * HD;
    float v[PER];
#pragma unroll
    for (int j = 0; j < PER; j++) v[j] = src[lane + 32 * j];
    if (!is_v) {
      const float* gn = is_q ? a.qn : a.kn;
      if (gn) {
        float ss = 0.0f;
#pragma unroll
        for (int j = 0; j < PER; j++) ss = fmaf(v[j], v[j], ss);
        ss = warp_sum(ss);
        const float inv = 1.0f / sqrtf(ss / (float)HD + a.eps);
#pragma unroll
        for (int j = 0; j < PER; j++) v[j] = v[j] * inv * gn[lane + 32 * j];
      }
#pragma unroll
      for (int j = 0; j < PER / 2; j++) {
        const int i = lane + 32 * j;
        float sn, cs;
        sincosf((float)pos * a.inv_freq[i], &sn, &cs);
        const float x1 = v[j], x2 = v[j + PER / 2];
        v[j] = x1 * cs - x2 * sn;
        v[j + PER / 2] = x1 * sn + x2 * cs;
      }
    }
    if (is_q) {
#pragma unroll
      for (int j = 0; j < PER; j++) qs[job][lane + 32 * j] = v[j];
    } else {
      void* cache = is_v ? a.vcache : a.kcache;
      uint8_t* nr = newrow[is_v ? 1 : 0];
#pragma unroll
      for (int j = 0; j < PER; j++) {
        const int d = lane + 32 * j;
        if constexpr (BF) {
          const uint16_t hb = f2bf(v[j]);
          reinterpret_cast<uint16_t*>(cache)[(row0 + pos) * HD + d] = hb;
          reinterpret_cast<uint16_t*>(nr)[d] = hb;
        } else {
          reinterpret_cast<float*>(cache)[(row0 + pos) * HD + d] = v[j];
          reinterpret_cast<float*>(nr)[d] = v[j];
        }
      }
    }
  }
  __syncthreads();  // queries and the new row are set
  ATT_TRACE(3);
  const float scale = 1.0f / sqrtf((float)HD);
  // Lane = (key of the pass, 16-byte chunk ch): the lane keeps its chunk of
  // every query head in registers, so a key row is read once, conflict-free
  // (the NC lanes of a key cover its contiguous row), and the chunk partial
  // dot products meet by xor-shuffles inside each key's lane group.
  const int ch = lane % NC, ksub = lane / NC;
  float qr[GM][VPC];
#pragma unroll
  for (int g = 0; g < GM; g++)
#pragma unroll
    for (int e = 0; e < VPC; e++) qr[g][e] = g < G ? qs[g][ch * VPC + e] : 0.0f;
  // Every warp runs its own online softmax over its 16 keys of each stage
  // (no block-wide reduction per stage); the 8 warp states merge at the end
  // in warp order (deterministic).
  float m_w[GM], l_w[GM], acc[GM][DPL];
#pragma unroll
  for (int g = 0; g < GM; g++) {
    m_w[g] = -INFINITY;
    l_w[g] = 0.0f;
#pragma unroll
    for (int e = 0; e < DPL; e++) acc[g][e] = 0.0f;
  }
  bool ok = true;
  for (int st = 0; st < nst; st++) {
    const int buf = st & 1;
    const int rows = min(C, n - st * C);
    if (cached(st) > 0) {
      bool done = false;
      for (uint32_t it = 0; it < (1u << 24) && !done; ++it) {
        uint32_t d;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(d)
            : "r"(bar_a(buf)), "r"((uint32_t)((st >> 1) & 1))
            : "memory");
        done = d != 0;
      }
      if (!done) ok = false;
    }
    uint8_t* Ks = tile(buf, 0);
    uint8_t* Vs = tile(buf, 1);
    if (pos >= st * C && pos < st * C + C && tid < 2 * NC) {  // the new row into its stage
      const int kv = tid / NC, cch = tid % NC;
      reinterpret_cast<uint4*>((kv ? Vs : Ks) + (size_t)(pos - st * C) * ROWB)[cch] =
          reinterpret_cast<const uint4*>(newrow[kv])[cch];
    }
    __syncthreads();
    // scores of the warp's keys kbase + it*KPI + ksub
    const int kbase = warp * KPW;
    float sc[NIT][GM];
#pragma unroll
    for (int it = 0; it < NIT; it++) {
      const int key = kbase + it * KPI + ksub;
      const bool valid = key < rows;
      float kv[VPC];
      if (valid) {
        const uint4 t = reinterpret_cast<const uint4*>(Ks + (size_t)key * ROWB)[ch];
        if constexpr (BF) {
          kv[0] = bf_lo(t.x); kv[1] = bf_hi(t.x); kv[2] = bf_lo(t.y); kv[3] = bf_hi(t.y);
          kv[4] = bf_lo(t.z); kv[5] = bf_hi(t.z); kv[6] = bf_lo(t.w); kv[7] = bf_hi(t.w);
        } else {
          kv[0] = __uint_as_float(t.x); kv[1] = __uint_as_float(t.y);
          kv[2] = __uint_as_float(t.z); kv[3] = __uint_as_float(t.w);
        }
      } else {
#pragma unroll
        for (int e = 0; e < VPC; e++) kv[e] = 0.0f;
      }
#pragma unroll
      for (int g = 0; g < GM; g++) {
        float d = 0.0f;
#pragma unroll
        for (int e = 0; e < VPC; e++) d = fmaf(qr[g][e], kv[e], d);
#pragma unroll
        for (int o = 1; o < NC; o <<= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
        sc[it][g] = valid ? d * scale : -INFINITY;
      }
    }
    // online softmax update per head over the warp's keys
    float pr[NIT][GM];
#pragma unroll
    for (int g = 0; g < GM; g++) {
      float mx = sc[0][g];
#pragma unroll
      for (int it = 1; it < NIT; it++) mx = fmaxf(mx, sc[it][g]);
#pragma unroll
      for (int o = NC; o < 32; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float mn = fmaxf(m_w[g], mx);
      const float f = m_w[g] == -INFINITY ? 0.0f : expf(m_w[g] - mn);
      float sum = 0.0f;
#pragma unroll
      for (int it = 0; it < NIT; it++) {
        pr[it][g] = sc[it][g] == -INFINITY ? 0.0f : expf(sc[it][g] - mn);
        sum += pr[it][g];
      }
#pragma unroll
      for (int o = NC; o < 32; o <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      l_w[g] = l_w[g] * f + sum;
#pragma unroll
      for (int e = 0; e < DPL; e++) acc[g][e] *= f;
      m_w[g] = mn;
    }
    // P.V over the warp's keys: lane owns dims [lane*DPL, +DPL)
    const int nk = min(KPW, rows - kbase);
#pragma unroll
    for (int kk = 0; kk < KPW; kk++) {
      if (kk >= nk) break;
      const uint8_t* vrow = Vs + (size_t)(kbase + kk) * ROWB;
      float v[DPL];
      if constexpr (BF) {
        if constexpr (DPL == 2) {
          const uint32_t t = reinterpret_cast<const uint32_t*>(vrow)[lane];
          v[0] = bf_lo(t);
          v[1] = bf_hi(t);
        } else {
          const uint2 t = reinterpret_cast<const uint2*>(vrow)[lane];
          v[0] = bf_lo(t.x); v[1] = bf_hi(t.x); v[2] = bf_lo(t.y); v[3] = bf_hi(t.y);
        }
      } else {
        if constexpr (DPL == 2) {
          const float2 t = reinterpret_cast<const float2*>(vrow)[lane];
          v[0] = t.x;
          v[1] = t.y;
        } else {
          const float4 t = reinterpret_cast<const float4*>(vrow)[lane];
          v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
        }
      }
#pragma unroll
      for (int g = 0; g < GM; g++) {
        const float pk = __shfl_sync(0xffffffffu, pr[kk / KPI][g], (kk % KPI) * NC);
#pragma unroll
        for (int e = 0; e < DPL; e++) acc[g][e] = fmaf(pk, v[e], acc[g][e]);
      }
    }
    __syncthreads();  // stage buffer consumed by every warp
    if (tid == 0 && st + 2 < nst) issue(st + 2);
    ATT_TRACE(4 + min(st, 3));
  }
  if (!ok && a.err && tid == 0) atomicExch(a.err, 3);
  ATT_TRACE(8);
  if (bad) return;
  // merge the warp states in warp order
#pragma unroll
  for (int g = 0; g < GM; g++) {
    if (g >= G) break;
    if (lane == 0) {
      wpart[warp][g][0] = m_w[g];
      wpart[warp][g][1] = l_w[g];
    }
#pragma unroll
    for (int e = 0; e < DPL; e++) wpart[warp][g][2 + lane * DPL + e] = acc[g][e];
  }
  __syncthreads();
  for (int i = tid; i < G * HD; i += NT) {
    const int g = i / HD, d = i % HD, h = kh * G + g;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < NW; w++) M = fmaxf(M, wpart[w][g][0]);
    float L = 0.0f, o = 0.0f;
#pragma unroll
    for (int w = 0; w < NW; w++) {
      const float mw = wpart[w][g][0];
      const float f = mw == -INFINITY ? 0.0f : expf(mw - M);
      L = fmaf(wpart[w][g][1], f, L);
      o = fmaf(wpart[w][g][2 + d], f, o);
    }
    o = o / L;
    const size_t oi = (size_t)b * nq * HD + (size_t)h * HD + d;
    if (a.out_b)
      a.out_b[oi] = f2bf(o);
    else
      a.out[oi] = o;
  }
  ATT_TRACE(9);
}

// Batched decode step split over the keys: grid (nkv, batch, S), clusters
// of the S splits of one (KV head, utterance).  Split s walks keys
// [s*per, min(n, (s+1)*per)) (per = ceil(n / S)) in 64-key stages through a
// two-stage ring of bulk copies issued before the wait on the previous
// kernel (the cached rows were written by earlier frames); every split
// rotates the G queries, the split holding the new position also norms,
// rotates and appends the new key/value row.  Each warp keeps an online
// softmax over its 16 keys of every stage; the warp states merge in warp
// order into the CTA's state (max, sum, unnormalised output), and after a
// cluster barrier CTA s finishes output elements [s*ceil(G*HD/S), ...) from
// the S states read over distributed shared memory in split order
// (deterministic).  Every CTA passes both cluster barriers, also with an
// out-of-range position (which only raises the error flag).
template <bool BF, int HD, int GM>
__global__ void __launch_bounds__(128) attn_split_kernel(const AttnArgs a) {
  constexpr int ES = BF ? 2 : 4;
  constexpr int ROWB = HD * ES;
  constexpr int NC = ROWB / 16;
  constexpr int VPC = 16 / ES;
  constexpr int PER = HD / 32;
  constexpr int C = 64;              // keys per stage
  constexpr int NT = 128;
  constexpr int NW = NT / 32;
  constexpr int KPW = C / NW;        // keys of a stage per warp
  constexpr int KPI = 32 / NC;       // keys per warp pass: NC lanes per key, one 16-byte chunk each
  constexpr int NIT = KPW / KPI;     // passes over the warp's keys
  constexpr int DPL = HD / 32;       // V dims per lane in the P.V pass
  static_assert(NC == 8 || NC == 16, "one key row is 8 or 16 chunks of 16 bytes");
  extern __shared__ __align__(128) uint8_t kv_smem[];  // [2][K|V][C][ROWB]
  __shared__ __align__(16) float qs[GM][HD];
  __shared__ __align__(16) uint8_t newrow[2][ROWB];  // new K, V row in the cache type
  __shared__ float wpart[NW][GM][HD + 2];            // per-warp [m, l, acc[HD]]
  __shared__ __align__(16) float cst[GM][HD + 2];    // this split's [m, l, o[HD]] (read by the cluster)
  __shared__ __align__(8) uint64_t bars[2];

  const int kh = blockIdx.x, b = blockIdx.y, split = blockIdx.z, S = gridDim.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nq = a.nq, nkv = a.nkv, G = nq / nkv;
  const int pos = a.pos[b];
  const bool bad = pos < 0 || pos >= a.cap;
  const int n = bad ? 0 : pos + 1;
  const int per = (n + S - 1) / S;
  const int k0 = min(n, split * per), k1 = min(n, k0 + per);
  const int nst = (k1 - k0 + C - 1) / C;
  const bool owns_new = !bad && pos >= k0 && pos < k1;
  const size_t row0 = ((size_t)b * nkv + kh) * a.cap;
  auto tile = [&](int buf, int kv) { return kv_smem + ((size_t)(buf * 2 + kv) * C) * ROWB; };
  auto bar_a = [&](int i) { return static_cast<uint32_t>(__cvta_generic_to_shared(&bars[i])); };
  // rows of stage st already in the cache (the new row at `pos` is not)
  auto cached = [&](int st) { return max(0, min(min(k0 + st * C + C, k1), pos) - (k0 + st * C)); };
  auto issue = [&](int st) {  // thread 0
    const int rows = cached(st);
    if (rows <= 0) return;
    const int buf = st & 1;
    const uint32_t bytes = (uint32_t)rows * ROWB;
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar_a(buf)), "r"(2 * bytes)
                 : "memory");
#pragma unroll
    for (int kv = 0; kv < 2; kv++) {
      const uint8_t* src =
          reinterpret_cast<const uint8_t*>(kv ? a.vcache : a.kcache) + (row0 + (size_t)k0 + (size_t)st * C) * ROWB;
      asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                       static_cast<uint32_t>(__cvta_generic_to_shared(tile(buf, kv)))),
                   "l"(src), "r"(bytes), "r"(bar_a(buf))
                   : "memory");
    }
  };
  if (tid == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar_a(0)));
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar_a(1)));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (tid == 0 && !bad) {  // cached rows were written frames ago
    issue(0);
    if (nst > 1) issue(1);
  }
  grid_dep_enter();
  if (bad && kh == 0 && split == 0 && tid == 0 && a.err) atomicExch(a.err, 1);

  // ---- queries (every split) and the new key/value row (its owner): one
  // warp per job
  const int width = (nq + 2 * nkv) * HD;
  const float* src_row = a.qkv + (size_t)b * width;
  const int jobs = bad ? 0 : (owns_new ? G + 2 : G);
  for (int job = warp; job < jobs; job += NW) {
    const bool is_q = job < G, is_v = job == G + 1;
    const int head = is_q ? kh * G + job : (is_v ? nq + nkv + kh : nq + kh);
    const float* src = src_row + head * HD;
    float v[PER];
#pragma unroll
    for (int j = 0; j < PER; j++) v[j] = src[lane + 32 * j];
    if (!is_v) {
      const float* gn = is_q ? a.qn : a.kn;
      if (gn) {
        float ss = 0.0f;
#pragma unroll
        for (int j = 0; j < PER; j++) ss = fmaf(v[j], v[j], ss);
        ss = warp_sum(ss);
        const float inv = 1.0f / sqrtf(ss / (float)HD + a.eps);
#pragma unroll
        for (int j = 0; j < PER; j++) v[j] = v[j] * inv * gn[lane + 32 * j];
      }
#pragma unroll
      for (int j = 0; j < PER / 2; j++) {
        const int i = lane + 32 * j;
        float sn, cs;
        sincosf((float)pos * a.inv_freq[i], &sn, &cs);
        const float x1 = v[j], x2 = v[j + PER / 2];
        v[j] = x1 * cs - x2 * sn;
        v[j + PER / 2] = x1 * sn + x2 * cs;
      }
    }
    if (is_q) {
#pragma unroll
      for (int j = 0; j < PER; j++) qs[job][lane + 32 * j] = v[j];
    } else {
      void* cache = is_v ? a.vcache : a.kcache;
      uint8_t* nr = newrow[is_v ? 1 : 0];
#pragma unroll
      for (int j = 0; j < PER; j++) {
        const int d = lane + 32 * j;
        if constexpr (BF) {
          const uint16_t hb = f2bf(v[j]);
          reinterpret_cast<uint16_t*>(cache)[(row0 + pos) * HD + d] = hb;
          reinterpret_cast<uint16_t*>(nr)[d] = hb;
        } else {
          reinterpret_cast<float*>(cache)[(row0 + pos) * HD + d] = v[j];
          reinterpret_cast<float*>(nr)[d] = v[j];
        }
      }
    }
  }
  __syncthreads();  // queries and the new row are set
  const float scale = 1.0f / sqrtf((float)HD);
  // Lane = (key of the pass, 16-byte chunk ch): the lane keeps its chunk of
  // every query head in registers, so a key row is read once, conflict-free,
  // and the chunk partial dot products meet by xor-shuffles inside each
  // key's lane group.
  const int ch = lane % NC, ksub = lane / NC;
  float qr[GM][VPC];
#pragma unroll
  for (int g = 0; g < GM; g++)
#pragma unroll
    for (int e = 0; e < VPC; e++) qr[g][e] = g < G ? qs[g][ch * VPC + e] : 0.0f;
  float m_w[GM], l_w[GM], acc[GM][DPL];
#pragma unroll
  for (int g = 0; g < GM; g++) {
    m_w[g] = -INFINITY;
    l_w[g] = 0.0f;
#pragma unroll
    for (int e = 0; e < DPL; e++) acc[g][e] = 0.0f;
  }
  bool ok = true;
  for (int st = 0; st < nst; st++) {
    const int buf = st & 1;
    const int kst = k0 + st * C;  // first key of the stage
    const int rows = min(C, k1 - kst);
    if (cached(st) > 0) {
      bool done = false;
      for (uint32_t it = 0; it < kWaitLimit && !done; ++it) {
        uint32_t d;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(d)
            : "r"(bar_a(buf)), "r"((uint32_t)((st >> 1) & 1))
            : "memory");
        done = d != 0;
      }
      if (!done) ok = false;
    }
    uint8_t* Ks = tile(buf, 0);
    uint8_t* Vs = tile(buf, 1);
    if (owns_new && pos >= kst && pos < kst + C && tid < 2 * NC) {  // the new row into its stage
      const int kv = tid / NC, cch = tid % NC;
      reinterpret_cast<uint4*>((kv ? Vs : Ks) + (size_t)(pos - kst) * ROWB)[cch] =
          reinterpret_cast<const uint4*>(newrow[kv])[cch];
    }
    __syncthreads();
    const int kbase = warp * KPW;
    float sc[NIT][GM];
#pragma unroll
    for (int it = 0; it < NIT; it++) {
      const int key = kbase + it * KPI + ksub;
      const bool valid = key < rows;
      float kv[VPC];
      if (valid) {
        const uint4 t = reinterpret_cast<const uint4*>(Ks + (size_t)key * ROWB)[ch];
        if constexpr (BF) {
          kv[0] = bf_lo(t.x); kv[1] = bf_hi(t.x); kv[2] = bf_lo(t.y); kv[3] = bf_hi(t.y);
          kv[4] = bf_lo(t.z); kv[5] = bf_hi(t.z); kv[6] = bf_lo(t.w); kv[7] = bf_hi(t.w);
        } else {
          kv[0] = __uint_as_float(t.x); kv[1] = __uint_as_float(t.y);
          kv[2] = __uint_as_float(t.z); kv[3] = __uint_as_float(t.w);
        }
      } else {
#pragma unroll
        for (int e = 0; e < VPC; e++) kv[e] = 0.0f;
      }
#pragma unroll
      for (int g = 0; g < GM; g++) {
        float d = 0.0f;
#pragma unroll
        for (int e = 0; e < VPC; e++) d = fmaf(qr[g][e], kv[e], d);
#pragma unroll
        for (int o = 1; o < NC; o <<= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
        sc[it][g] = valid ? d * scale : -INFINITY;
      }
    }
    float pr[NIT][GM];
#pragma unroll
    for (int g = 0; g < GM; g++) {
      float mx = sc[0][g];
#pragma unroll
      for (int it = 1; it < NIT; it++) mx = fmaxf(mx, sc[it][g]);
#pragma unroll
      for (int o = NC; o < 32; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float mn = fmaxf(m_w[g], mx);
      const float f = m_w[g] == -INFINITY ? 0.0f : expf(m_w[g] - mn);
      float sum = 0.0f;
#pragma unroll
      for (int it = 0; it < NIT; it++) {
        pr[it][g] = sc[it][g] == -INFINITY ? 0.0f : expf(sc[it][g] - mn);
        sum += pr[it][g];
      }
#pragma unroll
      for (int o = NC; o < 32; o <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      l_w[g] = l_w[g] * f + sum;
#pragma unroll
      for (int e = 0; e < DPL; e++) acc[g][e] *= f;
      m_w[g] = mn;
    }
    const int nk = min(KPW, rows - kbase);
#pragma unroll
    for (int kk = 0; kk < KPW; kk++) {
      if (kk >= nk) break;
      const uint8_t* vrow = Vs + (size_t)(kbase + kk) * ROWB;
      float v[DPL];
      if constexpr (BF) {
        if constexpr (DPL == 2) {
          const uint32_t t = reinterpret_cast<const uint32_t*>(vrow)[lane];
          v[0] = bf_lo(t);
          v[1] = bf_hi(t);
        } else {
          const uint2 t = reinterpret_cast<const uint2*>(vrow)[lane];
          v[0] = bf_lo(t.x); v[1] = bf_hi(t.x); v[2] = bf_lo(t.y); v[3] = bf_hi(t.y);
        }
      } else {
        if constexpr (DPL == 2) {
          const float2 t = reinterpret_cast<const float2*>(vrow)[lane];
          v[0] = t.x;
          v[1] = t.y;
        } else {
          const float4 t = reinterpret_cast<const float4*>(vrow)[lane];
          v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
        }
      }
#pragma unroll
      for (int g = 0; g < GM; g++) {
        const float pk = __shfl_sync(0xffffffffu, pr[kk / KPI][g], (kk % KPI) * NC);
#pragma unroll
        for (int e = 0; e < DPL; e++) acc[g][e] = fmaf(pk, v[e], acc[g][e]);
      }
    }
    __syncthreads();  // stage buffer consumed by every warp
    if (tid == 0 && st + 2 < nst) issue(st + 2);
  }
  if (!ok && a.err && tid == 0) atomicExch(a.err, 3);
  // ---- this split's state: the warp states merged in warp order
#pragma unroll
  for (int g = 0; g < GM; g++) {
    if (g >= G) break;
    if (lane == 0) {
      wpart[warp][g][0] = m_w[g];
      wpart[warp][g][1] = l_w[g];
    }
#pragma unroll
    for (int e = 0; e < DPL; e++) wpart[warp][g][2 + lane * DPL + e] = acc[g][e];
  }
  __syncthreads();
  for (int i = tid; i < G * (HD + 1); i += NT) {
    const int g = i / (HD + 1), d = i % (HD + 1);  // d == HD: the row's max and sum
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < NW; w++) M = fmaxf(M, wpart[w][g][0]);
    float acc_o = 0.0f;
#pragma unroll
    for (int w = 0; w < NW; w++) {
      const float mw = wpart[w][g][0];
      const float f = mw == -INFINITY ? 0.0f : expf(mw - M);
      acc_o = fmaf(d == HD ? wpart[w][g][1] : wpart[w][g][2 + d], f, acc_o);
    }
    if (d == HD) {
      cst[g][0] = M;
      cst[g][1] = acc_o;
    } else {
      cst[g][2 + d] = acc_o;
    }
  }
  // every split's state is written
  cluster_sync();
  if (!bad) {
    const int tot = G * HD, share = (tot + S - 1) / S;
    const uint32_t base = static_cast<uint32_t>(__cvta_generic_to_shared(&cst[0][0]));
    for (int i = split * share + tid; i < min(tot, split * share + share); i += NT) {
      const int g = i / HD, d = i % HD, h = kh * G + g;
      const uint32_t row = base + (uint32_t)(g * (HD + 2)) * 4u;
      float M = -INFINITY;
      for (int r = 0; r < S; r++) M = fmaxf(M, __uint_as_float(ld_dsmem_u32(mapa_shared(row, (uint32_t)r))));
      float L = 0.0f, o = 0.0f;
      for (int r = 0; r < S; r++) {
        const uint32_t rr = mapa_shared(row, (uint32_t)r);
        const float mr = __uint_as_float(ld_dsmem_u32(rr));
        const float f = mr == -INFINITY ? 0.0f : expf(mr - M);
        L = fmaf(__uint_as_float(ld_dsmem_u32(rr + 4u)), f, L);
        o = fmaf(__uint_as_float(ld_dsmem_u32(rr + (uint32_t)(2 + d) * 4u)), f, o);
      }
      o = o / L;
      const size_t oi = (size_t)b * nq * HD + (size_t)h * HD + d;
      if (a.out_b)
        a.out_b[oi] = f2bf(o);
      else
        a.out[oi] = o;
    }
  }
  // no CTA leaves while a peer may still read its state
  cluster_sync();
}

// ---- tensor-core form of the split decode step (bf16 cache)
//
// Same split, cluster merge and new-row handling as attn_split_kernel; the
// two products run on mma.sync.m16n8k16 (bf16 in, fp32 accumulate): scores
// S[q][key] = Q . K^T with the G query heads as the rows of the A operand
// (rows G..15 zero) and 8-key column tiles read by ldmatrix from the K
// stage, then O += P . V with P as the A operand and V read transposed.
// Q enters as a bf16 pair hi + lo (hi = bf16(x), lo = bf16(x - hi)), so the
// scores keep about 16 significant bits (the exponential amplifies their
// error); P, in [0, 1], enters in bf16 with the products accumulated in
// fp32.  Stages of 64 keys arrive by TMA tensor
// copies with the 128-byte swizzle ([box of 64 dims][64 keys][128 B]; the
// ldmatrix rows of a warp fall in distinct banks), kAttnRing stages in
// flight per CTA.  Each warp owns 16
// keys of a stage and an online softmax over its keys; the merges follow
// attn_split_kernel.
constexpr int kAttnRing = 3;  // attn_mma_kernel: 64-key stages in flight per CTA

CTTS_DEV uint32_t pack_bf2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
// x = hi + lo with both parts in bf16 (hi rounded to nearest), packed pairs
CTTS_DEV void split_bf2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  hi = pack_bf2(x0, x1);
  lo = pack_bf2(x0 - bf_lo(hi), x1 - bf_hi(hi));
}
// (register operands only: not volatile, so independent MMAs interleave)
CTTS_DEV void mma_bf16_16816(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
CTTS_DEV void ldsm_x4(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
CTTS_DEV void ldsm_x4_t(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

template <int HD>
__global__ void __launch_bounds__(128) attn_mma_kernel(const __grid_constant__ CUtensorMap tmK,
                                                       const __grid_constant__ CUtensorMap tmV, const AttnArgs a) {
  constexpr int ROWB = HD * 2;
  constexpr int NB = HD / 64;          // 128-byte boxes per key row
  constexpr int C = 64;                // keys per stage
  constexpr int NT = 128, NW = NT / 32;
  constexpr int KS = HD / 16;          // k-steps of the score product
  constexpr int NO = HD / 8;           // 8-dim column tiles of the output
  constexpr uint32_t kBox = C * 128;   // one box: 64 keys x 128 bytes
  constexpr uint32_t kTile = NB * kBox;  // one K or V stage
  constexpr int RW = 8;                // query rows held (G <= 8)
  constexpr int NS = kAttnRing;        // stages in flight
  extern __shared__ __align__(1024) uint8_t dyn_smem[];  // [NS][K|V][NB][C][128] swizzled
  __shared__ __align__(16) float qs[RW][HD];
  __shared__ __align__(16) uint8_t newrow[2][ROWB];
  __shared__ __align__(16) float cst[RW][HD + 2];
  __shared__ __align__(8) uint64_t bars[NS];
  ATT_TRACE(0);
  uint8_t* kv_smem = dyn_smem + ((1024u - (static_cast<uint32_t>(__cvta_generic_to_shared(dyn_smem)) & 1023u)) & 1023u);
  const uint32_t kv_base = static_cast<uint32_t>(__cvta_generic_to_shared(kv_smem));

  const int kh = blockIdx.x, b = blockIdx.y, split = blockIdx.z, S = gridDim.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nq = a.nq, nkv = a.nkv, G = nq / nkv;
  const int pos = a.pos[b];
  const bool bad = pos < 0 || pos >= a.cap;
  const int n = bad ? 0 : pos + 1;
  const int per = (n + S - 1) / S;
  const int k0 = min(n, split * per), k1 = min(n, k0 + per);
  const int nst = (k1 - k0 + C - 1) / C;
  const bool owns_new = !bad && pos >= k0 && pos < k1;
  const size_t row0 = ((size_t)b * nkv + kh) * a.cap;
  auto tile = [&](int buf, int kv) { return kv_base + (uint32_t)(buf * 2 + kv) * kTile; };
  auto bar_a = [&](int i) { return static_cast<uint32_t>(__cvta_generic_to_shared(&bars[i])); };
  // byte offset of (key, 16-byte chunk) in a stage tile: 128-byte swizzle
  auto sw = [](int key, int chunk) {
    return (uint32_t)(chunk >> 3) * kBox + (uint32_t)key * 128u + (uint32_t)(((chunk & 7) ^ (key & 7)) << 4);
  };
  auto issue = [&](int st) {  // thread 0: the stage's K and V boxes (rows past the cache read as stale or zero)
    const int buf = st % NS;
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar_a(buf)), "r"(2u * kTile)
                 : "memory");
    const int y = (int)(row0 + (size_t)k0 + (size_t)st * C);
#pragma unroll
    for (int kv = 0; kv < 2; kv++)
#pragma unroll
      for (int bx = 0; bx < NB; bx++)
        asm volatile(
            "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
            "[%4];" ::"r"(tile(buf, kv) + (uint32_t)bx * kBox),
            "l"(reinterpret_cast<uint64_t>(kv ? &tmV : &tmK)), "r"(bx * 64), "r"(y), "r"(bar_a(buf))
            : "memory");
  };
  if (tid == 0) {
    for (int i = 0; i < NS; i++) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar_a(i)));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  for (int i = tid; i < RW * HD; i += NT) qs[i / HD][i % HD] = 0.0f;
  __syncthreads();
  if (tid == 0 && !bad)  // cached rows were written frames ago
    for (int st = 0; st < min(nst, NS); st++) issue(st);
  // what the prologue needs besides the new q/k/v rows depends on weights
  // and the position only: the RoPE angles of this position and the
  // QK-Norm gains of this lane's dims, ready before the wait
  constexpr int PH = HD / 16;
  const int hl = lane & 15;
  float rcs[PH / 2], rsn[PH / 2], gnq[PH], gnk[PH];
#pragma unroll
  for (int j = 0; j < PH / 2; j++) sincosf((float)(bad ? 0 : pos) * a.inv_freq[hl + 16 * j], &rsn[j], &rcs[j]);
#pragma unroll
  for (int j = 0; j < PH; j++) {
    gnq[j] = a.qn ? a.qn[hl + 16 * j] : 1.0f;
    gnk[j] = a.kn ? a.kn[hl + 16 * j] : 1.0f;
  }
  ATT_TRACE(1);
  grid_dep_enter();
  ATT_TRACE(2);
  if (bad && kh == 0 && split == 0 && tid == 0 && a.err) atomicExch(a.err, 1);

  // ---- queries (every split) and the new key/value row (its owner): one
  // job per half-warp (lanes 16h..16h+15 of warp w take job 2w + h), a lane
  // holding dims l, l + 16, ...; the RoPE pairs (d, d + HD/2) stay in the
  // lane and every lane takes part in the half-warp norm reduction
  const int width = (nq + 2 * nkv) * HD;
  const float* src_row = a.qkv + (size_t)b * width;
  const int jobs = bad ? 0 : (owns_new ? G + 2 : G);
  for (int j0 = 2 * warp; j0 < jobs; j0 += 2 * NW) {
    const int job = j0 + (lane >> 4);
    const bool act = job < jobs;
    const bool is_q = job < G, is_v = job == G + 1;
    const int head = is_q ? kh * G + job : (is_v ? nq + nkv + kh : nq + kh);
    const float* src = src_row + head * HD;
    float v[PH];
#pragma unroll
    for (int j = 0; j < PH; j++) v[j] = act ? src[hl + 16 * j] : 0.0f;
    float ss = 0.0f;
#pragma unroll
    for (int j = 0; j < PH; j++) ss = fmaf(v[j], v[j], ss);
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (act && !is_v) {
      if (is_q ? a.qn != nullptr : a.kn != nullptr) {
        const float inv = 1.0f / sqrtf(ss / (float)HD + a.eps);
#pragma unroll
        for (int j = 0; j < PH; j++) v[j] = v[j] * inv * (is_q ? gnq[j] : gnk[j]);
      }
#pragma unroll
      for (int j = 0; j < PH / 2; j++) {
        const float x1 = v[j], x2 = v[j + PH / 2];
        v[j] = x1 * rcs[j] - x2 * rsn[j];
        v[j + PH / 2] = x1 * rsn[j] + x2 * rcs[j];
      }
    }
    if (act && is_q) {
#pragma unroll
      for (int j = 0; j < PH; j++) qs[job][hl + 16 * j] = v[j];
    } else if (act) {
      void* cache = is_v ? a.vcache : a.kcache;
      uint16_t* nr = reinterpret_cast<uint16_t*>(newrow[is_v ? 1 : 0]);
#pragma unroll
      for (int j = 0; j < PH; j++) {
        const int d = hl + 16 * j;
        const uint16_t hb = f2bf(v[j]);
        reinterpret_cast<uint16_t*>(cache)[(row0 + pos) * HD + d] = hb;
        nr[d] = hb;
      }
    }
  }
  __syncthreads();  // queries and the new row are set
  ATT_TRACE(3);

  // A fragments of Q (rows 0..7 = query heads, rows 8..15 zero), hi and lo
  const int gq = lane >> 2, tq = lane & 3;
  uint32_t qa_hi[KS][2], qa_lo[KS][2];
#pragma unroll
  for (int ks = 0; ks < KS; ks++) {
    const float* qrow = qs[gq] + ks * 16 + 2 * tq;
    split_bf2(qrow[0], qrow[1], qa_hi[ks][0], qa_lo[ks][0]);
    split_bf2(qrow[8], qrow[9], qa_hi[ks][1], qa_lo[ks][1]);
  }
  const float scale = 1.0f / sqrtf((float)HD);
  float m_w = -INFINITY, l_w = 0.0f;  // row gq of this warp's keys
  float o[NO][4];
#pragma unroll
  for (int t = 0; t < NO; t++) o[t][0] = o[t][1] = o[t][2] = o[t][3] = 0.0f;
  const int kbase = warp * 16;
  bool ok = true;
  for (int st = 0; st < nst; st++) {
    const int buf = st % NS;
    const int kst = k0 + st * C;
    const int rows = min(C, k1 - kst);
    {
      bool done = false;
      for (uint32_t it = 0; it < kWaitLimit && !done; ++it) {
        uint32_t d;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(d)
            : "r"(bar_a(buf)), "r"((uint32_t)((st / NS) & 1))
            : "memory");
        done = d != 0;
      }
      if (!done) ok = false;
    }
    ATT_TRACE(4 + 2 * min(st, 3));
    if (owns_new && pos >= kst && pos < kst + C && tid < 2 * (ROWB / 16)) {  // the new row into its stage
      const int kv = tid / (ROWB / 16), cch = tid % (ROWB / 16);
      *reinterpret_cast<uint4*>(kv_smem + (tile(buf, kv) - kv_base) + sw(pos - kst, cch)) =
          reinterpret_cast<const uint4*>(newrow[kv])[cch];
    }
    // value rows past the split's keys (stale cache rows or the next
    // split's) enter P.V with weight 0: make them finite zeros
    for (int i = tid; i < (C - rows) * (ROWB / 16); i += NT) {
      const int r = rows + i / (ROWB / 16), cch = i % (ROWB / 16);
      *reinterpret_cast<uint4*>(kv_smem + (tile(buf, 1) - kv_base) + sw(r, cch)) = make_uint4(0u, 0u, 0u, 0u);
    }
    __syncthreads();
    // scores of the warp's 16 keys: two 8-key column tiles
    // the hi and lo products accumulate separately (four independent MMA
    // chains instead of two), summed once
    float s[2][4], sl[2][4];
#pragma unroll
    for (int j = 0; j < 2; j++) {
      s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.0f;
      sl[j][0] = sl[j][1] = sl[j][2] = sl[j][3] = 0.0f;
    }
    const uint32_t kt = tile(buf, 0), vt = tile(buf, 1);
#pragma unroll
    for (int ks = 0; ks < KS; ks++) {
      // matrices: (keys 0-7, dims lo), (keys 0-7, dims hi), (keys 8-15, lo), (keys 8-15, hi)
      const int mi = lane >> 3, key = kbase + 8 * (mi >> 1) + (lane & 7);
      uint32_t kb[4];
      ldsm_x4(kt + sw(key, 2 * ks + (mi & 1)), kb);
      const uint32_t ah[4] = {qa_hi[ks][0], 0u, qa_hi[ks][1], 0u};
      const uint32_t al[4] = {qa_lo[ks][0], 0u, qa_lo[ks][1], 0u};
      mma_bf16_16816(s[0], ah, kb[0], kb[1]);
      mma_bf16_16816(sl[0], al, kb[0], kb[1]);
      mma_bf16_16816(s[1], ah, kb[2], kb[3]);
      mma_bf16_16816(sl[1], al, kb[2], kb[3]);
    }
#pragma unroll
    for (int j = 0; j < 2; j++)
#pragma unroll
      for (int e = 0; e < 4; e++) s[j][e] += sl[j][e];
    // online softmax of row gq over the warp's keys kbase + 8j + 2tq + e
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < 2; j++)
#pragma unroll
      for (int e = 0; e < 2; e++) {
        const int key = kbase + 8 * j + 2 * tq + e;
        s[j][e] = key < rows ? s[j][e] * scale : -INFINITY;
        mx = fmaxf(mx, s[j][e]);
      }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float mn = fmaxf(m_w, mx);
    const float f = m_w == -INFINITY ? 0.0f : expf(m_w - mn);
    float p[2][2], sum = 0.0f;
#pragma unroll
    for (int j = 0; j < 2; j++)
#pragma unroll
      for (int e = 0; e < 2; e++) {
        p[j][e] = s[j][e] == -INFINITY ? 0.0f : expf(s[j][e] - mn);
        sum += p[j][e];
      }
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    l_w = l_w * f + sum;
    m_w = mn;
#pragma unroll
    for (int t = 0; t < NO; t++) {
      o[t][0] *= f;
      o[t][1] *= f;
    }
    // P as the A operand in bf16 (rows 8..15 zero): probabilities in
    // [0, 1], products accumulated in fp32
    uint32_t ph[4] = {0u, 0u, 0u, 0u};
    ph[0] = pack_bf2(p[0][0], p[0][1]);
    ph[2] = pack_bf2(p[1][0], p[1][1]);
#pragma unroll
    for (int t = 0; t < NO; t += 2) {
      // matrices: (keys 0-7, dims 8t..), (keys 8-15, 8t..), (keys 0-7, 8t+8..), (keys 8-15, 8t+8..)
      const int mi = lane >> 3, key = kbase + 8 * (mi & 1) + (lane & 7);
      uint32_t vb[4];
      ldsm_x4_t(vt + sw(key, t + (mi >> 1)), vb);
      mma_bf16_16816(o[t], ph, vb[0], vb[1]);
      mma_bf16_16816(o[t + 1], ph, vb[2], vb[3]);
    }
    __syncthreads();  // stage buffer consumed by every warp
    ATT_TRACE(5 + 2 * min(st, 3));
    if (tid == 0 && st + NS < nst) issue(st + NS);
  }
  if (!ok && a.err && tid == 0) atomicExch(a.err, 3);
  // ---- this split's state: the warp states merged in warp order (the
  // per-warp states reuse the stage area: every copy into it was waited on
  // and every warp passed the last stage's barrier)
  float (*wpart)[RW][HD + 2] = reinterpret_cast<float (*)[RW][HD + 2]>(kv_smem);
  static_assert(NW * RW * (HD + 2) * 4 <= 2 * NS * kTile, "warp states fit the stage area");
  if (gq < G) {
    if (tq == 0) {
      wpart[warp][gq][0] = m_w;
      wpart[warp][gq][1] = l_w;
    }
#pragma unroll
    for (int t = 0; t < NO; t++) {
      wpart[warp][gq][2 + 8 * t + 2 * tq] = o[t][0];
      wpart[warp][gq][2 + 8 * t + 2 * tq + 1] = o[t][1];
    }
  }
  __syncthreads();
  for (int i = tid; i < G * (HD + 1); i += NT) {
    const int g = i / (HD + 1), d = i % (HD + 1);  // d == HD: the row's max and sum
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < NW; w++) M = fmaxf(M, wpart[w][g][0]);
    float acc_o = 0.0f;
#pragma unroll
    for (int w = 0; w < NW; w++) {
      const float mw = wpart[w][g][0];
      const float fw = mw == -INFINITY ? 0.0f : expf(mw - M);
      acc_o = fmaf(d == HD ? wpart[w][g][1] : wpart[w][g][2 + d], fw, acc_o);
    }
    if (d == HD) {
      cst[g][0] = M;
      cst[g][1] = acc_o;
    } else {
      cst[g][2 + d] = acc_o;
    }
  }
  // every split's state is written
  ATT_TRACE(12);
  cluster_sync();
  ATT_TRACE(13);
  if (!bad) {
    const int tot = G * HD, share = (tot + S - 1) / S;
    const uint32_t base = static_cast<uint32_t>(__cvta_generic_to_shared(&cst[0][0]));
    for (int i = split * share + tid; i < min(tot, split * share + share); i += NT) {
      const int g = i / HD, d = i % HD, h = kh * G + g;
      const uint32_t row = base + (uint32_t)(g * (HD + 2)) * 4u;
      float M = -INFINITY;
      for (int r = 0; r < S; r++) M = fmaxf(M, __uint_as_float(ld_dsmem_u32(mapa_shared(row, (uint32_t)r))));
      float L = 0.0f, ov = 0.0f;
      for (int r = 0; r < S; r++) {
        const uint32_t rr = mapa_shared(row, (uint32_t)r);
        const float mr = __uint_as_float(ld_dsmem_u32(rr));
        const float fr = mr == -INFINITY ? 0.0f : expf(mr - M);
        L = fmaf(__uint_as_float(ld_dsmem_u32(rr + 4u)), fr, L);
        ov = fmaf(__uint_as_float(ld_dsmem_u32(rr + (uint32_t)(2 + d) * 4u)), fr, ov);
      }
      ov = ov / L;
      const size_t oi = (size_t)b * nq * HD + (size_t)h * HD + d;
      if (a.out_b)
        a.out_b[oi] = f2bf(ov);
      else
        a.out[oi] = ov;
    }
  }
  ATT_TRACE(14);
  // no CTA leaves while a peer may still read its state
  cluster_sync();
  ATT_TRACE(15);
}

// causal prefill attention: grid (T, nq), 128 threads, dyn smem n floats
template <bool BF>
__global__ void __launch_bounds__(128) attn_prefill_kernel(const AttnArgs a) {
  extern __shared__ float ps[];
  grid_dep_enter();
  const int i = blockIdx.x, h = blockIdx.y;
  const int hd = a.hd, nq = a.nq, G = nq / a.nkv, kh = h / G;
  const int b = a.prefill_b;
  const int n = a.pos0 + i + 1;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  __shared__ float qs[kMaxHd];
  __shared__ float red[4];
  __shared__ float accs[128];
  const float* q = a.qrot + (size_t)i * nq * hd + h * hd;
  for (int d = tid; d < hd; d += blockDim.x) qs[d] = q[d];
  __syncthreads();
  const float scale = 1.0f / sqrtf((float)hd);
  const size_t kvbase = ((size_t)b * a.nkv + kh) * a.cap * hd;
  float mloc = -INFINITY;
  for (int j = tid; j < n; j += blockDim.x) {
    float s = 0.0f;
    for (int d = 0; d < hd; d++) s = fmaf(qs[d], ld_kv<BF>(a.kcache, kvbase + (size_t)j * hd + d), s);
    s *= scale;
    ps[j] = s;
    mloc = fmaxf(mloc, s);
  }
  mloc = warp_max(mloc);
  if (lane == 0) red[warp] = mloc;
  __syncthreads();
  const float M = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  __syncthreads();
  float lloc = 0.0f;
  for (int j = tid; j < n; j += blockDim.x) {
    float p = expf(ps[j] - M);
    ps[j] = p;
    lloc += p;
  }
  lloc = warp_sum(lloc);
  if (lane == 0) red[warp] = lloc;
  __syncthreads();
  const float L = red[0] + red[1] + red[2] + red[3];
  const int parts = blockDim.x / hd;
  const int d = tid % hd, pp = tid / hd;
  float acc = 0.0f;
  if (pp < parts)
    for (int j = pp; j < n; j += parts) acc = fmaf(ps[j], ld_kv<BF>(a.vcache, kvbase + (size_t)j * hd + d), acc);
  accs[tid] = acc;
  __syncthreads();
  if (pp == 0) {
    for (int p2 = 1; p2 < parts; p2++) acc += accs[p2 * hd + d];
    const size_t o = (size_t)i * nq * hd + h * hd + d;
    if (a.out_b)
      a.out_b[o] = f2bf(acc / L);
    else
      a.out[o] = acc / L;
  }
}

__global__ void advance_pos_kernel(int* pos, int batch) {
  grid_dep_enter();
  int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < batch) pos[b] += 1;
}

// one warp per row
__global__ void rmsnorm_rows_kernel(const float* x, int M, int K, const float* w, float eps,
                                    float* y) {
  grid_dep_enter();
  int row = blockIdx.x * 4 + (threadIdx.x >> 5);
  int lane = threadIdx.x & 31;
  if (row >= M) return;
  const float* xr = x + (size_t)row * K;
  if ((K & 127) == 0 && K <= 2048) {
    float4 v[16];
    const float ss = warp_load_row<16>(xr, K, v);
    const float inv = 1.0f / sqrtf(ss / (float)K + eps);
#pragma unroll
    for (int i = 0; i < 16; i++) {
      if (i >= (K >> 7)) break;
      const int k = lane * 4 + 128 * i;
      float4 o = make_float4(v[i].x * inv * w[k], v[i].y * inv * w[k + 1], v[i].z * inv * w[k + 2],
                             v[i].w * inv * w[k + 3]);
      *reinterpret_cast<float4*>(y + (size_t)row * K + k) = o;
    }
    return;
  }
  float ss = 0.0f;
  for (int k = lane; k < K; k += 32) ss = fmaf(xr[k], xr[k], ss);
  ss = warp_sum(ss);
  float inv = 1.0f / sqrtf(ss / (float)K + eps);
  for (int k = lane; k < K; k += 32) y[(size_t)row * K + k] = xr[k] * inv * w[k];
}

template <bool BF>
__global__ void embed_gather_kernel(const void* table, int vocab, int H, const int64_t* ids,
                                    int n, float* out, int* bad) {
  grid_dep_enter();
  int r = blockIdx.x;
  if (r >= n) return;
  int64_t id = ids[r];
  float* o = out + (size_t)r * H;
  if (id < 0 || id >= vocab) {
    for (int k = threadIdx.x; k < H; k += blockDim.x) o[k] = 0.0f;
    if (threadIdx.x == 0 && bad) atomicAdd(bad, 1);
    return;
  }
  for (int k = threadIdx.x; k < H; k += blockDim.x) o[k] = ld_kv<BF>(table, (size_t)id * H + k);
}

__global__ void rope_inplace_kernel(float* x, int M, int heads, int hd, const int* pos,
                                    const float* inv_freq) {
  grid_dep_enter();
  int m = blockIdx.x, h = blockIdx.y;
  int half = hd / 2;
  float* v = x + ((size_t)m * heads + h) * hd;
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    float ang = (float)pos[m] * inv_freq[i];
    float sn, cs;
    sincosf(ang, &sn, &cs);
    float x1 = v[i], x2 = v[i + half];
    v[i] = x1 * cs - x2 * sn;
    v[i + half] = x1 * sn + x2 * cs;
  }
}

__global__ void swiglu_kernel(const float* gu, int M, int F, float* out) {
  grid_dep_enter();
  size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (size_t)M * F) return;
  size_t m = i / F, f = i % F;
  float g = gu[m * 2 * F + f], u = gu[m * 2 * F + F + f];
  out[i] = silu(g) * u;
}

}  // namespace

cudaError_t launch_qk_rope_append(const AttnArgs& a, cudaStream_t s) {
  if (a.hd % 64 != 0 || a.hd > kMaxHd) return cudaErrorInvalidValue;
  dim3 grid(a.rows, (a.nq + 2 * a.nkv + 3) / 4);
  if (a.kv_bf16)
    CTTS_LK(launch_k(qk_rope_append_kernel<true>, dim3(grid), dim3(128), 0, s, a));
  else
    CTTS_LK(launch_k(qk_rope_append_kernel<false>, dim3(grid), dim3(128), 0, s, a));
  return cudaGetLastError();
}

template <bool BF, int HD>
cudaError_t launch_attn_step_t(const AttnArgs& a, cudaStream_t s) {
  const size_t smem = (size_t)2 * a.chunk * HD * (BF ? 2 : 4);
  // opt in whenever the dynamic size grows: the static arrays count against
  // the 48 KB default as well (fp32, head_dim 128: 32 KB + 16.5 KB)
  static SmemOptIn opt;
  if (cudaError_t e = opt.ensure((const void*)attn_step_kernel<BF, HD>, smem)) return e;
  CTTS_LK(launch_k(attn_step_kernel<BF, HD>, dim3(a.nsplit, a.nkv, a.batch), dim3(128), smem, s, a));
  return cudaGetLastError();
}

template <bool BF, int HD, int GM>
cudaError_t launch_attn_loop_g(const AttnArgs& a, cudaStream_t s) {
  const size_t smem = (size_t)2 * 2 * 128 * HD * (BF ? 2 : 4);
  static SmemOptIn opt;
  if (cudaError_t e = opt.ensure((const void*)attn_loop_kernel<BF, HD, GM>, smem)) return e;
  CTTS_LK(launch_k(attn_loop_kernel<BF, HD, GM>, dim3(a.nkv, a.batch), dim3(256), smem, s, a));
  return cudaGetLastError();
}
// Splits per (utterance, KV head) for the split kernel: the most (up to 8,
// a portable cluster) that keep the whole grid resident in one wave.
template <bool BF, int HD, int GM>
int attn_splits(const AttnArgs& a, size_t smem) {
  static PerDeviceInt per_sm;  // resident CTAs per SM of this instance
  int nb = per_sm.get([&] {
    int v = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, attn_split_kernel<BF, HD, GM>, 128, smem) != cudaSuccess) {
      (void)cudaGetLastError();
      v = 0;
    }
    return v;
  });
  const int pairs = a.batch * a.nkv;
  const int slots = nb * device_sms();
  return std::max(1, std::min(8, pairs > 0 ? slots / pairs : 1));
}

template <bool BF, int HD, int GM>
cudaError_t launch_attn_split_g(const AttnArgs& a, int S, size_t smem, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.nkv, a.batch, S);
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = S;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  CTTS_LK(cudaLaunchKernelEx(&cfg, attn_split_kernel<BF, HD, GM>, a));
  return cudaGetLastError();
}

// Tensor-core decode step (bf16 cache, head_dim 64 or 128, G <= 8): the
// splits per (utterance, KV head) keep the grid in one wave; tensor maps
// over this layer's K and V caches ([batch*nkv*cap, hd], 64-key boxes).
template <int HD>
cudaError_t launch_attn_mma(const AttnArgs& a, cudaStream_t s) {
  const size_t smem = (size_t)kAttnRing * 2 * (HD / 64) * 64 * 128 + 1024;
  static SmemOptIn opt;
  if (cudaError_t e = opt.ensure((const void*)attn_mma_kernel<HD>, smem)) return e;
  static PerDeviceInt per_sm;
  const int nb = per_sm.get([&] {
    int v = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, attn_mma_kernel<HD>, 128, smem) != cudaSuccess) {
      (void)cudaGetLastError();
      v = 0;
    }
    return v;
  });
  const int pairs = a.batch * a.nkv;
  const int S = std::max(1, std::min(8, pairs > 0 ? nb * device_sms() / pairs : 1));
  if (!encode_fn()) return cudaErrorNotSupported;
  const int rows = a.batch * a.nkv * a.cap;
  CUtensorMap tmK, tmV;
  if (!make_map(&tmK, a.kcache, rows, HD, 64) || !make_map(&tmV, a.vcache, rows, HD, 64))
    return cudaErrorInvalidPitchValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.nkv, a.batch, S);
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = S;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  CTTS_LK(cudaLaunchKernelEx(&cfg, attn_mma_kernel<HD>, tmK, tmV, a));
  return cudaGetLastError();
}

// Batched decode: the key-split cluster kernel when it takes at least two
// splits, else one CTA per (utterance, KV head) walking all its keys.
template <bool BF, int HD, int GM>
cudaError_t launch_attn_batched_g(const AttnArgs& a, cudaStream_t s) {
  const size_t smem = (size_t)2 * 2 * 64 * HD * (BF ? 2 : 4);
  static SmemOptIn opt;
  if (cudaError_t e = opt.ensure((const void*)attn_split_kernel<BF, HD, GM>, smem)) return e;
  const int S = attn_splits<BF, HD, GM>(a, smem);
  if (S >= 2) return launch_attn_split_g<BF, HD, GM>(a, S, smem, s);
  return launch_attn_loop_g<BF, HD, GM>(a, s);
}

// query heads per KV head held in registers: 1, 2, 3 or 4 (G <= 4)
template <bool BF, int HD>
cudaError_t launch_attn_loop_t(const AttnArgs& a, cudaStream_t s) {
  const int G = a.nq / a.nkv;
  if (G == 1) return launch_attn_batched_g<BF, HD, 1>(a, s);
  if (G == 2) return launch_attn_batched_g<BF, HD, 2>(a, s);
  if (G == 3) return launch_attn_batched_g<BF, HD, 3>(a, s);  // the benchmark LM: 12 query / 4 KV heads
  return launch_attn_batched_g<BF, HD, 4>(a, s);
}

cudaError_t launch_attn_decode(const AttnArgs& a, cudaStream_t s) {
  const int G = a.nq / a.nkv;
  if (G > kMaxG || a.nq % a.nkv != 0 || (a.hd != 64 && a.hd != 128) || a.chunk <= 0 || a.chunk > 128 ||
      a.chunk % 16 != 0 || a.nsplit * a.chunk < a.cap || a.rows != a.batch || !a.cnt)
    return cudaErrorInvalidValue;
  // bf16 cache: the tensor-core step (any batch; splits fill the GPU)
  if (a.kv_bf16 && G <= 8) return a.hd == 64 ? launch_attn_mma<64>(a, s) : launch_attn_mma<128>(a, s);
  // enough (utterance, kv head) pairs to fill the GPU: one CTA per pair
  // walking all its keys; otherwise split the keys over CTAs
  if (a.batch * a.nkv >= 128 && (a.kv_bf16 || a.hd == 64) && G <= 4) {
    if (a.kv_bf16) return a.hd == 64 ? launch_attn_loop_t<true, 64>(a, s) : launch_attn_loop_t<true, 128>(a, s);
    return launch_attn_loop_t<false, 64>(a, s);  // fp32 rows of head_dim 64 only
  }
  if (a.kv_bf16) return a.hd == 64 ? launch_attn_step_t<true, 64>(a, s) : launch_attn_step_t<true, 128>(a, s);
  return a.hd == 64 ? launch_attn_step_t<false, 64>(a, s) : launch_attn_step_t<false, 128>(a, s);
}

cudaError_t launch_attn_prefill(const AttnArgs& a, cudaStream_t s) {
  if (a.hd > kMaxHd || 128 % a.hd != 0) return cudaErrorInvalidValue;
  size_t smem = (size_t)(a.pos0 + a.rows) * sizeof(float);
  if (smem > 48 * 1024) return cudaErrorInvalidValue;
  dim3 grid(a.rows, a.nq);
  if (a.kv_bf16)
    CTTS_LK(launch_k(attn_prefill_kernel<true>, dim3(grid), dim3(128), smem, s, a));
  else
    CTTS_LK(launch_k(attn_prefill_kernel<false>, dim3(grid), dim3(128), smem, s, a));
  return cudaGetLastError();
}

cudaError_t launch_advance_pos(int* pos, int batch, cudaStream_t s) {
  CTTS_LK(launch_k(advance_pos_kernel, dim3((batch + 127) / 128), dim3(128), 0, s, pos, batch));
  return cudaGetLastError();
}

cudaError_t launch_rmsnorm_rows(const float* x, int M, int K, const float* w, float eps,
                                float* y, cudaStream_t s) {
  CTTS_LK(launch_k(rmsnorm_rows_kernel, dim3((M + 3) / 4), dim3(128), 0, s, x, M, K, w, eps, y));
  return cudaGetLastError();
}

cudaError_t launch_embed_gather(const void* table, int table_bf16, int vocab, int H,
                                const int64_t* ids, int n, float* out, int* bad,
                                cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  if (table_bf16)
    CTTS_LK(launch_k(embed_gather_kernel<true>, dim3(n), dim3(256), 0, s, table, vocab, H, ids, n, out, bad));
  else
    CTTS_LK(launch_k(embed_gather_kernel<false>, dim3(n), dim3(256), 0, s, table, vocab, H, ids, n, out, bad));
  return cudaGetLastError();
}

cudaError_t launch_rope_inplace(float* x, int M, int heads, int hd, const int* pos,
                                const float* inv_freq, cudaStream_t s) {
  if (M <= 0) return cudaSuccess;
  CTTS_LK(launch_k(rope_inplace_kernel, dim3(M, heads), dim3(64), 0, s, x, M, heads, hd, pos, inv_freq));
  return cudaGetLastError();
}

cudaError_t launch_swiglu(const float* gu, int M, int F, float* out, cudaStream_t s) {
  size_t n = (size_t)M * F;
  if (n == 0) return cudaSuccess;
  CTTS_LK(launch_k(swiglu_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, s, gu, M, F, out));
  return cudaGetLastError();
}

}  // namespace ctts

#ifdef CTTS_ATT_TRACE
// Copies the recorded timeline out ([launch][event] timestamps, 0 = not
// recorded; *n = launches) and resets it.
extern "C" __attribute__((visibility("default"))) int ctts_att_trace(long long* out, int* n) {
  cudaMemcpyFromSymbol(n, ctts::g_att_launch, sizeof(int));
  if (*n > ctts::kAttTraceLaunches) *n = ctts::kAttTraceLaunches;
  cudaMemcpyFromSymbol(out, ctts::g_att_trace, sizeof(ctts::g_att_trace));
  static long long zeros[ctts::kAttTraceLaunches * ctts::kAttTraceEvents] = {};
  cudaMemcpyToSymbol(ctts::g_att_trace, zeros, sizeof(zeros));
  int z = 0;
  return cudaMemcpyToSymbol(ctts::g_att_launch, &z, sizeof(int)) == cudaSuccess ? 0 : -2;
}
#endif
