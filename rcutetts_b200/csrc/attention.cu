// attention.cu -- LM attention blocks and small LM ops.
//
// qk_rope_append: QK-Norm + NeoX RoPE of the new q/k rows and the KV-cache
//   append (qwen.rs:323-340 decode, 255-272 prefill).
// attn_decode: GQA decode attention over each utterance's ragged cache
//   (qwen.rs:341-362).  Split over the sequence so a batch of one still
//   fills the GPU: CTA (split, kv_head, utterance) scores its chunk of keys
//   for all query heads of the group (the K/V rows are read once per group,
//   not once per query head), then a combine pass merges the splits with
//   the usual max-rescaled softmax sums.
// attn_prefill: causal attention of T new rows against the cache
//   (qwen.rs:273-297).
#include "common.cuh"
#include "kernels.cuh"

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

// grid (nsplit, nkv, batch), 128 threads.  Partial layout per
// (b, q head, split): [m, l, acc[hd]].
template <bool BF>
__global__ void __launch_bounds__(128) attn_decode_kernel(const AttnArgs a) {
  grid_dep_enter();
  const int split = blockIdx.x, kh = blockIdx.y, b = blockIdx.z;
  const int hd = a.hd, nq = a.nq, nkv = a.nkv;
  const int G = nq / nkv;
  const int tid = threadIdx.x;
  const int n = min(a.pos[b] + 1, a.cap);  // keys incl. the row appended this step
  const int r0 = split * a.chunk;
  const int r1 = min(r0 + a.chunk, n);
  float* part_base = a.part + (((size_t)b * nq + kh * G) * a.nsplit + split) * (hd + 2);
  const size_t pstride = (size_t)a.nsplit * (hd + 2);

  __shared__ __align__(16) float qs[kMaxG * kMaxHd];
  __shared__ float sc[kMaxG][128];
  __shared__ float red[kMaxG][4];
  __shared__ float stat[kMaxG][2];
  __shared__ __align__(16) float accs[kMaxG][kMaxHd];

  if (r0 >= r1) {  // empty split: neutral partial
    for (int i = tid; i < G * (hd + 2); i += blockDim.x) {
      int g = i / (hd + 2), c = i % (hd + 2);
      part_base[g * pstride + c] = c == 0 ? -INFINITY : 0.0f;
    }
    return;
  }
  const float scale = 1.0f / sqrtf((float)hd);
  for (int i = tid; i < G * hd; i += blockDim.x) {
    int g = i / hd, d = i % hd;
    qs[i] = a.qrot[(size_t)b * nq * hd + (kh * G + g) * hd + d];
  }
  __syncthreads();

  const size_t kvbase = ((size_t)b * nkv + kh) * a.cap * hd;
  // phase 1: one thread per key row
  const int j = r0 + tid;
  float s[kMaxG];
#pragma unroll
  for (int g = 0; g < kMaxG; g++) s[g] = -INFINITY;
  if (j < r1) {
#pragma unroll
    for (int g = 0; g < kMaxG; g++) s[g] = 0.0f;
    const size_t kr = kvbase + (size_t)j * hd;
#pragma unroll 8
    for (int d = 0; d < hd; d += 8) {
      float kv[8];
      if (BF) {
        uint4 t = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(a.kcache) + kr + d);
        kv[0] = bf_lo(t.x); kv[1] = bf_hi(t.x); kv[2] = bf_lo(t.y); kv[3] = bf_hi(t.y);
        kv[4] = bf_lo(t.z); kv[5] = bf_hi(t.z); kv[6] = bf_lo(t.w); kv[7] = bf_hi(t.w);
      } else {
        const float* kp = reinterpret_cast<const float*>(a.kcache) + kr + d;
        float4 t0 = *reinterpret_cast<const float4*>(kp);
        float4 t1 = *reinterpret_cast<const float4*>(kp + 4);
        kv[0] = t0.x; kv[1] = t0.y; kv[2] = t0.z; kv[3] = t0.w;
        kv[4] = t1.x; kv[5] = t1.y; kv[6] = t1.z; kv[7] = t1.w;
      }
#pragma unroll
      for (int g = 0; g < kMaxG; g++) {
        if (g >= G) break;
        const float* q = qs + g * hd + d;
#pragma unroll
        for (int e = 0; e < 8; e++) s[g] = fmaf(q[e], kv[e], s[g]);
      }
    }
#pragma unroll
    for (int g = 0; g < kMaxG; g++) s[g] *= scale;
  }
  // phase 2: max and sum per head
  const int lane = tid & 31, warp = tid >> 5;
#pragma unroll
  for (int g = 0; g < kMaxG; g++) {
    if (g >= G) break;
    float m = warp_max(s[g]);
    if (lane == 0) red[g][warp] = m;
  }
  __syncthreads();
  if (tid < G) {
    float m = fmaxf(fmaxf(red[tid][0], red[tid][1]), fmaxf(red[tid][2], red[tid][3]));
    stat[tid][0] = m;
  }
  __syncthreads();
#pragma unroll
  for (int g = 0; g < kMaxG; g++) {
    if (g >= G) break;
    float p = j < r1 ? expf(s[g] - stat[g][0]) : 0.0f;
    sc[g][tid] = p;
    float l = warp_sum(p);
    if (lane == 0) red[g][warp] = l;
  }
  __syncthreads();
  if (tid < G) stat[tid][1] = red[tid][0] + red[tid][1] + red[tid][2] + red[tid][3];
  __syncthreads();
  // phase 3: P.V ; thread -> (dim d, row partition)
  const int parts = blockDim.x / hd;  // 2 for hd=64
  const int d = tid % hd, pp = tid / hd;
  float acc[kMaxG];
#pragma unroll
  for (int g = 0; g < kMaxG; g++) acc[g] = 0.0f;
  if (pp < parts) {
    // eight V rows in flight per iteration
    for (int j0 = r0 + pp; j0 < r1; j0 += 8 * parts) {
      float vv[8];
#pragma unroll
      for (int u = 0; u < 8; u++) {
        const int jj = j0 + u * parts;
        vv[u] = jj < r1 ? ld_kv<BF>(a.vcache, kvbase + (size_t)jj * hd + d) : 0.0f;
      }
#pragma unroll
      for (int u = 0; u < 8; u++) {
        const int jj = j0 + u * parts;
        if (jj >= r1) break;
#pragma unroll
        for (int g = 0; g < kMaxG; g++) {
          if (g >= G) break;
          acc[g] = fmaf(sc[g][jj - r0], vv[u], acc[g]);
        }
      }
    }
  }
  for (int p2 = 1; p2 < parts; p2++) {
    __syncthreads();
    if (pp == p2)
      for (int g = 0; g < G; g++) accs[g][d] = acc[g];
    __syncthreads();
    if (pp == 0)
      for (int g = 0; g < G; g++) acc[g] += accs[g][d];
  }
  __syncthreads();
  if (pp == 0) {
    for (int g = 0; g < G; g++) {
      float* pb = part_base + g * pstride;
      pb[2 + d] = acc[g];
      if (d == 0) {
        pb[0] = stat[g][0];
        pb[1] = stat[g][1];
      }
    }
  }
}

// grid (batch, nq), hd threads
__global__ void attn_combine_kernel(const AttnArgs a) {
  grid_dep_enter();
  const int b = blockIdx.x, h = blockIdx.y, d = threadIdx.x;
  const int hd = a.hd;
  const float* p = a.part + ((size_t)b * a.nq + h) * a.nsplit * (hd + 2);
  float M = -INFINITY;
  for (int s = 0; s < a.nsplit; s++) M = fmaxf(M, p[s * (hd + 2)]);
  float L = 0.0f, acc = 0.0f;
  for (int s = 0; s < a.nsplit; s++) {
    const float* ps = p + s * (hd + 2);
    if (ps[0] == -INFINITY) continue;
    float w = expf(ps[0] - M);
    L = fmaf(ps[1], w, L);
    acc = fmaf(ps[2 + d], w, acc);
  }
  const size_t o = (size_t)b * a.nq * hd + h * hd + d;
  if (a.out_b)
    a.out_b[o] = f2bf(acc / L);
  else
    a.out[o] = acc / L;
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

cudaError_t launch_attn_decode(const AttnArgs& a, cudaStream_t s) {
  const int G = a.nq / a.nkv;
  if (G > kMaxG || a.hd % 8 != 0 || a.hd > kMaxHd || a.chunk != 128 || 128 % a.hd != 0)
    return cudaErrorInvalidValue;
  dim3 grid(a.nsplit, a.nkv, a.batch);
  if (a.kv_bf16)
    CTTS_LK(launch_k(attn_decode_kernel<true>, dim3(grid), dim3(128), 0, s, a));
  else
    CTTS_LK(launch_k(attn_decode_kernel<false>, dim3(grid), dim3(128), 0, s, a));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  CTTS_LK(launch_k(attn_combine_kernel, dim3(a.batch, a.nq), dim3(a.hd), 0, s, a));
  return cudaGetLastError();
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
