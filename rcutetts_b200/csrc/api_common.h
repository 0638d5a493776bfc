// api_common.h -- host-side plumbing shared by the C ABI translation units:
// error reporting, device allocations owned by a handle, and named weight
// slots that accept float32 / bf16 host tensors and store them in the
// handle's weight dtype.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <array>
#include <cmath>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/cutetts_b200.h"
#include "kernels.cuh"
#include "safetensors.h"
#include "tc_linear.cuh"

namespace ctts {

int set_error(int code, const std::string& msg);

// On failure the runtime's last-error slot is cleared too, so a
// non-sticky error cannot resurface in a later, unrelated launch check.
#define CTTS_CK(call)                                                                   \
  do {                                                                                  \
    cudaError_t _e = (call);                                                            \
    if (_e != cudaSuccess) {                                                            \
      (void)cudaGetLastError();                                                         \
      return ::ctts::set_error(CTTS_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(_e)); \
    }                                                                                   \
  } while (0)

#define CTTS_REQ(cond, code, msg)                       \
  do {                                                  \
    if (!(cond)) return ::ctts::set_error(code, msg);   \
  } while (0)

inline uint16_t host_f2bf(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x7FFFFFu)) return (uint16_t)((u >> 16) | 0x40);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}
inline float host_bf2f(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

// Owner of device allocations (freed on destruction).
struct DevArena {
  std::vector<void*> ptrs;
  ~DevArena() {
    for (void* p : ptrs) cudaFree(p);
  }
  template <class T>
  T* alloc(size_t n) {
    void* p = nullptr;
    if (cudaMalloc(&p, n * sizeof(T) + 16) != cudaSuccess) return nullptr;
    // zeroed before any stream (blocking or not) can touch it
    cudaMemset(p, 0, n * sizeof(T) + 16);
    cudaStreamSynchronize(cudaStreamLegacy);
    ptrs.push_back(p);
    return reinterpret_cast<T*>(p);
  }
};

// A named destination for one checkpoint tensor.
struct Slot {
  void* dst = nullptr;           // device destination (row offset applied)
  std::vector<int64_t> shape;    // expected shape
  bool weight = true;            // true: stored in the model dtype; false: float32
  bool set = false;
  bool optional = false;
  // transform applied on the host before upload (e.g. transpose-conv repack)
  int transform = 0;
  int t_a = 0, t_b = 0, t_c = 0;
  // weight-norm pair bookkeeping (VAE): g/v collected then fused
  std::vector<float> wn_g, wn_v;
};

struct SlotTable {
  std::unordered_map<std::string, Slot> slots;
  int model_bf16 = 0;

  void add(const std::string& name, void* dst, std::vector<int64_t> shape, bool weight,
           bool optional = false) {
    Slot s;
    s.dst = dst;
    s.shape = std::move(shape);
    s.weight = weight;
    s.optional = optional;
    slots[name] = s;
  }
  int missing() const {
    int n = 0;
    for (auto& kv : slots)
      if (!kv.second.set && !kv.second.optional) n++;
    return n;
  }
  std::string first_missing() const {
    for (auto& kv : slots)
      if (!kv.second.set && !kv.second.optional) return kv.first;
    return "";
  }
};

// Convert `n` host elements (f32 or bf16 bits) to float32.
inline void host_to_f32(const void* src, int dtype, size_t n, std::vector<float>* out) {
  out->resize(n);
  if (dtype == CTTS_F32) {
    memcpy(out->data(), src, n * 4);
  } else {
    const uint16_t* s = reinterpret_cast<const uint16_t*>(src);
    for (size_t i = 0; i < n; i++) (*out)[i] = host_bf2f(s[i]);
  }
}

constexpr int kXformNone = 0;
constexpr int kXformTranspose = 1;      // VAE ConvTranspose repack (api_vae.cu)
constexpr int kXformRowInterleave = 2;  // 64-row groups at a 128-row pitch (t_b = row length)

// Upload float32 host data into a slot (converting to the model dtype).
// kXformRowInterleave places rows [64g, 64g+64) of the tensor at rows
// [128g, 128g+64) of the destination: the gate/up tile interleave the
// SwiGLU linears read.
inline int upload_f32(const Slot& s, const float* data, size_t n, int model_bf16) {
  const bool bf = s.weight && model_bf16;
  const size_t es = bf ? 2 : 4;
  std::vector<uint16_t> b;
  const void* src = data;
  if (bf) {
    b.resize(n);
    for (size_t i = 0; i < n; i++) b[i] = host_f2bf(data[i]);
    src = b.data();
  }
  if (s.transform == kXformRowInterleave) {
    const size_t row = (size_t)s.t_b * es, rows = n / (size_t)s.t_b;
    if (rows % 64) return set_error(CTTS_ERR_ARG, "interleaved tensor rows must be a multiple of 64");
    CTTS_CK(cudaMemcpy2D(s.dst, 128 * row, src, 64 * row, 64 * row, rows / 64, cudaMemcpyHostToDevice));
  } else {
    CTTS_CK(cudaMemcpy(s.dst, src, n * es, cudaMemcpyHostToDevice));
  }
  // a pageable-source copy may return before its DMA lands; the handle's
  // kernels run on non-blocking streams, so wait for it here
  CTTS_CK(cudaStreamSynchronize(cudaStreamLegacy));
  return CTTS_OK;
}

// Device scratch for the split-K tensor-core linears.
struct TcScratch {
  float* part = nullptr;
  size_t part_floats = 0;
  int* counters = nullptr;
  int ncounters = 0;
  int* err = nullptr;
};

// Scratch floats the widest of `shapes` (M, N, K triples) needs.
inline size_t tc_scratch_need(const std::vector<std::array<int, 3>>& shapes, int max_splitk,
                              int* counters) {
  size_t need = 0;
  int cnt = 0;
  for (auto& sh : shapes) {
    TcPlan p = tc_plan(sh[0], sh[1], sh[2], tc_num_sms(), max_splitk);
    need = std::max(need, tc_scratch_floats(p));
    cnt = std::max(cnt, p.ntiles * p.mtiles);
  }
  if (counters) *counters = cnt;
  return need;
}

inline int tc_alloc(DevArena& arena, TcScratch* sc, const std::vector<std::array<int, 3>>& shapes,
                    int* err) {
  int cnt = 0;
  size_t need = tc_scratch_need(shapes, 64, &cnt);
  sc->part = arena.alloc<float>(std::max<size_t>(need, 1));
  sc->part_floats = need;
  sc->counters = arena.alloc<int>(std::max(cnt, 1));
  sc->ncounters = cnt;
  sc->err = err;
  if (!sc->part || !sc->counters) return set_error(CTTS_ERR_NOMEM, "tensor-core scratch allocation failed");
  return CTTS_OK;
}

// Y = epi(X[M,K] . W[N,K]^T) on the tensor cores; falls back to fewer K
// splits (down to 1) when the scratch is too small for the planned split.
inline int tc_run(const TcScratch& sc, const uint16_t* x, int M, int K, const void* w, int N,
                  const TcArgs& epi, cudaStream_t s, int* nl) {
  TcCall c;
  c.x = x;
  c.w = reinterpret_cast<const uint16_t*>(w);
  c.M = M;
  c.N = N;
  c.K = K;
  c.epi = epi;
  c.part = sc.part;
  c.part_floats = sc.part_floats;
  c.counters = sc.counters;
  c.counter_count = sc.ncounters;
  c.err = sc.err;
  // split-K partials are reduced in the cluster's shared memory: the plan
  // needs no global scratch, so any K split the planner picks can run
  c.max_splitk = M > 256 ? 1 : 64;
  cudaError_t e = launch_tc_linear(c, s);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return set_error(CTTS_ERR_CUDA, std::string("tc_linear: ") + cudaGetErrorString(e));
  }
  if (nl) *nl += tc_plan(M, N, K, tc_num_sms(), c.max_splitk).mtiles;
  return CTTS_OK;
}

inline size_t shape_numel(const std::vector<int64_t>& s) {
  size_t n = 1;
  for (int64_t d : s) n *= (size_t)d;
  return n;
}

std::string shape_str(const std::vector<int64_t>& s);

// Generic set_tensor over a slot table (no transforms).
int slot_set(SlotTable& t, const char* name, const void* host, int dtype, const int64_t* shape,
             int ndim);

// Load every tensor with `prefix` from a safetensors file into a slot table
// through `setter` (name without prefix).
template <class F>
int load_safetensors(const char* path, const char* prefix, F setter) {
  CTTS_REQ(path, CTTS_ERR_ARG, "null path");
  StFile f;
  std::string err = st_read(path, &f);
  CTTS_REQ(err.empty(), CTTS_ERR_IO, err);
  std::string pre = prefix ? prefix : "";
  int n = 0;
  for (auto& kv : f.tensors) {
    if (kv.first.compare(0, pre.size(), pre) != 0) continue;
    const StTensor& t = kv.second;
    int dt;
    if (t.dtype == "F32")
      dt = CTTS_F32;
    else if (t.dtype == "BF16")
      dt = CTTS_BF16;
    else
      return set_error(CTTS_ERR_IO, "unsupported dtype " + t.dtype + " for " + kv.first);
    size_t expect = shape_numel(t.shape) * (dt == CTTS_F32 ? 4 : 2);
    CTTS_REQ(expect == t.end - t.begin, CTTS_ERR_IO, "size mismatch for " + kv.first);
    std::string name = kv.first.substr(pre.size());
    int rc = setter(name.c_str(), f.data(t), dt, t.shape.data(), (int)t.shape.size());
    if (rc == CTTS_ERR_ARG && ::ctts_last_error() && strstr(::ctts_last_error(), "unknown tensor"))
      continue;  // tensors of other modules in a combined checkpoint
    if (rc != CTTS_OK) return rc;
    n++;
  }
  CTTS_REQ(n > 0, CTTS_ERR_IO, "no tensors with prefix '" + pre + "'");
  return CTTS_OK;
}

inline cudaStream_t as_stream(void* s, cudaStream_t dflt) {
  return s ? reinterpret_cast<cudaStream_t>(s) : dflt;
}

// RoPE inverse frequencies theta^(-2i/d) in float32 (qwen.rs:160, dit.rs:282).
inline std::vector<float> rope_inv_freq(int hd, float theta) {
  std::vector<float> v(hd / 2);
  for (int i = 0; i < hd / 2; i++) v[i] = powf(theta, -((float)(2 * i)) / (float)hd);
  return v;
}

}  // namespace ctts
