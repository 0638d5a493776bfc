// api_common.h -- host-side plumbing shared by the C ABI translation units:
// error reporting, device allocations owned by a handle, and named weight
// slots that accept float32 / bf16 host tensors and store them in the
// handle's weight dtype.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <cmath>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/cutetts_b200.h"
#include "kernels.cuh"
#include "safetensors.h"

namespace ctts {

int set_error(int code, const std::string& msg);

#define CTTS_CK(call)                                                                   \
  do {                                                                                  \
    cudaError_t _e = (call);                                                            \
    if (_e != cudaSuccess)                                                              \
      return ::ctts::set_error(CTTS_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(_e)); \
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
    cudaMemset(p, 0, n * sizeof(T) + 16);
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

// Upload float32 host data into a slot (converting to the model dtype).
inline int upload_f32(const Slot& s, const float* data, size_t n, int model_bf16) {
  if (s.weight && model_bf16) {
    std::vector<uint16_t> b(n);
    for (size_t i = 0; i < n; i++) b[i] = host_f2bf(data[i]);
    CTTS_CK(cudaMemcpy(s.dst, b.data(), n * 2, cudaMemcpyHostToDevice));
  } else {
    CTTS_CK(cudaMemcpy(s.dst, data, n * 4, cudaMemcpyHostToDevice));
  }
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
