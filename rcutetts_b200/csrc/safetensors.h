// safetensors.h -- minimal reader for the .safetensors container
// (8-byte little-endian header length, JSON header, raw tensor bytes), the
// format the reference loads with the `safetensors` crate
// (qwen.rs:75-120, dit.rs:104-159, weights.rs:98-186).
#pragma once

#include <stdint.h>

#include <map>
#include <string>
#include <vector>

namespace ctts {

struct StTensor {
  std::string dtype;  // "F32", "BF16", "F16", ...
  std::vector<int64_t> shape;
  uint64_t begin = 0, end = 0;  // byte offsets into the data section
};

struct StFile {
  std::vector<uint8_t> bytes;
  size_t data_off = 0;
  std::map<std::string, StTensor> tensors;
  const uint8_t* data(const StTensor& t) const { return bytes.data() + data_off + t.begin; }
};

// Returns an empty string on success, else an error message.
std::string st_read(const char* path, StFile* out);

}  // namespace ctts
