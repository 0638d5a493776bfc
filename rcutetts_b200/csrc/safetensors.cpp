// safetensors.cpp -- minimal .safetensors reader (see safetensors.h).
#include "safetensors.h"

#include <cstdio>
#include <cstring>

namespace ctts {

namespace {

struct Json {
  const char* p;
  const char* e;
  std::string err;

  void ws() {
    while (p < e && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) p++;
  }
  bool expect(char c) {
    ws();
    if (p >= e || *p != c) {
      err = std::string("expected '") + c + "'";
      return false;
    }
    p++;
    return true;
  }
  bool str(std::string* s) {
    ws();
    if (p >= e || *p != '"') return (err = "expected string", false);
    p++;
    s->clear();
    while (p < e && *p != '"') {
      if (*p == '\\') {
        p++;
        if (p >= e) break;
        char c = *p;
        if (c == 'u') {  // keep escaped code units verbatim (names are ASCII)
          if (e - p < 5) return (err = "bad escape", false);
          s->append(p - 1, 6);
          p += 5;
          continue;
        }
        s->push_back(c == 'n' ? '\n' : c == 't' ? '\t' : c);
        p++;
        continue;
      }
      s->push_back(*p++);
    }
    if (p >= e) return (err = "unterminated string", false);
    p++;
    return true;
  }
  bool num(int64_t* v) {
    ws();
    char* end = nullptr;
    long long x = strtoll(p, &end, 10);
    if (end == p) return (err = "expected number", false);
    p = end;
    *v = x;
    return true;
  }
  // skip any value
  bool skip() {
    ws();
    if (p >= e) return (err = "eof", false);
    if (*p == '"') {
      std::string s;
      return str(&s);
    }
    if (*p == '{' || *p == '[') {
      char open = *p, close = open == '{' ? '}' : ']';
      p++;
      ws();
      if (p < e && *p == close) return p++, true;
      while (true) {
        if (open == '{') {
          std::string k;
          if (!str(&k) || !expect(':')) return false;
        }
        if (!skip()) return false;
        ws();
        if (p < e && *p == ',') {
          p++;
          continue;
        }
        return expect(close);
      }
    }
    while (p < e && *p != ',' && *p != '}' && *p != ']') p++;
    return true;
  }
};

}  // namespace

std::string st_read(const char* path, StFile* out) {
  FILE* f = fopen(path, "rb");
  if (!f) return std::string("cannot open ") + path;
  fseek(f, 0, SEEK_END);
  long sz = ftell(f);
  fseek(f, 0, SEEK_SET);
  if (sz < 8) {
    fclose(f);
    return "file too small";
  }
  out->bytes.resize((size_t)sz);
  size_t rd = fread(out->bytes.data(), 1, (size_t)sz, f);
  fclose(f);
  if (rd != (size_t)sz) return "short read";
  uint64_t hlen = 0;
  memcpy(&hlen, out->bytes.data(), 8);
  if (hlen > (uint64_t)sz - 8) return "bad header length";
  out->data_off = 8 + hlen;
  Json j{reinterpret_cast<const char*>(out->bytes.data()) + 8,
         reinterpret_cast<const char*>(out->bytes.data()) + 8 + hlen, {}};
  if (!j.expect('{')) return j.err;
  j.ws();
  if (j.p < j.e && *j.p == '}') return "";
  while (true) {
    std::string name;
    if (!j.str(&name) || !j.expect(':')) return j.err;
    if (name == "__metadata__") {
      if (!j.skip()) return j.err;
    } else {
      StTensor t;
      if (!j.expect('{')) return j.err;
      while (true) {
        std::string key;
        if (!j.str(&key) || !j.expect(':')) return j.err;
        if (key == "dtype") {
          if (!j.str(&t.dtype)) return j.err;
        } else if (key == "shape" || key == "data_offsets") {
          if (!j.expect('[')) return j.err;
          std::vector<int64_t> v;
          j.ws();
          if (j.p < j.e && *j.p == ']') {
            j.p++;
          } else {
            while (true) {
              int64_t x;
              if (!j.num(&x)) return j.err;
              v.push_back(x);
              j.ws();
              if (j.p < j.e && *j.p == ',') {
                j.p++;
                continue;
              }
              if (!j.expect(']')) return j.err;
              break;
            }
          }
          if (key == "shape") {
            t.shape = v;
          } else {
            if (v.size() != 2) return "bad data_offsets for " + name;
            t.begin = (uint64_t)v[0];
            t.end = (uint64_t)v[1];
          }
        } else if (!j.skip()) {
          return j.err;
        }
        j.ws();
        if (j.p < j.e && *j.p == ',') {
          j.p++;
          continue;
        }
        if (!j.expect('}')) return j.err;
        break;
      }
      if (t.end < t.begin || out->data_off + t.end > (uint64_t)sz) return "tensor out of file: " + name;
      out->tensors[name] = t;
    }
    j.ws();
    if (j.p < j.e && *j.p == ',') {
      j.p++;
      continue;
    }
    if (!j.expect('}')) return j.err;
    break;
  }
  return "";
}

}  // namespace ctts
