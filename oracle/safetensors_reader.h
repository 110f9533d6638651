// TEST INFRASTRUCTURE ONLY - internal header of the CPU oracle: a minimal
// safetensors reader shared by the Depthformer and SpectroStream oracles.
// Nothing in the engine includes this file.
#pragma once

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <map>
#include <stdexcept>
#include <string>
#include <vector>

namespace oracle {

// ---------------------------------------------------------------------------
// safetensors reader (the format MLX's load_safetensors reads,
// weights.cpp:29-35): 8-byte little-endian header length, JSON header,
// raw little-endian tensor bytes. F32 and BF16 tensors are accepted.
// ---------------------------------------------------------------------------
struct TensorInfo {
  std::string dtype;
  std::vector<int64_t> shape;
  uint64_t begin = 0, end = 0;
};

struct JsonCursor {
  const char* p;
  const char* e;
  void ws() { while (p < e && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p; }
  bool eat(char c) { ws(); if (p < e && *p == c) { ++p; return true; } return false; }
  void need(char c) { if (!eat(c)) throw std::runtime_error(std::string("safetensors header: expected '") + c + "'"); }
  std::string str() {
    ws();
    if (p >= e || *p != '"') throw std::runtime_error("safetensors header: expected string");
    ++p;
    std::string out;
    while (p < e && *p != '"') {
      if (*p == '\\' && p + 1 < e) { ++p; }
      out.push_back(*p++);
    }
    if (p >= e) throw std::runtime_error("safetensors header: unterminated string");
    ++p;
    return out;
  }
  int64_t num() {
    ws();
    char* q = nullptr;
    long long v = std::strtoll(p, &q, 10);
    if (q == p) throw std::runtime_error("safetensors header: expected number");
    p = q;
    return v;
  }
  void skip_value() {
    ws();
    if (p >= e) throw std::runtime_error("safetensors header: truncated");
    if (*p == '"') { str(); return; }
    if (*p == '{') {
      ++p;
      if (eat('}')) return;
      do { str(); need(':'); skip_value(); } while (eat(','));
      need('}');
      return;
    }
    if (*p == '[') {
      ++p;
      if (eat(']')) return;
      do { skip_value(); } while (eat(','));
      need(']');
      return;
    }
    while (p < e && *p != ',' && *p != '}' && *p != ']') ++p;
  }
};

struct SafeTensors {
  std::map<std::string, TensorInfo> info;
  const uint8_t* data = nullptr;
  size_t data_size = 0;
  void* map = nullptr;
  size_t map_size = 0;

  explicit SafeTensors(const char* path) {
    int fd = ::open(path, O_RDONLY);
    if (fd < 0) throw std::runtime_error(std::string("cannot open ") + path);
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size < 8) { ::close(fd); throw std::runtime_error("bad safetensors file"); }
    map_size = (size_t)st.st_size;
    map = mmap(nullptr, map_size, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (map == MAP_FAILED) { map = nullptr; throw std::runtime_error("mmap failed"); }
    const uint8_t* b = (const uint8_t*)map;
    uint64_t hlen = 0;
    std::memcpy(&hlen, b, 8);
    if (hlen + 8 > map_size) throw std::runtime_error("safetensors header length out of range");
    JsonCursor c{(const char*)b + 8, (const char*)b + 8 + hlen};
    c.need('{');
    if (!c.eat('}')) {
      do {
        std::string key = c.str();
        c.need(':');
        if (key == "__metadata__") { c.skip_value(); continue; }
        TensorInfo ti;
        c.need('{');
        do {
          std::string f = c.str();
          c.need(':');
          if (f == "dtype") ti.dtype = c.str();
          else if (f == "shape") {
            c.need('[');
            if (!c.eat(']')) { do { ti.shape.push_back(c.num()); } while (c.eat(',')); c.need(']'); }
          } else if (f == "data_offsets") {
            c.need('['); ti.begin = (uint64_t)c.num(); c.need(','); ti.end = (uint64_t)c.num(); c.need(']');
          } else c.skip_value();
        } while (c.eat(','));
        c.need('}');
        info[key] = ti;
      } while (c.eat(','));
      c.need('}');
    }
    data = b + 8 + hlen;
    data_size = map_size - 8 - hlen;
  }
  ~SafeTensors() { if (map) munmap(map, map_size); }

  // Tensor `key` as float32, checking the element count (weights.cpp:37-44
  // throws std::out_of_range for a missing key).
  std::vector<float> get(const std::string& key, int64_t expect_numel) const {
    auto it = info.find(key);
    if (it == info.end()) throw std::out_of_range("missing key \"" + key + "\"");
    const TensorInfo& t = it->second;
    int64_t n = 1;
    for (auto s : t.shape) n *= s;
    if (n != expect_numel) throw std::runtime_error("shape mismatch for " + key);
    if (t.end > data_size || t.begin > t.end) throw std::runtime_error("offsets out of range for " + key);
    std::vector<float> out((size_t)n);
    if (t.dtype == "F32") {
      if (t.end - t.begin != (uint64_t)n * 4) throw std::runtime_error("size mismatch for " + key);
      std::memcpy(out.data(), data + t.begin, (size_t)n * 4);
    } else if (t.dtype == "BF16") {
      if (t.end - t.begin != (uint64_t)n * 2) throw std::runtime_error("size mismatch for " + key);
      const uint16_t* s = (const uint16_t*)(data + t.begin);
      for (int64_t i = 0; i < n; ++i) { uint32_t u = (uint32_t)s[i] << 16; std::memcpy(&out[i], &u, 4); }
    } else {
      throw std::runtime_error("unsupported dtype " + t.dtype + " for " + key);
    }
    return out;
  }
};

}  // namespace oracle
