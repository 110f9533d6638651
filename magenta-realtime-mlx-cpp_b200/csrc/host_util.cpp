// Host utilities: errors, bf16 rounding, safetensors I/O, the reference's
// weight key layout, the random-init generator, presets, bucket table.
#include "host_util.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <stdexcept>
#include <thread>

namespace mrtdf {

static thread_local std::string g_last_error;

void set_error(int code, const std::string& msg) {
  (void)code;
  g_last_error = msg;
}
const char* last_error() { return g_last_error.c_str(); }

float bf16_round_host(float x) {
  uint32_t u;
  std::memcpy(&u, &x, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) {
    u = (u | 0x00400000u) & 0xffff0000u;
  } else {
    u = (u + 0x7fffu + ((u >> 16) & 1u)) & 0xffff0000u;
  }
  float r;
  std::memcpy(&r, &u, 4);
  return r;
}

uint16_t bf16_bits(float x) {
  const float r = bf16_round_host(x);
  uint32_t u;
  std::memcpy(&u, &r, 4);
  return (uint16_t)(u >> 16);
}

// ---------------------------------------------------------------------------
// safetensors: 8-byte little-endian header length, JSON header
// {"key": {"dtype": .., "shape": [..], "data_offsets": [b, e]}, ...},
// then the raw little-endian data (the format weights.cpp:29-35 loads
// through mx::load_safetensors).
// ---------------------------------------------------------------------------
namespace {
struct Json {
  const char* p;
  const char* e;
  [[noreturn]] void fail(const char* what) { throw Error{MRTDF_ERR_IO, std::string("safetensors header: ") + what}; }
  void ws() {
    while (p < e && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
  }
  bool eat(char c) {
    ws();
    if (p < e && *p == c) {
      ++p;
      return true;
    }
    return false;
  }
  void need(char c) {
    if (!eat(c)) fail("unexpected character");
  }
  std::string str() {
    ws();
    if (p >= e || *p != '"') fail("expected string");
    ++p;
    std::string out;
    while (p < e && *p != '"') {
      if (*p == '\\' && p + 1 < e) ++p;
      out.push_back(*p++);
    }
    if (p >= e) fail("unterminated string");
    ++p;
    return out;
  }
  int64_t num() {
    ws();
    char* q = nullptr;
    const long long v = std::strtoll(p, &q, 10);
    if (q == p) fail("expected number");
    p = q;
    return v;
  }
  void skip() {
    ws();
    if (p >= e) fail("truncated");
    if (*p == '"') {
      str();
      return;
    }
    if (*p == '{') {
      ++p;
      if (eat('}')) return;
      do {
        str();
        need(':');
        skip();
      } while (eat(','));
      need('}');
      return;
    }
    if (*p == '[') {
      ++p;
      if (eat(']')) return;
      do {
        skip();
      } while (eat(','));
      need(']');
      return;
    }
    while (p < e && *p != ',' && *p != '}' && *p != ']') ++p;
  }
};
}  // namespace

SafetensorsFile::SafetensorsFile(const std::string& path) {
  const int fd = ::open(path.c_str(), O_RDONLY);
  if (fd < 0) throw Error{MRTDF_ERR_IO, "WeightBundle: not a file: " + path};
  struct stat st;
  if (fstat(fd, &st) != 0 || st.st_size < 8) {
    ::close(fd);
    throw Error{MRTDF_ERR_IO, "not a safetensors file: " + path};
  }
  size_ = (size_t)st.st_size;
  map_ = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd, 0);
  ::close(fd);
  if (map_ == MAP_FAILED) {
    map_ = nullptr;
    throw Error{MRTDF_ERR_IO, "mmap failed: " + path};
  }
  const uint8_t* b = (const uint8_t*)map_;
  uint64_t hlen = 0;
  std::memcpy(&hlen, b, 8);
  if (hlen > size_ - 8) throw Error{MRTDF_ERR_IO, "safetensors header length out of range: " + path};
  const uint8_t* data = b + 8 + hlen;
  const size_t data_size = size_ - 8 - hlen;
  Json j{(const char*)b + 8, (const char*)b + 8 + hlen};
  j.need('{');
  if (!j.eat('}')) {
    do {
      const std::string key = j.str();
      j.need(':');
      if (key == "__metadata__") {
        j.skip();
        continue;
      }
      TensorRef t;
      uint64_t beg = 0, end = 0;
      j.need('{');
      do {
        const std::string f = j.str();
        j.need(':');
        if (f == "dtype") {
          t.dtype = j.str();
        } else if (f == "shape") {
          j.need('[');
          if (!j.eat(']')) {
            do {
              t.shape.push_back(j.num());
            } while (j.eat(','));
            j.need(']');
          }
        } else if (f == "data_offsets") {
          j.need('[');
          beg = (uint64_t)j.num();
          j.need(',');
          end = (uint64_t)j.num();
          j.need(']');
        } else {
          j.skip();
        }
      } while (j.eat(','));
      j.need('}');
      if (end < beg || end > data_size) throw Error{MRTDF_ERR_IO, "tensor data out of range: " + key};
      const size_t esize = t.dtype == "F32" ? 4 : (t.dtype == "BF16" ? 2 : 0);
      if (esize == 0) throw Error{MRTDF_ERR_IO, "unsupported dtype " + t.dtype + " for " + key};
      if ((uint64_t)t.numel() * esize != end - beg) throw Error{MRTDF_ERR_IO, "size mismatch for " + key};
      t.data = data + beg;
      t.nbytes = end - beg;
      tensors_[key] = t;
    } while (j.eat(','));
    j.need('}');
  }
}

SafetensorsFile::~SafetensorsFile() {
  if (map_) munmap(map_, size_);
}

const TensorRef* SafetensorsFile::find(const std::string& key) const {
  auto it = tensors_.find(key);
  return it == tensors_.end() ? nullptr : &it->second;
}

void write_safetensors(const std::string& path, const std::vector<OutTensor>& tensors) {
  std::vector<const OutTensor*> order;
  for (const auto& t : tensors) order.push_back(&t);
  std::sort(order.begin(), order.end(), [](const OutTensor* a, const OutTensor* b) { return a->key < b->key; });
  std::string h = "{";
  uint64_t off = 0;
  for (size_t i = 0; i < order.size(); ++i) {
    const OutTensor& t = *order[i];
    int64_t n = 1;
    for (auto s : t.shape) n *= s;
    if (i) h += ",";
    h += "\"" + t.key + "\":{\"dtype\":\"F32\",\"shape\":[";
    for (size_t k = 0; k < t.shape.size(); ++k) h += (k ? "," : "") + std::to_string(t.shape[k]);
    h += "],\"data_offsets\":[" + std::to_string(off) + "," + std::to_string(off + (uint64_t)n * 4) + "]}";
    off += (uint64_t)n * 4;
  }
  h += "}";
  while ((h.size() + 8) % 8) h += " ";
  FILE* f = std::fopen(path.c_str(), "wb");
  if (!f) throw Error{MRTDF_ERR_IO, "cannot write " + path};
  const uint64_t hl = h.size();
  bool ok = std::fwrite(&hl, 8, 1, f) == 1 && std::fwrite(h.data(), 1, h.size(), f) == h.size();
  for (const OutTensor* t : order) {
    int64_t n = 1;
    for (auto s : t->shape) n *= s;
    ok = ok && std::fwrite(t->data, 4, (size_t)n, f) == (size_t)n;
  }
  ok = (std::fclose(f) == 0) && ok;
  if (!ok) throw Error{MRTDF_ERR_IO, "short write: " + path};
}

// ---------------------------------------------------------------------------
// Weight layout: key names built as in model.cpp:82-109, 177-198 and the
// module constructors (modules.cpp:64, 92, 108, 127-128, 218-220, 238-241,
// 342-347, 369-381). Linear weights are (out, in).
// ---------------------------------------------------------------------------
std::vector<WeightSpec> weight_specs(const mrtdf_config& c) {
  const int64_t d = c.d_model, in = (int64_t)c.num_heads * c.d_kv, ff = c.d_ff, V = c.vocab_size;
  std::vector<WeightSpec> s;
  s.push_back({"token_embedding.weight", {V, d}, false});
  for (int i = 0; i < c.num_encoder_layers; ++i) {
    const std::string p = "encoder_layers." + std::to_string(i) + ".";
    s.push_back({p + "pre_attn_norm.weight", {d}, true});
    s.push_back({p + "self_attn.q_proj.weight", {in, d}, false});
    s.push_back({p + "self_attn.k_proj.weight", {in, d}, false});
    s.push_back({p + "self_attn.v_proj.weight", {in, d}, false});
    s.push_back({p + "self_attn.o_proj.weight", {d, in}, false});
    s.push_back({p + "pre_ffn_norm.weight", {d}, true});
    s.push_back({p + "ffn.wi_0.weight", {ff, d}, false});
    s.push_back({p + "ffn.wi_1.weight", {ff, d}, false});
    s.push_back({p + "ffn.wo.weight", {d, ff}, false});
  }
  s.push_back({"encoder_norm.weight", {d}, true});
  s.push_back({"temporal_rel_pos.relative_attention_bias.weight", {c.temporal_num_buckets, c.num_heads}, false});
  auto dec = [&](const std::string& fam, int n, bool cross) {
    for (int i = 0; i < n; ++i) {
      const std::string p = fam + "." + std::to_string(i) + ".";
      s.push_back({p + "pre_self_attn_norm.weight", {d}, true});
      s.push_back({p + "self_attn.q_proj.weight", {in, d}, false});
      s.push_back({p + "self_attn.k_proj.weight", {in, d}, false});
      s.push_back({p + "self_attn.v_proj.weight", {in, d}, false});
      s.push_back({p + "self_attn.o_proj.weight", {d, in}, false});
      if (cross) {
        s.push_back({p + "pre_cross_attn_norm.weight", {d}, true});
        s.push_back({p + "cross_attn.q_proj.weight", {in, d}, false});
        s.push_back({p + "cross_attn.k_proj.weight", {in, d}, false});
        s.push_back({p + "cross_attn.v_proj.weight", {in, d}, false});
        s.push_back({p + "cross_attn.o_proj.weight", {d, in}, false});
      }
      s.push_back({p + "pre_ffn_norm.weight", {d}, true});
      s.push_back({p + "ffn.wi_0.weight", {ff, d}, false});
      s.push_back({p + "ffn.wi_1.weight", {ff, d}, false});
      s.push_back({p + "ffn.wo.weight", {d, ff}, false});
    }
  };
  dec("temporal_layers", c.num_temporal_layers, true);
  s.push_back({"depth_rel_pos.relative_attention_bias.weight", {c.depth_num_buckets, c.num_heads}, false});
  dec("depth_layers", c.num_depth_layers, false);
  s.push_back({"decoder_norm.weight", {d}, true});
  s.push_back({"lm_head.weight", {V, d}, false});
  return s;
}

// Philox4x32-10 (Salmon et al., SC'11), host copy for the weight generator.
static void philox(uint32_t c[4], uint32_t k0, uint32_t k1) {
  for (int r = 0; r < 10; ++r) {
    const uint64_t p0 = (uint64_t)0xD2511F53u * c[0];
    const uint64_t p1 = (uint64_t)0xCD9E8D57u * c[2];
    const uint32_t n0 = (uint32_t)(p1 >> 32) ^ c[1] ^ k0;
    const uint32_t n2 = (uint32_t)(p0 >> 32) ^ c[3] ^ k1;
    c[1] = (uint32_t)p1;
    c[3] = (uint32_t)p0;
    c[0] = n0;
    c[2] = n2;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
}

void parallel_for(int64_t n, const std::function<void(int64_t, int64_t)>& fn) {
  int nt = (int)std::thread::hardware_concurrency();
  if (nt < 1) nt = 1;
  if (nt > 64) nt = 64;
  if (n < 65536 || nt == 1) {
    fn(0, n);
    return;
  }
  std::vector<std::thread> th;
  for (int t = 0; t < nt; ++t) {
    const int64_t a = n * t / nt, b = n * (t + 1) / nt;
    th.emplace_back([&fn, a, b]() { fn(a, b); });
  }
  for (auto& x : th) x.join();
}

void fill_random_tensor(uint64_t seed, int ordinal, float stddev, bool is_norm, bool norm_ones, float* out,
                        int64_t numel) {
  if (is_norm && norm_ones) {
    std::fill(out, out + numel, 1.0f);
    return;
  }
  const uint32_t k0 = (uint32_t)seed, k1 = (uint32_t)(seed >> 32);
  parallel_for((numel + 1) / 2, [&](int64_t a, int64_t b) {
    for (int64_t pr = a; pr < b; ++pr) {
      uint32_t c[4] = {(uint32_t)pr, (uint32_t)((uint64_t)pr >> 32), (uint32_t)ordinal, 0x5EEDu};
      philox(c, k0, k1);
      // Box-Muller on two uniforms in (0, 1).
      const double u1 = ((double)c[0] + 0.5) * (1.0 / 4294967296.0);
      const double u2 = ((double)c[1] + 0.5) * (1.0 / 4294967296.0);
      const double r = std::sqrt(-2.0 * std::log(u1));
      const double th = 6.283185307179586 * u2;
      const int64_t i = 2 * pr;
      out[i] = (float)(r * std::cos(th) * stddev);
      if (i + 1 < numel) out[i + 1] = (float)(r * std::sin(th) * stddev);
    }
  });
}

std::unique_ptr<HostWeights> random_host_weights(const mrtdf_config& c, uint64_t seed, float stddev, bool norm_ones) {
  auto hw = std::make_unique<HostWeights>();
  const auto specs = weight_specs(c);
  for (size_t i = 0; i < specs.size(); ++i) {
    int64_t n = 1;
    for (auto s : specs[i].shape) n *= s;
    std::vector<float> v((size_t)n);
    fill_random_tensor(seed, (int)i, stddev, specs[i].is_norm, norm_ones, v.data(), n);
    auto& slot = hw->owned[specs[i].key];
    slot = std::move(v);
    hw->ptr[specs[i].key] = slot.data();
  }
  return hw;
}

// ---------------------------------------------------------------------------
// Presets: DepthformerConfig::base() / large() (model.cpp:34-48,
// model.h:47-68) with SystemConfig's vocab layout (system.h:51-82).
// ---------------------------------------------------------------------------
bool config_preset(const std::string& name, mrtdf_config* o) {
  mrtdf_config c{};
  c.vocab_size = 29824;
  c.d_model = 768;
  c.d_kv = 64;
  c.d_ff = 2048;
  c.num_heads = 12;
  c.num_encoder_layers = 12;
  c.num_temporal_layers = 20;
  c.num_depth_layers = 4;
  c.max_encoder_length = 1006;
  c.rvq_depth = 16;
  c.temporal_num_buckets = 128;
  c.temporal_max_distance = 128;
  c.depth_num_buckets = 16;
  c.depth_max_distance = 16;
  c.codebook_size = 1024;
  c.codec_offset = 2;
  c.max_frames = 50;
  c.dtype = MRTDF_DTYPE_BF16;
  if (name == "base") {
  } else if (name == "large") {
    c.d_model = 1024;
    c.d_ff = 2816;
    c.num_heads = 16;
    c.num_encoder_layers = 24;
    c.num_temporal_layers = 40;
    c.num_depth_layers = 8;
  } else if (name == "hybrid") {
    // The benchmark architecture: large widths with base depths, 32 / 128
    // temporal buckets, 16 RVQ levels x 1024 codes + 4 specials.
    c.d_model = 1024;
    c.d_ff = 2816;
    c.num_heads = 16;
    c.vocab_size = 16388;
    c.temporal_num_buckets = 32;
    c.temporal_max_distance = 128;
  } else if (name == "tiny") {
    c.vocab_size = 2 + 16 * 64 + 2;
    c.d_model = 128;
    c.d_ff = 352;
    c.num_heads = 2;
    c.num_encoder_layers = 2;
    c.num_temporal_layers = 2;
    c.num_depth_layers = 2;
    c.max_encoder_length = 106;
    c.temporal_num_buckets = 32;
    c.temporal_max_distance = 128;
    c.codebook_size = 64;
    c.max_frames = 8;
  } else {
    return false;
  }
  *o = c;
  return true;
}

std::string config_check(const mrtdf_config& c) {
  if (c.d_kv != 64) return "d_kv must be 64";
  if (c.num_heads <= 0 || c.d_model <= 0 || c.d_ff <= 0) return "sizes must be positive";
  if (c.d_model % 32 != 0) return "d_model must be a multiple of 32";
  if (c.d_ff % 32 != 0) return "d_ff must be a multiple of 32";
  if (c.vocab_size < c.codec_offset + c.rvq_depth * c.codebook_size) return "vocab too small for the codec levels";
  if (c.max_frames <= 0 || c.rvq_depth <= 0 || c.max_encoder_length <= 0) return "lengths must be positive";
  if (c.dtype != MRTDF_DTYPE_FP32 && c.dtype != MRTDF_DTYPE_BF16) return "dtype must be fp32 or bf16";
  if (c.temporal_num_buckets < 2 || c.depth_num_buckets < 2) return "need at least 2 buckets";
  // decode self-attention handles up to 64 keys; split-K cross attention up to
  // 8 x 128 encoder positions
  if (c.max_frames > 64 || c.rvq_depth > 64) return "max_frames and rvq_depth must be <= 64";
  if (c.max_encoder_length > 1024) return "max_encoder_length must be <= 1024";
  return "";
}

// T5 relative-position bucket, unidirectional (modules.cpp:139-174).
int relative_bucket(int rel, int num_buckets, int max_distance) {
  int n = -rel;
  if (n < 0) n = 0;
  const int max_exact = num_buckets / 2;
  if (n < max_exact) return n;
  const float log_ratio = std::log((float)max_distance / (float)max_exact);
  const float v =
      (float)max_exact + (std::log((float)n / (float)max_exact) / log_ratio) * (float)(num_buckets - max_exact);
  const int b = (int)v;
  return std::min(b, num_buckets - 1);
}

// build_sinusoidal_position_embedding (model.cpp:54-80).
std::vector<float> sinusoid_table(int max_length, int features) {
  std::vector<float> data((size_t)max_length * features, 0.f);
  const int half = features / 2;
  const float scale_factor = -std::log(10000.0f / 1.0f) / (float)(half - 1);
  std::vector<float> div(half);
  for (int i = 0; i < half; ++i) div[i] = 1.0f * std::exp((float)i * scale_factor);
  for (int pos = 0; pos < max_length; ++pos)
    for (int i = 0; i < half; ++i) {
      const float a = (float)pos * div[i];
      data[(size_t)pos * features + i] = std::sin(a);
      data[(size_t)pos * features + half + i] = std::cos(a);
    }
  return data;
}

}  // namespace mrtdf
