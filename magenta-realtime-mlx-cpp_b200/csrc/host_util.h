// Host-side utilities of the engine: error reporting, bf16 rounding, the
// safetensors reader/writer, the reference's weight key layout and the
// random-init weight generator. No CUDA types in here.
#pragma once

#include <cstdint>
#include <functional>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/mrtdf.h"

namespace mrtdf {

// ---- errors ----------------------------------------------------------------
struct Error {
  int code;
  std::string msg;
};
void set_error(int code, const std::string& msg);
const char* last_error();

// Body of a C ABI entry point: runs f, turns a thrown Error (or any
// std::exception, as MRTDF_ERR_INVALID) into the status code and the
// thread-local message of mrtdf_last_error().
template <typename F>
int guarded(F&& f) {
  try {
    f();
    return MRTDF_OK;
  } catch (const Error& e) {
    set_error(e.code, e.msg);
    return e.code;
  } catch (const std::exception& e) {
    set_error(MRTDF_ERR_INVALID, e.what());
    return MRTDF_ERR_INVALID;
  }
}

// ---- numerics --------------------------------------------------------------
float bf16_round_host(float x);
uint16_t bf16_bits(float x);  // RNE

// ---- safetensors -------------------------------------------------------------
struct TensorRef {
  std::string dtype;  // "F32" or "BF16"
  std::vector<int64_t> shape;
  const uint8_t* data = nullptr;
  size_t nbytes = 0;
  int64_t numel() const {
    int64_t n = 1;
    for (auto s : shape) n *= s;
    return n;
  }
};

class SafetensorsFile {
 public:
  // Maps `path`; throws Error{MRTDF_ERR_IO} on a missing / malformed file.
  explicit SafetensorsFile(const std::string& path);
  ~SafetensorsFile();
  SafetensorsFile(const SafetensorsFile&) = delete;
  SafetensorsFile& operator=(const SafetensorsFile&) = delete;
  const TensorRef* find(const std::string& key) const;
  const std::map<std::string, TensorRef>& tensors() const { return tensors_; }

 private:
  void* map_ = nullptr;
  size_t size_ = 0;
  std::map<std::string, TensorRef> tensors_;
};

// Write float32 tensors as a safetensors file (header keys sorted).
struct OutTensor {
  std::string key;
  std::vector<int64_t> shape;
  const float* data;
};
void write_safetensors(const std::string& path, const std::vector<OutTensor>& tensors);

// ---- weight layout -----------------------------------------------------------
// One entry per tensor of the reference bundle, in model construction order
// (model.cpp:173-198): key, shape, and whether it is an RMSNorm scale.
struct WeightSpec {
  std::string key;
  std::vector<int64_t> shape;
  bool is_norm;
};
std::vector<WeightSpec> weight_specs(const mrtdf_config& c);

// Fill `out` (numel floats) with tensor `ordinal` of the random-init bundle:
// N(0, stddev) via Box-Muller over Philox4x32-10 keyed by `seed`, counter
// (pair index low, pair index high, ordinal, 0x5EED). Norm scales are 1.0
// when `norm_ones`.
void fill_random_tensor(uint64_t seed, int ordinal, float stddev, bool is_norm, bool norm_ones, float* out,
                        int64_t numel);

// Random-init bundle held in host memory (float32), keyed like the file.
struct HostWeights {
  std::map<std::string, std::vector<float>> owned;
  std::map<std::string, const float*> ptr;
};
std::unique_ptr<HostWeights> random_host_weights(const mrtdf_config& c, uint64_t seed, float stddev, bool norm_ones);

// Run fn(i) for i in [0, n) on the host's cores.
void parallel_for(int64_t n, const std::function<void(int64_t, int64_t)>& fn);

// ---- config ------------------------------------------------------------------
bool config_preset(const std::string& name, mrtdf_config* out);
// Returns an empty string when the engine supports `c`, else the reason.
std::string config_check(const mrtdf_config& c);

// ---- relative-position buckets and the sinusoid table -----------------------
int relative_bucket(int rel, int num_buckets, int max_distance);
std::vector<float> sinusoid_table(int max_length, int features);

}  // namespace mrtdf
