// mrtdf.hpp - header-only C++ face of the C ABI (mrtdf.h) for C++ callers
// of the reference's Depthformer API (rhymeswithlion/magenta-realtime-mlx-cpp).
//
// It re-exposes the reference's entry points with their argument order and
// exception types, over host arrays instead of mx::array:
//
//   reference (src/magenta_realtime_mlx/...)             here
//   Depthformer(bundle, config, dtype)  model.h:74-75    Depthformer(path, config, dtype, device)
//   empty_temporal_cache / empty_depth_cache             Depthformer::empty_cache()  (one KV arena)
//                                       model.h:103-104
//   encode(tokens)                      model.h:81       encode(tokens, cache)
//   temporal_step(frame_emb, encoder_output, cache,      temporal_step(frame_emb, encoder_output,
//                 frame_idx, bias)      model.h:113-117                cache, frame_idx)
//   depth_step(tok_emb, cache, depth_idx, bias)          depth_step(tok_emb, cache, depth_idx)
//                                       model.h:121-124
//   token_embedding()(ids)              model.h:127      token_embedding(ids)
//   generate_tokens(model, enc_tokens, opts, masks, ...) generate_tokens(model, cache, enc_tokens, opts)
//                                       decode.h:112-119
//
// Differences that follow from the engine's design: the KV arena (both
// caches) lives on the GPU inside a Cache object instead of a caller-held
// vector<LayerCache>; the cross-attention K/V of every temporal layer are
// projected by encode into that cache (the reference projects them on frame
// 0 of temporal_step, modules.cpp:258-278), so temporal_step's
// encoder_output argument is kept for the argument order only; the
// relative-position biases are precomputed at weight load
// (precompute_*_biases, model.cpp:302-320), so no bias argument is taken;
// vocab masks are the per-level codec ranges System::build_vocab_masks builds
// (system.cpp:135-157), switched on by GenerateOptions::use_vocab_masks.
//
// Errors throw where the reference throws: std::out_of_range for an index
// past a maximum or a missing weight key (model.cpp:216-218,
// weights.cpp:40-41), std::runtime_error for everything else (cache-size
// mismatch model.cpp:326-328, shape errors, CUDA failures). Both carry the
// C ABI status in mrtdf::Error / mrtdf::RangeError.
#ifndef MRTDF_HPP_
#define MRTDF_HPP_

#include <cstdint>
#include <filesystem>
#include <memory>
#include <optional>
#include <stdexcept>
#include <string>
#include <string_view>
#include <utility>
#include <vector>

#include "mrtdf.h"

namespace mrtdf {

class Error : public std::runtime_error {
 public:
  Error(int code, const std::string& msg) : std::runtime_error(msg), code_(code) {}
  int code() const { return code_; }

 private:
  int code_;
};

class RangeError : public std::out_of_range {
 public:
  RangeError(int code, const std::string& msg) : std::out_of_range(msg), code_(code) {}
  int code() const { return code_; }

 private:
  int code_;
};

inline void check(int rc) {
  if (rc == MRTDF_OK) return;
  const std::string msg = mrtdf_last_error();
  if (rc == MRTDF_ERR_RANGE || rc == MRTDF_ERR_KEY) throw RangeError(rc, msg);
  throw Error(rc, msg);
}

// Row-major host array with its shape.
template <typename T>
struct Array {
  std::vector<T> data;
  std::vector<int64_t> shape;
  Array() = default;
  Array(std::vector<int64_t> s) : shape(std::move(s)) { data.resize(static_cast<size_t>(numel())); }
  Array(std::vector<int64_t> s, std::vector<T> d) : data(std::move(d)), shape(std::move(s)) {
    if (static_cast<int64_t>(data.size()) != numel()) throw Error(MRTDF_ERR_INVALID, "array: data / shape mismatch");
  }
  int64_t numel() const {
    int64_t n = 1;
    for (int64_t v : shape) n *= v;
    return n;
  }
  int64_t dim(int i) const { return shape.at(static_cast<size_t>(i < 0 ? static_cast<int>(shape.size()) + i : i)); }
  T* ptr() { return data.data(); }
  const T* ptr() const { return data.data(); }
};
using FloatArray = Array<float>;
using IntArray = Array<int32_t>;

// DepthformerConfig (model.h:47-68) + the decode loop's vocab layout.
struct Config : mrtdf_config {
  static Config preset(const std::string& name, int dtype = MRTDF_DTYPE_BF16) {
    Config c{};
    check(mrtdf_config_preset(name.c_str(), &c));
    c.dtype = dtype;
    return c;
  }
  static Config base(int dtype = MRTDF_DTYPE_BF16) { return preset("base", dtype); }    // model.cpp:34-36
  static Config large(int dtype = MRTDF_DTYPE_BF16) { return preset("large", dtype); }  // model.cpp:38-48
};

// GenerateOptions (decode.h:48-57); the defaults are the reference's.
struct GenerateOptions {
  int num_frames = 50;
  int rvq_depth = 16;
  float temperature = 1.1f;
  int top_k = 40;
  float guidance_weight = 4.0f;
  std::optional<uint64_t> seed;
  bool use_vocab_masks = true;
};

class Depthformer;

// The KV arena of one stream (empty_temporal_cache + empty_depth_cache,
// model.h:103-104): temporal self K/V, cross K/V and depth self K/V on the
// GPU, `num_sequences` CFG pairs (2 rows each) or single rows.
class Cache {
 public:
  Cache(const Cache&) = delete;
  Cache& operator=(const Cache&) = delete;
  Cache(Cache&& o) noexcept : st_(std::exchange(o.st_, nullptr)), rows_(o.rows_), nseq_(o.nseq_) {}
  Cache& operator=(Cache&& o) noexcept {
    if (this != &o) {
      reset();
      st_ = std::exchange(o.st_, nullptr);
      rows_ = o.rows_;
      nseq_ = o.nseq_;
    }
    return *this;
  }
  ~Cache() { reset(); }
  int rows() const { return rows_; }
  int num_sequences() const { return nseq_; }
  mrtdf_stream* handle() const { return st_; }

 private:
  friend class Depthformer;
  Cache(mrtdf_engine* eng, int num_sequences, bool cfg) : nseq_(num_sequences) {
    check(mrtdf_stream_create(eng, num_sequences, cfg ? 1 : 0, &st_));
    rows_ = mrtdf_stream_rows(st_);
  }
  void reset() {
    if (st_) mrtdf_stream_destroy(st_);
    st_ = nullptr;
  }
  mrtdf_stream* st_ = nullptr;
  int rows_ = 0;
  int nseq_ = 0;
};

class Depthformer {
 public:
  // Depthformer(bundle, config, dtype) (model.h:74-75): `weights_path` is a
  // safetensors bundle with the reference's key names (F32 or BF16 tensors).
  Depthformer(const std::string& weights_path, const Config& config, int dtype = MRTDF_DTYPE_BF16, int device = 0)
      : cfg_(config) {
    cfg_.dtype = dtype;
    check(mrtdf_create(&cfg_, device, &eng_));
    try {
      check(mrtdf_load_safetensors(eng_, weights_path.c_str()));
    } catch (...) {
      mrtdf_destroy(eng_);
      throw;
    }
  }
  // The random-init weights of `seed` (N(0, stddev), RMSNorm scales 1).
  static Depthformer random(const Config& config, uint64_t seed, int dtype = MRTDF_DTYPE_BF16, int device = 0,
                            float stddev = 0.02f) {
    Depthformer m(config, dtype, device);
    check(mrtdf_load_random(m.eng_, seed, stddev, 1));
    return m;
  }
  Depthformer(const Depthformer&) = delete;
  Depthformer& operator=(const Depthformer&) = delete;
  Depthformer(Depthformer&& o) noexcept : cfg_(o.cfg_), eng_(std::exchange(o.eng_, nullptr)) {}
  ~Depthformer() {
    if (eng_) mrtdf_destroy(eng_);
  }

  const Config& config() const { return cfg_; }
  mrtdf_engine* handle() const { return eng_; }

  // empty_temporal_cache() + empty_depth_cache() (model.h:103-104).
  Cache empty_cache(int num_sequences = 1, bool cfg = true) const { return Cache(eng_, num_sequences, cfg); }

  // encode(tokens) (model.h:81): tokens (rows, S) int32 -> (rows, S, d);
  // also fills `cache`'s cross K/V and resets its temporal cache.
  FloatArray encode(const IntArray& tokens, Cache& cache) const {
    if (tokens.shape.size() != 2 || tokens.dim(0) != cache.rows())
      throw Error(MRTDF_ERR_INVALID, "encode: tokens must be (rows, seq_len)");
    const int S = static_cast<int>(tokens.dim(1));
    FloatArray out({tokens.dim(0), S, cfg_.d_model});
    check(mrtdf_encode(cache.handle(), tokens.ptr(), S, out.ptr()));
    return out;
  }

  // temporal_step(frame_emb, encoder_output, cache, frame_idx, bias)
  // (model.h:113-117): frame_emb (rows, 1, d) or null for PAD (frame 0)
  // -> (rows, 1, d). encoder_output is not read (see the file comment).
  FloatArray temporal_step(const FloatArray* frame_emb, const FloatArray& encoder_output, Cache& cache,
                           int frame_idx) const {
    (void)encoder_output;
    FloatArray out({cache.rows(), 1, cfg_.d_model});
    if (frame_emb && frame_emb->numel() != static_cast<int64_t>(cache.rows()) * cfg_.d_model)
      throw Error(MRTDF_ERR_INVALID, "temporal_step: frame_emb must be (rows, 1, d_model)");
    check(mrtdf_temporal_step(cache.handle(), frame_emb ? frame_emb->ptr() : nullptr, frame_idx, out.ptr()));
    return out;
  }

  // depth_step(tok_emb, cache, depth_idx, bias) (model.h:121-124): tok_emb
  // (rows, 1, d) or null for the last temporal output -> logits (rows, V).
  FloatArray depth_step(const FloatArray* tok_emb, Cache& cache, int depth_idx) const {
    FloatArray out({cache.rows(), cfg_.vocab_size});
    if (tok_emb && tok_emb->numel() != static_cast<int64_t>(cache.rows()) * cfg_.d_model)
      throw Error(MRTDF_ERR_INVALID, "depth_step: tok_emb must be (rows, 1, d_model)");
    check(mrtdf_depth_step(cache.handle(), tok_emb ? tok_emb->ptr() : nullptr, depth_idx, out.ptr()));
    return out;
  }

  // token_embedding()(ids) (model.h:127): ids (n) -> (n, d).
  FloatArray token_embedding(const IntArray& ids) const {
    FloatArray out({ids.numel(), cfg_.d_model});
    check(mrtdf_token_embedding(eng_, ids.ptr(), static_cast<int>(ids.numel()), out.ptr()));
    return out;
  }

 private:
  Depthformer(const Config& config, int dtype, int device) : cfg_(config) {
    cfg_.dtype = dtype;
    check(mrtdf_create(&cfg_, device, &eng_));
  }
  Config cfg_;
  mrtdf_engine* eng_ = nullptr;
};

inline mrtdf_gen_opts to_c(const GenerateOptions& o) {
  mrtdf_gen_opts c{};
  c.num_frames = o.num_frames;
  c.rvq_depth = o.rvq_depth;
  c.temperature = o.temperature;
  c.top_k = o.top_k;
  c.guidance_weight = o.guidance_weight;
  c.use_vocab_masks = o.use_vocab_masks ? 1 : 0;
  c.seed = o.seed.value_or(0);
  c.uniforms = nullptr;
  return c;
}

// generate_tokens(model, enc_tokens, opts, vocab_masks, ...) (decode.h:112-119,
// non-speculative): enc_tokens (rows, S) -> (num_sequences, num_frames,
// rvq_depth) LLM ids; `seeds` (one per sequence) override opts.seed + i.
inline IntArray generate_tokens(const Depthformer& model, Cache& cache, const IntArray& enc_tokens,
                                const GenerateOptions& opts, const std::vector<uint64_t>* seeds = nullptr) {
  if (enc_tokens.shape.size() != 2 || enc_tokens.dim(0) != cache.rows())
    throw Error(MRTDF_ERR_INVALID, "generate_tokens: enc_tokens must be (rows, seq_len)");
  if (seeds && static_cast<int>(seeds->size()) != cache.num_sequences())
    throw Error(MRTDF_ERR_INVALID, "generate_tokens: one seed per sequence");
  (void)model;
  const mrtdf_gen_opts c = to_c(opts);
  IntArray out({cache.num_sequences(), opts.num_frames, opts.rvq_depth});
  check(mrtdf_generate_tokens(cache.handle(), enc_tokens.ptr(), static_cast<int>(enc_tokens.dim(1)), &c,
                              seeds ? seeds->data() : nullptr, out.ptr()));
  return out;
}

// ---- streaming glue (System, system.cpp) -------------------------------------
// build_encoder_inputs_host (system.cpp:62-95): context (frames, rvq_depth)
// RVQ codes (negative = empty) + style ids -> (2, frames * enc_depth + style).
inline IntArray build_encoder_inputs(const IntArray& context, const std::vector<int32_t>& style, int enc_depth,
                                     const Config& c) {
  const int frames = static_cast<int>(context.dim(0)), depth = static_cast<int>(context.dim(1));
  IntArray out({2, frames * enc_depth + static_cast<int64_t>(style.size())});
  check(mrtdf_build_encoder_inputs(context.ptr(), frames, depth, enc_depth, style.data(),
                                   static_cast<int>(style.size()), c.codebook_size, c.codec_offset, out.ptr()));
  return out;
}

// llm_to_rvq (rvq.cpp:112-134): (n, rvq_depth) LLM ids -> RVQ codes.
inline IntArray llm_to_rvq(const IntArray& llm, const Config& c) {
  IntArray out(llm.shape);
  check(mrtdf_llm_to_rvq(llm.ptr(), static_cast<int>(llm.dim(0)), static_cast<int>(llm.dim(1)), c.codebook_size,
                         c.codec_offset, out.ptr()));
  return out;
}

// Context roll (system.cpp:320-333), in place.
inline void context_roll(IntArray& context, const IntArray& new_codes) {
  check(mrtdf_context_roll(context.ptr(), static_cast<int>(context.dim(0)), static_cast<int>(context.dim(1)),
                           new_codes.ptr(), static_cast<int>(new_codes.dim(0))));
}

// InferenceBundlePaths (weights.h:70-78).
struct InferenceBundlePaths {
  std::filesystem::path spectrostream_encoder, spectrostream_decoder, spectrostream_codebooks;
  std::filesystem::path musiccoca_encoder, musiccoca_codebooks, musiccoca_vocab;
  std::filesystem::path depthformer;
};

// resolve_inference_bundle(cache_root, tag) (weights.cpp:72-120): throws
// mrtdf::Error (a std::runtime_error) when the root is not a directory or a
// file of the bundle is missing, with the reference's message.
inline InferenceBundlePaths resolve_inference_bundle(const std::filesystem::path& cache_root, std::string_view tag) {
  std::unique_ptr<mrtdf_bundle_paths> c(new mrtdf_bundle_paths());
  check(mrtdf_resolve_inference_bundle(cache_root.string().c_str(), std::string(tag).c_str(), c.get()));
  InferenceBundlePaths p;
  p.spectrostream_encoder = c->spectrostream_encoder;
  p.spectrostream_decoder = c->spectrostream_decoder;
  p.spectrostream_codebooks = c->spectrostream_codebooks;
  p.musiccoca_encoder = c->musiccoca_encoder;
  p.musiccoca_codebooks = c->musiccoca_codebooks;
  p.musiccoca_vocab = c->musiccoca_vocab;
  p.depthformer = c->depthformer;
  return p;
}

}  // namespace mrtdf

#endif  // MRTDF_HPP_
