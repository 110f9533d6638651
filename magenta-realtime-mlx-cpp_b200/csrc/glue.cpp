// Streaming glue around the chunk loop: encoder-input build, context roll
// and RVQ <-> LLM id maps. Integer work on the host (microseconds per chunk).
//
// Reference (rhymeswithlion/magenta-realtime-mlx-cpp):
//   build_encoder_inputs_host  src/magenta_realtime_mlx/system.cpp:62-95
//   context roll               system.cpp:320-333
//   rvq_to_llm / llm_to_rvq    src/magenta_realtime_mlx/rvq.cpp:105-134
//   resolve_inference_bundle   src/magenta_realtime_mlx/weights.cpp:72-120
#include <cstring>
#include <filesystem>
#include <string>

#include "host_util.h"

using namespace mrtdf;

namespace {
constexpr int kMaskToken = 1;  // SystemConfig::vocab_mask_token (system.h:75)
}  // namespace

extern "C" {

int mrtdf_build_encoder_inputs(const int32_t* context, int ctx_frames, int rvq_depth, int enc_depth,
                               const int32_t* style, int style_depth, int codebook_size, int codec_offset,
                               int32_t* out) {
  return guarded([&] {
    if (!context || !out || (style_depth > 0 && !style)) throw Error{MRTDF_ERR_INVALID, "NULL argument"};
    if (ctx_frames < 0 || rvq_depth <= 0 || enc_depth < 0 || enc_depth > rvq_depth || style_depth < 0)
      throw Error{MRTDF_ERR_INVALID, "bad sizes"};
    const int enc_len = ctx_frames * enc_depth + style_depth;
    // Row 0: visible context levels mapped into the LLM vocab, MASK for
    // empty (negative) slots, then the style ids.
    for (int f = 0; f < ctx_frames; ++f)
      for (int d = 0; d < enc_depth; ++d) {
        const int32_t v = context[f * rvq_depth + d];
        out[f * enc_depth + d] = v >= 0 ? codec_offset + d * codebook_size + v : kMaskToken;
      }
    if (style_depth > 0) std::memcpy(&out[ctx_frames * enc_depth], style, sizeof(int32_t) * style_depth);
    // Row 1: the same codec context with the style masked (CFG uncond row).
    std::memcpy(&out[enc_len], &out[0], sizeof(int32_t) * ctx_frames * enc_depth);
    for (int i = ctx_frames * enc_depth; i < enc_len; ++i) out[enc_len + i] = kMaskToken;
  });
}

int mrtdf_context_roll(int32_t* context, int ctx_frames, int rvq_depth, const int32_t* new_codes,
                       int chunk_frames) {
  return guarded([&] {
    if (!context || !new_codes) throw Error{MRTDF_ERR_INVALID, "NULL argument"};
    if (chunk_frames < 0 || chunk_frames > ctx_frames) throw Error{MRTDF_ERR_INVALID, "chunk longer than context"};
    // new[f] = old[(f + chunk_frames) % ctx_frames] for the kept frames,
    // then the chunk's codes fill the last chunk_frames frames.
    const int keep = ctx_frames - chunk_frames;
    std::memmove(context, context + (size_t)chunk_frames * rvq_depth, sizeof(int32_t) * keep * rvq_depth);
    std::memcpy(context + (size_t)keep * rvq_depth, new_codes, sizeof(int32_t) * chunk_frames * rvq_depth);
  });
}

int mrtdf_llm_to_rvq(const int32_t* llm, int n, int rvq_depth, int codebook_size, int codec_offset, int32_t* out) {
  return guarded([&] {
    if (!llm || !out || codebook_size <= 0) throw Error{MRTDF_ERR_INVALID, "bad argument"};
    for (int i = 0; i < n; ++i)
      for (int d = 0; d < rvq_depth; ++d) {
        const int32_t shifted = llm[i * rvq_depth + d] - codec_offset;
        // mx::remainder follows Python semantics: result has the divisor's sign.
        int32_t r = shifted % codebook_size;
        if (r < 0) r += codebook_size;
        if (shifted - r != d * codebook_size)
          throw Error{MRTDF_ERR_INVALID, "llm_to_rvq: token levels do not match expected RVQ structure"};
        out[i * rvq_depth + d] = r;
      }
  });
}

int mrtdf_resolve_inference_bundle(const char* cache_root, const char* tag, mrtdf_bundle_paths* out) {
  return guarded([&] {
    if (!cache_root || !tag || !out) throw Error{MRTDF_ERR_INVALID, "NULL argument"};
    namespace fs = std::filesystem;
    const fs::path root(cache_root);
    std::error_code ec;
    if (!fs::is_directory(root, ec))
      throw Error{MRTDF_ERR_IO, "resolve_inference_bundle: not a directory: " + root.string()};
    struct Entry {
      const char* label;
      fs::path path;
      char* dst;
    };
    const Entry entries[] = {
        {"SpectroStream encoder", root / "spectrostream_encoder.safetensors", out->spectrostream_encoder},
        {"SpectroStream decoder", root / "spectrostream_decoder.safetensors", out->spectrostream_decoder},
        {"SpectroStream codebooks", root / "spectrostream_codebooks.safetensors", out->spectrostream_codebooks},
        {"MusicCoCa encoder", root / "musiccoca_encoder.safetensors", out->musiccoca_encoder},
        {"MusicCoCa codebooks", root / "musiccoca_codebooks.safetensors", out->musiccoca_codebooks},
        {"MusicCoCa SentencePiece vocab", root / "musiccoca_vocab.model", out->musiccoca_vocab},
        {"Depthformer checkpoint", root / "depthformer" / ("depthformer_" + std::string(tag) + ".safetensors"),
         out->depthformer},
    };
    std::string missing;
    for (const Entry& e : entries)
      if (!fs::is_regular_file(e.path, ec)) missing += "  - " + std::string(e.label) + ": " + e.path.string() + "\n";
    if (!missing.empty())
      throw Error{MRTDF_ERR_IO, "Incomplete Magenta RT C++ inference bundle (looked under " + root.string() + "):\n" +
                                    missing + "Run `make ensure-weights-cache` to download + bundle."};
    for (const Entry& e : entries) {
      const std::string s = e.path.string();
      if (s.size() >= MRTDF_PATH_MAX) throw Error{MRTDF_ERR_RANGE, "bundle path too long: " + s};
      std::memcpy(e.dst, s.c_str(), s.size() + 1);
    }
  });
}

int mrtdf_rvq_to_llm(const int32_t* rvq, int n, int rvq_depth, int codebook_size, int codec_offset, int32_t* out) {
  return guarded([&] {
    if (!rvq || !out) throw Error{MRTDF_ERR_INVALID, "NULL argument"};
    for (int i = 0; i < n; ++i)
      for (int d = 0; d < rvq_depth; ++d) out[i * rvq_depth + d] = codec_offset + d * codebook_size + rvq[i * rvq_depth + d];
  });
}

}  // extern "C"
