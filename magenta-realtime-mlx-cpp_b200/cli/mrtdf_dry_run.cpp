// mrtdf_dry_run - the streaming chunk loop of the reference CLI's dry run
// (cli/main.cpp:436-516 in rhymeswithlion/magenta-realtime-mlx-cpp) driven
// through the C++ wrapper (include/mrtdf.hpp) of this engine.
//
// As in the reference: W warm-up chunks with seed + w, then N timed chunks,
// each seeded with seed + chunk_index (main.cpp:459; warm-up chunks advance
// the state and the chunk index too), every chunk one System::generate_chunk
// step (system.cpp:177-333): encoder ids from the rolling context
// (build_encoder_inputs_host) -> generate_tokens -> llm_to_rvq -> context
// roll. Reports "dry-run: N chunks in T s -> RTF Rx" and the per-chunk
// latency mean / p50 / p99 / min / max (main.cpp:496-514) on stderr, and one
// JSON line on stdout. The codec stage and playback are not part of this
// driver (the engine's hot path is the token loop).
//
//   mrtdf_dry_run [--preset hybrid] [--weights bundle.safetensors]
//                 [--dtype bf16|fp32] [--chunks 10] [--warmup 1] [--seed 1]
//                 [--temperature 1.1] [--top-k 40] [--guidance 4.0]
//                 [--style-seed 0] [--device 0] [--out ids.bin]
//
// Without --weights the random-init weights of seed 0 are used. --out
// writes every timed chunk's LLM ids as int32 (chunks, frames, rvq_depth).
#include <algorithm>
#include <chrono>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <iostream>
#include <memory>
#include <string>
#include <vector>

#include "mrtdf.hpp"

namespace {

struct Args {
  std::string preset = "hybrid";
  std::string weights;
  int dtype = MRTDF_DTYPE_BF16;
  int chunks = 10;
  int warmup = 1;
  uint64_t seed = 1;
  float temperature = 1.1f;
  int top_k = 40;
  float guidance = 4.0f;
  uint64_t style_seed = 0;
  int device = 0;
  std::string out;
};

Args parse(int argc, char** argv) {
  Args a;
  for (int i = 1; i < argc; ++i) {
    const std::string k = argv[i];
    auto val = [&]() -> std::string {
      if (i + 1 >= argc) throw std::runtime_error("missing value for " + k);
      return argv[++i];
    };
    if (k == "--preset") a.preset = val();
    else if (k == "--weights") a.weights = val();
    else if (k == "--dtype") a.dtype = val() == "fp32" ? MRTDF_DTYPE_FP32 : MRTDF_DTYPE_BF16;
    else if (k == "--chunks") a.chunks = std::stoi(val());
    else if (k == "--warmup") a.warmup = std::stoi(val());
    else if (k == "--seed") a.seed = std::stoull(val());
    else if (k == "--temperature") a.temperature = std::stof(val());
    else if (k == "--top-k") a.top_k = std::stoi(val());
    else if (k == "--guidance") a.guidance = std::stof(val());
    else if (k == "--style-seed") a.style_seed = std::stoull(val());
    else if (k == "--device") a.device = std::stoi(val());
    else if (k == "--out") a.out = val();
    else throw std::runtime_error("unknown argument " + k);
  }
  if (a.chunks < 1 || a.warmup < 0) throw std::runtime_error("--chunks must be >= 1 and --warmup >= 0");
  return a;
}

// The streaming state of System (system.h, SystemState): the rolling RVQ
// context of ctx_frames frames and the chunk index.
struct State {
  mrtdf::IntArray context;
  uint64_t chunk_index = 0;
};

}  // namespace

int main(int argc, char** argv) {
  try {
    const Args a = parse(argc, argv);
    const mrtdf::Config cfg = mrtdf::Config::preset(a.preset, a.dtype);
    std::unique_ptr<mrtdf::Depthformer> model;
    if (a.weights.empty())
      model = std::make_unique<mrtdf::Depthformer>(mrtdf::Depthformer::random(cfg, 0, a.dtype, a.device));
    else
      model = std::make_unique<mrtdf::Depthformer>(a.weights, cfg, a.dtype, a.device);
    mrtdf::Cache cache = model->empty_cache(1, true);

    // Context geometry of System: 4 encoder levels per frame + 6 style ids
    // fill max_encoder_length (250 frames x 4 + 6 = 1006 at the reference's).
    const int enc_depth = 4, style_depth = 6;
    const int ctx_frames = (cfg.max_encoder_length - style_depth) / enc_depth;
    const int frames = std::min(cfg.max_frames, ctx_frames);
    State state;
    state.context = mrtdf::IntArray({ctx_frames, cfg.rvq_depth},
                                    std::vector<int32_t>((size_t)ctx_frames * cfg.rvq_depth, -1));
    // Style ids: splitmix64 draws of --style-seed, uniform in the codec range
    // (stand-in for the MusicCoCa style tokens).
    std::vector<int32_t> style(style_depth);
    uint64_t x = a.style_seed;
    for (auto& s : style) {
      x += 0x9E3779B97F4A7C15ull;
      uint64_t z = x;
      z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
      z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
      z ^= z >> 31;
      s = cfg.codec_offset + (int32_t)(z % (uint64_t)(cfg.rvq_depth * cfg.codebook_size));
    }

    mrtdf::GenerateOptions base;
    base.num_frames = frames;
    base.rvq_depth = cfg.rvq_depth;
    base.temperature = a.temperature;
    base.top_k = a.top_k;
    base.guidance_weight = a.guidance;

    auto generate_chunk = [&](uint64_t seed) {
      const mrtdf::IntArray enc = mrtdf::build_encoder_inputs(state.context, style, enc_depth, cfg);
      mrtdf::GenerateOptions o = base;
      o.seed = seed;
      const mrtdf::IntArray toks = mrtdf::generate_tokens(*model, cache, enc, o);
      mrtdf::IntArray llm({frames, cfg.rvq_depth}, toks.data);
      const mrtdf::IntArray rvq = mrtdf::llm_to_rvq(llm, cfg);
      mrtdf::context_roll(state.context, rvq);
      ++state.chunk_index;
      return toks;
    };

    std::cerr << "warmup: " << a.warmup << " chunk(s)\n";
    for (int w = 0; w < a.warmup; ++w) generate_chunk(a.seed + (uint64_t)w);

    std::vector<double> per_chunk_ms;
    std::vector<int32_t> ids;
    const auto t0 = std::chrono::steady_clock::now();
    for (int i = 0; i < a.chunks; ++i) {
      const auto c0 = std::chrono::steady_clock::now();
      const mrtdf::IntArray toks = generate_chunk(a.seed + state.chunk_index);
      per_chunk_ms.push_back(
          std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - c0).count());
      ids.insert(ids.end(), toks.data.begin(), toks.data.end());
    }
    const double dt = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    const double chunk_s = frames * 0.04;  // 25 Hz codec frames
    std::vector<double> sorted = per_chunk_ms;
    std::sort(sorted.begin(), sorted.end());
    auto pct = [&](double p) {
      if (sorted.size() == 1) return sorted.front();
      const double idx = p * (sorted.size() - 1);
      const size_t lo = (size_t)idx, hi = std::min(lo + 1, sorted.size() - 1);
      return sorted[lo] * (1.0 - (idx - lo)) + sorted[hi] * (idx - lo);
    };
    double sum = 0.0;
    for (double v : per_chunk_ms) sum += v;
    const double mean = sum / per_chunk_ms.size();
    std::fprintf(stderr, "dry-run: %d chunks in %.2f s -> RTF %.2fx\n", a.chunks, dt, a.chunks * chunk_s / dt);
    std::fprintf(stderr, "  latency ms  mean=%.1f p50=%.1f p99=%.1f min=%.1f max=%.1f\n", mean, pct(0.5), pct(0.99),
                 sorted.front(), sorted.back());
    std::printf(
        "{\"chunks\": %d, \"warmup\": %d, \"frames\": %d, \"seconds\": %.6f, \"rtf\": %.4f, \"ms_mean\": %.4f, "
        "\"ms_p50\": %.4f, \"ms_p99\": %.4f, \"ms_min\": %.4f, \"ms_max\": %.4f, \"tokens_per_s\": %.2f}\n",
        a.chunks, a.warmup, frames, dt, a.chunks * chunk_s / dt, mean, pct(0.5), pct(0.99), sorted.front(),
        sorted.back(), (double)ids.size() / dt);
    if (!a.out.empty()) {
      FILE* f = std::fopen(a.out.c_str(), "wb");
      if (!f || std::fwrite(ids.data(), 4, ids.size(), f) != ids.size())
        throw std::runtime_error("cannot write " + a.out);
      std::fclose(f);
    }
    return 0;
  } catch (const std::out_of_range& e) {
    std::cerr << "mrtdf_dry_run: out of range: " << e.what() << "\n";
    return 3;
  } catch (const std::exception& e) {
    std::cerr << "mrtdf_dry_run: " << e.what() << "\n";
    return 2;
  }
}
