/*
 * mrtdf.h - C ABI of the B200 Depthformer decoding engine.
 *
 * This is the drop-in boundary for the per-chunk hot path of the C++ Magenta
 * RealTime reimplementation (rhymeswithlion/magenta-realtime-mlx-cpp). Each
 * entry point names the reference interface it replaces (file:line inside that
 * project). All arguments are plain C types: host pointers unless the name
 * ends in `_dev`, sizes as int, status as int (0 = MRTDF_OK). On failure the
 * thread-local message from mrtdf_last_error() says what went wrong; the
 * reference throws C++ exceptions in the same places.
 *
 * Threading: a handle may be used by one host thread at a time. Different
 * mrtdf_stream handles of one engine may be driven from different threads.
 */
#ifndef MRTDF_H_
#define MRTDF_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes -------------------------------------------------------- */
#define MRTDF_OK 0
#define MRTDF_ERR_INVALID 1 /* bad argument or shape (std::runtime_error in the reference) */
#define MRTDF_ERR_CUDA 2    /* a CUDA runtime call failed */
#define MRTDF_ERR_IO 3      /* file missing or malformed safetensors */
#define MRTDF_ERR_STATE 4   /* call order: e.g. temporal_step before encode */
#define MRTDF_ERR_KEY 5     /* weight key missing (std::out_of_range, weights.cpp:40-41) */
#define MRTDF_ERR_TIMEOUT 6 /* a device-side bounded wait gave up */
#define MRTDF_ERR_RANGE 7   /* index past a maximum (std::out_of_range, model.cpp:216-218) */

#define MRTDF_DTYPE_FP32 0
#define MRTDF_DTYPE_BF16 1

/*
 * Model hyperparameters. Mirrors DepthformerConfig (depthformer/model.h:47-68)
 * plus the vocabulary layout constants of SystemConfig (system.h:51-82) that
 * the decode loop needs, and the compute dtype (parse_dtype, dtype.h:36).
 */
typedef struct mrtdf_config {
  int vocab_size;
  int d_model;
  int d_kv;
  int d_ff;
  int num_heads;
  int num_encoder_layers;
  int num_temporal_layers;
  int num_depth_layers;
  int max_encoder_length;
  int rvq_depth;
  int temporal_num_buckets;
  int temporal_max_distance;
  int depth_num_buckets;
  int depth_max_distance;
  int codebook_size;  /* codec_rvq_codebook_size (system.h:51) */
  int codec_offset;   /* vocab_codec_offset = PAD + MASK (system.h:76) */
  int max_frames;     /* temporal self-KV capacity = chunk_length_frames (system.h:62-64) */
  int dtype;          /* MRTDF_DTYPE_FP32 or MRTDF_DTYPE_BF16 */
} mrtdf_config;

/*
 * Options of one generate_tokens call. Mirrors GenerateOptions
 * (depthformer/decode.h:48-57). The reference seeds MLX's RNG once per chunk
 * (decode.cpp:246-248); this engine draws its uniforms from Philox4x32-10
 * keyed by `seed`, counter = (vocab index / 4, frame * rvq_depth + level), so
 * two runs with the same seed give the same tokens. `use_vocab_masks` = 1
 * applies the per-level codec ranges that System::build_vocab_masks builds
 * (system.cpp:135-157). `uniforms`, when not NULL, replaces the RNG with
 * caller-given draws: num_frames * rvq_depth * vocab_size floats in (0, 1),
 * one row of vocab_size per (frame, level) step.
 */
typedef struct mrtdf_gen_opts {
  int num_frames;
  int rvq_depth;
  float temperature;
  int top_k;
  float guidance_weight;
  int use_vocab_masks;
  uint64_t seed;
  const float* uniforms;
} mrtdf_gen_opts;

typedef struct mrtdf_engine mrtdf_engine;
typedef struct mrtdf_stream mrtdf_stream;

/* Thread-local text of the last error; never NULL. */
const char* mrtdf_last_error(void);

/* Library version string, e.g. "mrtdf 0.1.0 sm_100a". */
const char* mrtdf_version(void);

/*
 * Fill `out` with a named preset: "base" (DepthformerConfig::base(),
 * model.cpp:34-36), "large" (model.cpp:38-48), "hybrid" (d_model 1024, 16x64
 * heads, d_ff 2816, layers 12/20/4, temporal buckets 32/128, vocab 16388) or
 * "tiny" (a small test model). dtype defaults to bf16.
 */
int mrtdf_config_preset(const char* name, mrtdf_config* out);

/*
 * Write a random-init weight bundle with the reference's key names and
 * (out, in) Linear layout (model.cpp:82-109, 173-198; modules.cpp:47-54) as
 * float32 safetensors. Matrices and tables are N(0, stddev) from Philox
 * keyed by `seed`; RMSNorm scales are 1.0 when `norm_ones` != 0, otherwise
 * N(0, stddev) too. The reference has no generator (weights.cpp:29-35 only
 * loads), so this defines one.
 */
int mrtdf_write_random_safetensors(const mrtdf_config* cfg, uint64_t seed, float stddev,
                                   int norm_ones, const char* path);

/* Replaces Depthformer::Depthformer(bundle, config, dtype) (model.h:74-75). */
int mrtdf_create(const mrtdf_config* cfg, int device, mrtdf_engine** out);
int mrtdf_destroy(mrtdf_engine* eng);

/* Load weights from a safetensors bundle: WeightBundle (weights.cpp:29-35)
 * plus load_param's cast to the compute dtype (modules.cpp:47-54). */
int mrtdf_load_safetensors(mrtdf_engine* eng, const char* path);

/* Generate the same weights as mrtdf_write_random_safetensors in memory and
 * upload them, without a file. */
int mrtdf_load_random(mrtdf_engine* eng, uint64_t seed, float stddev, int norm_ones);

/*
 * A decoding stream: `num_sequences` independent sequences, each one CFG pair
 * (2 rows, cond + uncond) when `cfg` != 0, else 1 row. Owns the KV arena
 * (empty_temporal_cache / empty_depth_cache, model.h:103-104; LayerCache,
 * model.h:70): temporal self K/V at max_frames, cross K/V at
 * max_encoder_length, depth self K/V at rvq_depth, all (rows, H, T, d_kv).
 */
int mrtdf_stream_create(mrtdf_engine* eng, int num_sequences, int cfg, mrtdf_stream** out);
int mrtdf_stream_destroy(mrtdf_stream* st);
/* Rows per step of this stream (num_sequences * (cfg ? 2 : 1)). */
int mrtdf_stream_rows(const mrtdf_stream* st);

/*
 * Depthformer::encode (model.h:81, model.cpp:226-241). `ids` is
 * (rows, seq_len) int32. Also projects the cross-attention K/V of every
 * temporal layer (modules.cpp:258-276, 323-333), which the reference does
 * on frame 0 of temporal_step; this resets the temporal cache. `enc_out`,
 * if not NULL, receives (rows, seq_len, d_model) float32.
 */
int mrtdf_encode(mrtdf_stream* st, const int32_t* ids, int seq_len, float* enc_out);

/*
 * Depthformer::temporal_step (model.h:113-117, model.cpp:322-514, eager
 * semantics). `x` is (rows, d_model) float32, rounded to the compute dtype
 * on upload; NULL means token_embedding(PAD=0) as on frame 0
 * (decode.cpp:366-368). Appends to the temporal self-KV at position
 * `frame_idx`, which must equal the number of frames already decoded
 * (frame 0 resets). `out` receives the stack output (rows, d_model) with no
 * final norm.
 */
int mrtdf_temporal_step(mrtdf_stream* st, const float* x, int frame_idx, float* out);

/*
 * Depthformer::depth_step (model.h:121-124, model.cpp:516-659). `x` is
 * (rows, d_model) float32; NULL means the last temporal_step output
 * (decode.cpp:455). depth_idx 0 resets the depth cache (decode.cpp:454).
 * `logits` receives (rows, vocab_size) float32.
 */
int mrtdf_depth_step(mrtdf_stream* st, const float* x, int depth_idx, float* logits);

/* token_embedding()(ids) (model.h:127; modules.cpp:110-112): n rows of d_model. */
int mrtdf_token_embedding(mrtdf_engine* eng, const int32_t* ids, int n, float* out);

/*
 * cfg_combine + apply_vocab_mask + sample_with_temperature
 * (decode.cpp:71-148, 465-474) on the device for one step. `logits` is
 * (cfg ? 2 : 1, vocab_size); `level` selects the vocab mask when
 * opts->use_vocab_masks; `uniforms` (vocab_size floats in (0, 1)) replaces
 * the Philox draws when not NULL, otherwise the draws for (frame, level)
 * of opts->seed are used. MRTDF_ERR_INVALID when no candidate can be drawn
 * (NaN logits, an empty range); `token` is then -1.
 */
int mrtdf_sample(mrtdf_engine* eng, const float* logits, int cfg, int frame, int level,
                 const mrtdf_gen_opts* opts, const float* uniforms, int32_t* token);

/*
 * mrtdf_sample for callers that cannot allocate GPU memory. No counterpart
 * in the reference: it exists for hosts that must not call cudaMalloc /
 * cudaFree on their decode thread - a real-time audio callback, where the
 * implicit device synchronisation and unbounded latency of an allocation
 * would glitch playback, or an embedding application that reserves all GPU
 * memory up front and forbids allocations afterwards.
 *
 * Same semantics and result as mrtdf_sample, but `logits_dev` ((cfg ? 2 : 1)
 * x vocab_size float32), `uniforms_dev` (vocab_size floats, or NULL for the
 * Philox draws of opts->seed) and `token_dev` (one int32) are DEVICE
 * pointers owned by the caller, the work is queued on `stream` (a
 * cudaStream_t, NULL = the legacy default stream) and the call does not
 * wait for it: it queues one kernel launch and nothing else (the seed
 * travels by value). Because the call returns before the draw, a draw that
 * fails (NaN logits, an empty range) is reported in the result: the kernel
 * stores -1 in *token_dev. The sampler's scratch is a fixed 64 KiB device
 * array inside the library, held by every GPU that loads it until the
 * process exits: rows x d_model x dtype bytes must be <= 21,760
 * (MRTDF_ERR_RANGE otherwise); nothing in it needs to start at zero, each
 * call writes what its kernel reads. The first call on a device looks up
 * that array's address; make it before any stream capture. All calls on a
 * device share the scratch, so calls that may overlap on the GPU race;
 * serialise them (one stream). Allocates nothing: no cudaMalloc, cudaFree
 * or allocating library routine.
 */
int mrtdf_sample_noalloc(mrtdf_engine* eng, const float* logits_dev, int cfg, int frame, int level,
                         const mrtdf_gen_opts* opts, const float* uniforms_dev, int32_t* token_dev, void* stream);

/*
 * generate_tokens (decode.h:112-119, decode.cpp:239-573; non-speculative
 * path): encode + num_frames x (temporal_step + rvq_depth x (depth_step +
 * sample)) entirely on the device. `enc_ids` is (rows, seq_len) int32;
 * `out_ids` receives (num_sequences, num_frames, rvq_depth) int32 LLM ids.
 * `seeds` holds one seed per sequence (NULL: opts->seed + sequence index).
 * The whole chunk runs as one CUDA graph, captured on first use.
 */
int mrtdf_generate_tokens(mrtdf_stream* st, const int32_t* enc_ids, int seq_len,
                          const mrtdf_gen_opts* opts, const uint64_t* seeds, int32_t* out_ids);

/* Same with device-resident ids in and out; runs on the stream's CUDA stream
 * and does not synchronize. */
int mrtdf_generate_tokens_dev(mrtdf_stream* st, const int32_t* enc_ids_dev, int seq_len,
                              const mrtdf_gen_opts* opts, const uint64_t* seeds,
                              int32_t* out_ids_dev);

/*
 * Teacher-forced decode: the generate_tokens loop with the sampled token of
 * (frame f, level l) replaced by tokens[f * rvq_depth + l], returning every
 * depth step's logits: (num_frames, rvq_depth, rows, vocab_size) float32.
 * Single-sequence streams only.
 */
int mrtdf_teacher_forced_logits(mrtdf_stream* st, const int32_t* enc_ids, int seq_len,
                                const int32_t* tokens, int num_frames, float* logits);

/* Wait for all work queued on the stream; returns MRTDF_ERR_TIMEOUT if a
 * device-side bounded wait gave up since the last call. */
int mrtdf_stream_sync(mrtdf_stream* st);

/* The stream's cudaStream_t, for callers that order their own work on it. */
void* mrtdf_stream_cuda(mrtdf_stream* st);

/*
 * Failure-detection check (no counterpart in the reference): queue on the
 * stream one CTA that waits on an mbarrier which no thread and no copy ever
 * completes, bounded by `timeout_us` microseconds of the GPU's global timer
 * (1 .. 1,000,000; every production wait uses the same routine with a
 * 0.5 s bound). The wait gives up, sets the timeout bit of the stream's error
 * word and the call returns MRTDF_ERR_TIMEOUT, as every call does after a
 * device-side wait gave up; the error word is cleared and the stream stays
 * usable.
 */
int mrtdf_check_wait_timeout(mrtdf_stream* st, int timeout_us);

/*
 * Measurement hook (no reference counterpart): replay, as one CUDA graph on
 * the stream, only the weight-streaming decode launches of one
 * generate_tokens chunk with options `opts` (same buffers and parameters as
 * the real chunk; encoder and sampler left out) of the stacks in
 * `stack_mask` (bit 0: the temporal layers, bit 1: the depth layers and
 * lm_head), `reps` times between two CUDA events. Returns the milliseconds
 * per replay, the launches per replay and their algorithmic bytes (weights,
 * attention K/V reads, input and output vectors). The stream must have run
 * a chunk or an encode before.
 */
int mrtdf_bench_phases(mrtdf_stream* st, const mrtdf_gen_opts* opts, int stack_mask, int reps, float* ms_per_rep,
                       long long* launches_per_rep, double* bytes_per_rep);

/*
 * Measurement hook (no reference counterpart): read a `bytes` device buffer
 * (rounded down to a multiple of 16 MiB) `reps` times with 16-byte loads
 * spread over every SM, after one untimed pass; a buffer well under the L2
 * size stays L2-resident, so this is the L2 read bandwidth the depth stack
 * can reach. Reports GB/s (bytes read / CUDA-event time).
 */
int mrtdf_bench_l2_read(mrtdf_engine* eng, size_t bytes, int reps, double* gbs);

/*
 * Measurement hook (no counterpart in the reference): the encoder pass
 * (embed + PE, encoder layers, encoder_norm, cross-K/V projection of every
 * temporal layer) for `rows` sequences of `seq_len` uniform-random ids
 * (seed 2), captured as one CUDA graph and replayed `reps` times on a
 * private stream. Reports ms per pass and the pass's algorithmic FLOPs
 * (2 per multiply-add: linears, attention, cross-K/V). Allocates its own
 * workspace (rows x seq_len activations + the cross-K/V cache) for the call.
 */
int mrtdf_bench_encoder(mrtdf_engine* eng, int rows, int seq_len, int reps, float* ms_per_rep,
                        double* flops_per_rep);

/*
 * Measurement hook (no counterpart in the reference): `frames` x rvq_depth
 * sequential depth steps (depth stack + decoder_norm + lm_head level slice
 * + sampler with embedding feedback), each frame starting from an N(0, 1)
 * temporal hidden state (seed 3) instead of a temporal step, captured as one
 * graph and replayed `reps` times on the stream. Reports us per depth step,
 * its algorithmic bytes (GEMV weights, inputs, outputs and the depth K/V
 * reads) and kernel launches per step. Overwrites the stream's depth cache,
 * token and feedback buffers.
 */
int mrtdf_bench_depth(mrtdf_stream* st, const mrtdf_gen_opts* opts, int frames, int reps, float* us_per_step,
                      double* bytes_per_step, long long* launches_per_step);

/*
 * Measurement hook (no counterpart in the reference): kernel nodes of the
 * CUDA graph of the chunk this stream ran last (every one is a kernel of this
 * library), or -1 when that chunk ran as stream launches (MRTDF_GRAPH=0).
 */
long long mrtdf_stream_chunk_kernels(const mrtdf_stream* st);

/* ---- single-layer probes ----------------------------------------------------
 * No counterpart in the reference: each runs ONE step of the production
 * launch sequence (the same kernels, launch shapes and epilogues as a chunk)
 * on caller-given float32 inputs, rounded to the compute dtype on upload, so
 * a CPU restatement can be checked layer by layer on identical inputs. They
 * use and overwrite the stream's activation and cache buffers.
 */

/* EncoderLayer `layer` (modules.cpp:349-358) over x (rows, seq_len,
 * d_model) -> out, same shape. */
int mrtdf_probe_encoder_layer(mrtdf_stream* st, int layer, const float* x, int seq_len, float* out);

/* Overwrite positions [0, len) of one layer's cache with (rows, H, len,
 * d_kv) float32 k / v: kind 0 = temporal self-attention, 1 = depth
 * self-attention, 2 = cross-attention (len = the encoder length the
 * temporal layers then attend over). */
int mrtdf_probe_set_cache(mrtdf_stream* st, int kind, int layer, const float* k, const float* v, int len);

/* DecoderLayer::forward (modules.cpp:384-446) of the temporal (stack 0) or
 * depth (stack 1) stack at cache position `pos`: x (rows, d_model) -> out;
 * the step's k / v are appended to the layer's cache at `pos`. */
int mrtdf_probe_decoder_layer(mrtdf_stream* st, int stack, int layer, int pos, const float* x, float* out);

/* decoder_norm + lm_head (model.cpp:653-658) of x (rows, d_model): the
 * codebook rows of RVQ level `level` (rows x codebook_size logits), or all
 * vocab_size rows when level < 0. */
int mrtdf_probe_lm_head(mrtdf_stream* st, int level, const float* x, float* logits);

/* ---- streaming glue (System, system.cpp) ---------------------------------- */

/*
 * The System::generate_chunk loop (system.cpp:177-333) for `num_chunks`
 * consecutive chunks without returning to the host: per chunk, encoder ids
 * from the context (build_encoder_inputs_host, system.cpp:62-95), the chunk
 * (generate_tokens), tokens -> RVQ codes (llm_to_rvq, rvq.cpp:112-134) and
 * the context roll (system.cpp:320-333), all on the stream.
 * context_dev: (num_sequences, ctx_frames, rvq_depth) int32 RVQ codes,
 * negative = empty, rolled in place; style_dev: (num_sequences,
 * style_depth) int32 LLM ids; rvq_out_dev: (num_chunks, num_sequences,
 * num_frames, rvq_depth) int32 codes. seeds: host (num_chunks *
 * num_sequences) or NULL (opts->seed + chunk, + i << 32 for sequence i).
 * Returns once the work is queued; mrtdf_stream_sync waits and reports
 * device errors (a token outside its level's range: MRTDF_ERR_INVALID).
 */
int mrtdf_generate_stream_dev(mrtdf_stream* st, int32_t* context_dev, int ctx_frames, int enc_depth,
                              const int32_t* style_dev, int style_depth, int num_chunks,
                              const mrtdf_gen_opts* opts, const uint64_t* seeds, int32_t* rvq_out_dev);

/*
 * build_encoder_inputs_host (system.cpp:62-95): context (ctx_frames,
 * rvq_depth) int32 RVQ codes (negative = empty) + style ids ->
 * (2, ctx_frames * enc_depth + style_depth) int32. Row 0 = codec context
 * levels < enc_depth mapped to codec_offset + d * codebook + v (MASK=1 when
 * v < 0) then the style ids; row 1 = same context, style masked.
 */
int mrtdf_build_encoder_inputs(const int32_t* context, int ctx_frames, int rvq_depth,
                               int enc_depth, const int32_t* style, int style_depth,
                               int codebook_size, int codec_offset, int32_t* out);

/* Context roll (system.cpp:320-333): shift left by chunk_frames frames and
 * append new RVQ codes (chunk_frames, rvq_depth). In place. */
int mrtdf_context_roll(int32_t* context, int ctx_frames, int rvq_depth, const int32_t* new_codes,
                       int chunk_frames);

/* llm_to_rvq with safe=true (rvq.cpp:112-134): (n, rvq_depth) LLM ids ->
 * RVQ codes; MRTDF_ERR_INVALID when an id is not in its level's range. */
int mrtdf_llm_to_rvq(const int32_t* llm, int n, int rvq_depth, int codebook_size,
                     int codec_offset, int32_t* out);

/* rvq_to_llm (rvq.cpp:105-110). */
int mrtdf_rvq_to_llm(const int32_t* rvq, int n, int rvq_depth, int codebook_size,
                     int codec_offset, int32_t* out);

/* Paths of the C++ inference bundle under one cache root (InferenceBundlePaths,
 * weights.h:70-78). Each is a NUL-terminated path of at most MRTDF_PATH_MAX - 1 bytes. */
#define MRTDF_PATH_MAX 4096
typedef struct mrtdf_bundle_paths {
  char spectrostream_encoder[MRTDF_PATH_MAX];
  char spectrostream_decoder[MRTDF_PATH_MAX];
  char spectrostream_codebooks[MRTDF_PATH_MAX];
  char musiccoca_encoder[MRTDF_PATH_MAX];
  char musiccoca_codebooks[MRTDF_PATH_MAX];
  char musiccoca_vocab[MRTDF_PATH_MAX];
  char depthformer[MRTDF_PATH_MAX]; /* <root>/depthformer/depthformer_<tag>.safetensors */
} mrtdf_bundle_paths;

/* resolve_inference_bundle (weights.cpp:72-120): the bundle's file paths
 * under `cache_root` for the Depthformer checkpoint `tag` ("base", "large").
 * A root that is not a directory, or any of the seven files missing, is
 * MRTDF_ERR_IO (std::runtime_error in the reference) with the reference's
 * message (the missing files listed one per line). A path longer than
 * MRTDF_PATH_MAX - 1 bytes is MRTDF_ERR_RANGE. No GPU is needed. */
int mrtdf_resolve_inference_bundle(const char* cache_root, const char* tag, mrtdf_bundle_paths* out);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* MRTDF_H_ */
