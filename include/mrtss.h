/*
 * mrtss.h - C ABI of the B200 SpectroStream decode phase (RVQ codes ->
 * decoder -> iSTFT -> stereo samples), the codec half of a chunk after the
 * Depthformer has produced its RVQ codes.
 *
 * Drop-in for the codec block of System::generate_chunk
 * (rhymeswithlion/magenta-realtime-mlx-cpp, src/magenta_realtime_mlx/
 * system.cpp:372-390): rvq_dequantization (rvq.cpp:68-87),
 * SpectroStreamDecoder (spectrostream.h:169-197, spectrostream.cpp:356-419)
 * and istft_postprocess (spectrostream.h:231-235, spectrostream.cpp:593-681).
 * The reference runs this decoder in float32 (system.cpp:118-119); this one
 * keeps float32 activations and computes the convolutions on the tensor
 * cores with tf32 operands and float32 accumulation.
 *
 * Conventions are those of mrtdf.h (same library, same status codes,
 * message from mrtdf_last_error()): host pointers unless the name ends in
 * `_dev`, int status, 0 = MRTDF_OK. A handle may be used by one host thread
 * at a time.
 */
#ifndef MRTSS_H_
#define MRTSS_H_

#include <stddef.h>
#include <stdint.h>

#include "mrtdf.h"

#ifdef __cplusplus
extern "C" {
#endif

#define MRTSS_EMBED_DIM 256      /* SpectroStreamDecoder::kEmbeddingDim (spectrostream.h:199) */
#define MRTSS_STFT_BINS 480      /* decoder output width = STFT bins without Nyquist */
#define MRTSS_FRAME_SAMPLES 1920 /* codec_sample_rate / codec_frame_rate (system.h:47-48) */

typedef struct mrtss_codec mrtss_codec;

/* Write a random-init decoder bundle with the reference's key layout and
 * canonical conv layouts (conv (O, I, kh, kw), transposed conv
 * (I, O, kh, kw); spectrostream.cpp:110-116) and a codebook bundle holding
 * "codebooks" (levels, 1024, 256). Weights N(0, 1 / fan_in), biases
 * N(0, 0.02^2), codebooks N(0, 0.25^2); Philox-keyed by seed. No reference
 * counterpart (the real bundles are downloaded; none is available here). */
int mrtss_write_random_safetensors(uint64_t seed, int levels, const char* decoder_path, const char* codebooks_path);

/* Device buffers for up to max_batch sequences of up to max_frames codec
 * frames per call. Replaces SpectroStreamDecoder's constructor
 * (spectrostream.cpp:356-363) together with the two load calls below. */
int mrtss_create(int device, int max_batch, int max_frames, mrtss_codec** out);
void mrtss_destroy(mrtss_codec* codec);

/* spectrostream_decoder.safetensors + the codebook bundle's "codebooks"
 * (K, C, D) (system.cpp:372-373). Missing key -> MRTDF_ERR_KEY. */
int mrtss_load_safetensors(mrtss_codec* codec, const char* decoder_path, const char* codebooks_path);
int mrtss_load_random(mrtss_codec* codec, uint64_t seed, int levels);

/* rvq_dequantization (rvq.cpp:68-87): codes (n, levels) -> (n, 256) float32,
 * summed over levels in order. A code outside [0, C) -> MRTDF_ERR_RANGE. */
int mrtss_rvq_dequantize(mrtss_codec* codec, const int32_t* codes, int n, int levels, float* out);

/* SpectroStreamDecoder::operator() (spectrostream.cpp:365-419):
 * embeddings (B, S, 256) -> spec (B, 4 S, 480, 4), channels
 * [left re, left im, right re, right im]. */
int mrtss_decode(mrtss_codec* codec, const float* embeddings, int B, int S, float* spec);

/* istft_postprocess (spectrostream.cpp:593-681): spec (B, frames, 480, 4)
 * -> audio (B, target, 2) interleaved; target <= (frames + 1) * 480. */
int mrtss_istft(mrtss_codec* codec, const float* spec, int B, int frames, int target, float* audio);

/* The codec block of System::generate_chunk (system.cpp:372-390) for B
 * sequences: codes (B, S, levels) -> audio (B, S * 1920, 2). One CUDA graph
 * per (B, S, levels). */
int mrtss_decode_tokens(mrtss_codec* codec, const int32_t* codes, int B, int S, int levels, float* audio);

/* The same on device buffers, enqueued on the codec's stream without a
 * synchronise (codes_dev (B, S, levels) int32, audio_dev (B, S * 1920, 2)
 * float32); a bad code sets the error that the next mrtss_sync reports. */
int mrtss_decode_tokens_dev(mrtss_codec* codec, const int32_t* codes_dev, int B, int S, int levels,
                            float* audio_dev);

/* Synchronise the codec's stream; reports device-side errors. */
int mrtss_sync(mrtss_codec* codec);
/* The codec's cudaStream_t (for events around mrtss_decode_tokens_dev). */
void* mrtss_cuda_stream(mrtss_codec* codec);
/* Kernel launches of one mrtss_decode_tokens(_dev) call at (B, S). No
 * reference counterpart (measurement hook). */
long long mrtss_decode_kernels(mrtss_codec* codec, int B, int S);

#ifdef __cplusplus
}
#endif

#endif /* MRTSS_H_ */
