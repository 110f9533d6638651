/*
 * mrtmc.h - C ABI of the B200 style path: the MusicCoCa text tower
 * (prompt token ids -> 768-d style embedding) and the residual vector
 * quantisation of that embedding into style tokens.
 *
 * Drop-in for the style block of System (rhymeswithlion/magenta-realtime-mlx-cpp,
 * src/magenta_realtime_mlx/system.cpp:110-124 and 158-161, style_model.cpp):
 * MusicCoCaEncoder::embed_text (musiccoca.h:173-174, musiccoca.cpp:272-295),
 * rvq_quantization (rvq.cpp:24-66) as StyleModel::tokenize
 * (style_model.h:61-63) and StyleModel::style_tokens_lm (style_model.h:65-71,
 * style_model.cpp:111-122). The SentencePiece step of
 * StyleModel::tokenize_text_ids stays with the caller: these entry points take
 * its output, the (B, L) token ids and the padding mask (1.0 = padding).
 * The reference runs MusicCoCa in float32 (system.cpp:116-124); so does this
 * path (float32 CUDA-core GEMMs and float32 attention).
 *
 * Conventions are those of mrtdf.h (same library, same status codes,
 * message from mrtdf_last_error()): host pointers, int status, 0 = MRTDF_OK.
 * A handle may be used by one host thread at a time.
 */
#ifndef MRTMC_H_
#define MRTMC_H_

#include <stddef.h>
#include <stdint.h>

#include "mrtdf.h"

#ifdef __cplusplus
extern "C" {
#endif

#define MRTMC_EMBED_DIM 768    /* MusicCoCaConfig::d_model (musiccoca.h:151-162) */
#define MRTMC_MAX_TEXT_LEN 128 /* MusicCoCaConfig::max_text_len, StyleModel::kMaxTextLength */
#define MRTMC_RVQ_DEPTH 12     /* StyleModel::kRVQDepth (style_model.h:42) */

typedef struct mrtmc_model mrtmc_model;

/* Device buffers for up to max_batch (1 .. 64) prompts of up to
 * MRTMC_MAX_TEXT_LEN tokens per call. Replaces MusicCoCaEncoder's and StyleModel's constructors
 * (musiccoca.h:166-168, style_model.h:49-52) together with the load below. */
int mrtmc_create(int device, int max_batch, mrtmc_model** out);
void mrtmc_destroy(mrtmc_model* model);

/* musiccoca_encoder.safetensors (the text tower's keys: token_embedding,
 * text_layers.{0..11}, text_exit_ln, text_pooler) and the codebook bundle's
 * "codebooks" (K, C, 768) (system.cpp:110-113, style_model.cpp). F32 or BF16
 * tensors. Missing key -> MRTDF_ERR_KEY; wrong shape -> MRTDF_ERR_INVALID. */
int mrtmc_load_safetensors(mrtmc_model* model, const char* encoder_path, const char* codebooks_path);

/* MusicCoCaEncoder::embed_text (musiccoca.cpp:272-295): ids (B, L) int32,
 * pad (B, L) float (1.0 = padding) -> out (B, 768) float32. B <= max_batch,
 * 1 <= L <= 128 (else MRTDF_ERR_RANGE); an id outside [0, vocab) is
 * MRTDF_ERR_RANGE. */
int mrtmc_embed_text(mrtmc_model* model, const int32_t* ids, const float* pad, int B, int L, float* out);

/* rvq_quantization (rvq.cpp:24-66) with the first `levels` codebooks
 * (StyleModel::tokenize uses 12): emb (N, 768) -> tokens (N, levels) int32;
 * per level the first codeword of least |r|^2 - 2 r.c + |c|^2, then r -= c.
 * 1 <= N <= 1024; levels <= K. */
int mrtmc_quantize(mrtmc_model* model, const float* emb, int N, int levels, int32_t* tokens);

/* StyleModel::style_tokens_lm (style_model.cpp:111-122) after tokenisation:
 * embed_text -> the first encoder_style_rvq_depth RVQ levels -> rvq_to_llm
 * (vocab_style_offset + level * style_rvq_codebook_size + token). ids / pad
 * (B, L) -> out (B, encoder_style_rvq_depth) int32. */
int mrtmc_style_tokens(mrtmc_model* model, const int32_t* ids, const float* pad, int B, int L,
                       int encoder_style_rvq_depth, int style_rvq_codebook_size, int vocab_style_offset,
                       int32_t* out);

/* The model's cudaStream_t (for events around the calls above). */
void* mrtmc_cuda_stream(mrtmc_model* model);
/* Kernel launches of one mrtmc_embed_text call at (B, L). No reference
 * counterpart (measurement hook). */
long long mrtmc_embed_kernels(mrtmc_model* model, int B, int L);

#ifdef __cplusplus
}
#endif

#endif /* MRTMC_H_ */
