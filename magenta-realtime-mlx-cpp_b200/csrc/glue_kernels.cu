// Streaming glue on the device, so consecutive chunks of a stream never
// return to the host: encoder ids from the RVQ context, and the chunk's
// tokens -> RVQ codes -> context roll.
//
// Reference (rhymeswithlion/magenta-realtime-mlx-cpp):
//   build_encoder_inputs_host  src/magenta_realtime_mlx/system.cpp:62-95
//   context roll               system.cpp:320-333
//   llm_to_rvq (safe)          src/magenta_realtime_mlx/rvq.cpp:112-134
// Integer work, a few KB per chunk: one CTA per sequence.
#include "common.cuh"
#include "glue_kernels.cuh"

namespace mrtdf {

namespace {
constexpr int kMaskToken = 1;  // SystemConfig::vocab_mask_token (system.h:75)
}

// Row 2s (cond): context levels < enc_depth -> codec_offset + d * codebook +
// v (MASK when v < 0), then the sequence's style ids. Row 2s + 1 (uncond,
// with CFG): the same context, style masked.
__global__ void stream_encoder_ids_kernel(const GlueParams p) {
  const int s = blockIdx.x;
  const int n_ctx = p.ctx_frames * p.enc_depth;
  const int S = n_ctx + p.style_depth;
  const int32_t* ctx = p.context + (size_t)s * p.ctx_frames * p.rvq_depth;
  int32_t* row0 = p.ids + (size_t)s * p.rows_per_seq * S;
  for (int i = threadIdx.x; i < S; i += blockDim.x) {
    int32_t id;
    if (i < n_ctx) {
      const int f = i / p.enc_depth, d = i - f * p.enc_depth;
      const int32_t v = ctx[(size_t)f * p.rvq_depth + d];
      id = v >= 0 ? p.codec_offset + d * p.codebook_size + v : kMaskToken;
    } else {
      id = p.style[(size_t)s * p.style_depth + (i - n_ctx)];
    }
    row0[i] = id;
    if (p.rows_per_seq == 2) row0[S + i] = i < n_ctx ? id : kMaskToken;
  }
}

// tokens (nseq, tok_stride) of the chunk -> RVQ codes (level check as
// llm_to_rvq with safe = true; a mismatch sets kErrBadToken and writes 0),
// written to rvq_out (nseq, frames, rvq_depth); then the context of the
// sequence shifts left by `frames` frames and the new codes fill its tail.
__global__ void stream_roll_kernel(const GlueParams p) {
  extern __shared__ int32_t keep_sm[];
  const int s = blockIdx.x;
  const int D = p.rvq_depth, F = p.frames;
  const int keep = (p.ctx_frames - F) * D;
  int32_t* ctx = p.context + (size_t)s * p.ctx_frames * D;
  for (int i = threadIdx.x; i < keep; i += blockDim.x) keep_sm[i] = ctx[(size_t)F * D + i];
  __syncthreads();
  for (int i = threadIdx.x; i < keep; i += blockDim.x) ctx[i] = keep_sm[i];
  for (int i = threadIdx.x; i < F * D; i += blockDim.x) {
    const int d = i % D;
    const int32_t shifted = p.tokens[(size_t)s * p.tok_stride + i] - p.codec_offset;
    int32_t r = shifted % p.codebook_size;  // remainder with the divisor's sign (mx::remainder)
    if (r < 0) r += p.codebook_size;
    if (shifted - r != d * p.codebook_size) {
      atomicOr(p.err, kErrBadToken);
      r = 0;
    }
    p.rvq_out[(size_t)s * F * D + i] = r;
    ctx[keep + i] = r;
  }
}

size_t glue_roll_smem(const GlueParams& p) { return (size_t)(p.ctx_frames - p.frames) * p.rvq_depth * 4; }

cudaError_t launch_stream_encoder_ids(const GlueParams& p, cudaStream_t s) {
  stream_encoder_ids_kernel<<<p.nseq, 256, 0, s>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_stream_roll(const GlueParams& p, cudaStream_t s) {
  const size_t smem = glue_roll_smem(p);
  if (smem > kGlueMaxSmem) return cudaErrorInvalidValue;
  stream_roll_kernel<<<p.nseq, 256, smem, s>>>(p);
  return cudaGetLastError();
}

}  // namespace mrtdf
