// Device-side streaming glue (encoder ids from the RVQ context; tokens ->
// RVQ codes -> context roll). Every pointer is device memory.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace mrtdf {

struct GlueParams {
  int32_t* context;      // (nseq, ctx_frames, rvq_depth) RVQ codes, negative = empty
  const int32_t* style;  // (nseq, style_depth)
  int32_t* ids;          // (nseq * rows_per_seq, ctx_frames * enc_depth + style_depth)
  const int32_t* tokens; // chunk tokens, sequence s at tokens + s * tok_stride, (frames, rvq_depth)
  int32_t* rvq_out;      // (nseq, frames, rvq_depth)
  int* err;
  int nseq, rows_per_seq;
  int ctx_frames, rvq_depth, enc_depth, style_depth;
  int frames, tok_stride;
  int codebook_size, codec_offset;
};

constexpr size_t kGlueMaxSmem = 48 * 1024;  // kept context frames x rvq_depth x 4 bytes
size_t glue_roll_smem(const GlueParams& p);
cudaError_t launch_stream_encoder_ids(const GlueParams& p, cudaStream_t s);
cudaError_t launch_stream_roll(const GlueParams& p, cudaStream_t s);

}  // namespace mrtdf
