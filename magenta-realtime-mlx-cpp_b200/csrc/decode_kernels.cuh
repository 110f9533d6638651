// Parameter blocks and launch entry points of the decode-step kernels
// (temporal_step / depth_step / sampler). Host code fills these structs;
// every pointer is device memory.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace mrtdf {

// Epilogues of the GEMV phase kernel.
enum GemvMode : int {
  kGemvStore = 0,   // out[b, off + u] = R(acc)
  kGemvResid = 1,   // out[b, u] = R(resid[b, u] + R(acc))      (residual add)
  kGemvQKV = 2,     // fused q/k/v: q -> out, k/v -> cache at `pos`
  kGemvGeglu = 3,   // unit = (wi_0 row, wi_1 row): out[b, u] = R(gelu(R(a)) * R(b))
  kGemvLogits = 4,  // float out[b, off + u] = R(acc)
  kGemvQKVCluster = 6,  // kGemvQKV on one thread-block cluster per head; the
                        // head's attention runs inside the cluster (bf16 only)
};
// q/k/v weight rows of a decoder layer are head-major: row h * 192 + s * 64
// + c is output c of head h in section s (0 = q, 1 = k, 2 = v).
constexpr int kQkvRowsPerHead = 192;
constexpr int kQkvCluster = 8;  // CTAs per head in kGemvQKVCluster (24 rows each)

struct GemvParams {
  const void* W;       // weight rows, (units * rows_per_unit, cols), row-major
  const void* x;       // input activations (B, x_stride)
  const void* norm_w;  // RMSNorm scale (cols), or null for a plain input
  void* out;
  const void* resid;
  void* kc;
  void* vc;
  int* err;
  // bf16 only, B <= 2: when not null, x = R(x + R(acc / 2^32)) per element
  // (a hidden state left by the fused decode phases; x is its residual)
  const long long* acc;
  int units;
  int cols;
  int B;
  int x_stride, out_stride, resid_stride;
  int out_offset;
  int inner, H, cap, pos;  // kGemvQKV
  int l2_keep;             // 1: keep these weights in L2 (evict_last), 0: stream them (evict_first)
  // kGemvQKVCluster: relative-position bias of this query (H, bias_stride)
  // or null, attention output (B, inner)
  const float* bias;
  int bias_stride;
  void* attn_out;
};

// Bytes of one TMA stage of the GEMV kernel and the number of stages.
constexpr int kGemvStageBytes = 24576;
constexpr int kGemvStages = 3;
constexpr int kGemvThreads = 256;
constexpr int kGemvMaxB = 8;
// Rows per step of a bf16 stream; above kGemvMaxB the projections run as
// RMSNorm + tcgen05 GEMM with the batch rows as M (one 128-row tile).
constexpr int kWideMaxRows = 128;

size_t gemv_smem_bytes(int B, int cols);
// Launch the GEMV phase. dtype 1 (bf16) runs the tensor-core kernel over
// enough CTAs (at least num_sms when there are that many units) that each
// CTA's rows fit in shared memory; dtype 0 (fp32) runs the CUDA-core kernel
// over min(units, num_sms) CTAs.
cudaError_t launch_gemv(int dtype, int mode, bool norm, const GemvParams& p, int num_sms, cudaStream_t s, bool pdl);
cudaError_t gemv_set_smem_limits();

struct AttnParams {
  const void* q;    // (B, inner)
  const void* K;    // (B, H, cap, 64)
  const void* V;
  const float* bias;  // (H, bias_stride) for this query position, or null
  int bias_stride;
  void* out;        // (B, inner)
  int* err;
  int B, H, cap, T;  // T = number of valid keys
  int inner;
  int nsplit;  // cross attention: key slices = CTAs of one cluster (1, 2, 4 or kCrossSplit)
};
cudaError_t launch_attn_self(int dtype, const AttnParams& p, cudaStream_t s, bool pdl);
cudaError_t launch_attn_cross(int dtype, const AttnParams& p, cudaStream_t s, bool pdl);
constexpr int kCrossSplit = 8;

struct SampleParams {
  const float* logits;  // (B, logits_stride); column c holds vocab id col_offset + c
  int logits_stride;
  int col_offset;
  int lo, hi;            // candidate vocab range
  int rows_per_seq;      // 2 with CFG, else 1
  float w, temperature;
  int top_k;
  const uint64_t* seeds;  // per sequence, or null: every sequence uses seed_value
  uint64_t seed_value;
  uint32_t step;          // frame * rvq_depth + level
  const float* uniforms;  // optional draws: this step's row of V for sequence 0
  long long uni_seq_stride;  // floats between the rows of consecutive sequences
  const int32_t* forced;  // optional forced token per sequence (teacher forcing)
  int32_t* tokens;        // tokens[seq * tok_stride + tok_index]
  int tok_stride, tok_index;
  const void* emb;        // (V, d)
  int d, V;
  void* din;              // (B, d) next depth input
  void* fsum;             // (B, d) running embedding sum of the frame
  void* tin;              // (B, d) next temporal input (written on the last level)
  int depth;
  int is_first, is_last;
  // When no candidate can be chosen (every candidate NaN or -inf, an empty
  // range) or a forced id is outside [0, V): the kErrBadToken bit goes to
  // *err (when err is not null), `bad_token` is stored as the token and id 0
  // feeds the embedding rows.
  int bad_token;
  int* err;
};
cudaError_t launch_sample(int dtype, const SampleParams& p, int num_seq, cudaStream_t s, bool pdl);
size_t sample_smem_bytes(int n_candidates);
cudaError_t sample_set_smem_limits();
constexpr int kSampleMaxSmem = 160 * 1024;

// Fixed device scratch of the allocation-free sampler: a 256-byte header
// (reserved) then three feedback rows of up to kSampleScratchRowBytes each.
constexpr size_t kSampleScratchBytes = 64 * 1024;
constexpr size_t kSampleScratchRowBytes = (kSampleScratchBytes - 256) / 3 / 256 * 256;
// Device address of that scratch on `device` (looked up once per device).
cudaError_t sample_scratch_address(int device, void** out);

// Read `bytes` (a multiple of 16 MiB) of `buf` once with 16-byte loads over
// 4 CTAs per SM; `sink` (4096 words) receives one word per CTA.
cudaError_t launch_l2_read(const void* buf, size_t bytes, unsigned* sink, int num_sms, cudaStream_t s);

// One CTA waiting on an mbarrier that nothing completes, bounded by
// timeout_ns: sets kErrMbarTimeout in *err (failure-detection check).
cudaError_t launch_wait_timeout_probe(int* err, unsigned long long timeout_ns, cudaStream_t s);

// out[r, :] = emb[ids[r], :] for r < rows (ids == null: id 0 = PAD).
cudaError_t launch_embed_rows(int dtype, const void* emb, const int32_t* ids, int rows, int d, void* out,
                              cudaStream_t s, bool pdl);
// out[r, :] = from_f(src_f32[r, :]) (host-provided inputs already on device).
cudaError_t launch_f32_to_act(int dtype, const float* src, size_t n, void* out, cudaStream_t s);
cudaError_t launch_act_to_f32(int dtype, const void* src, size_t n, float* out, cudaStream_t s);

}  // namespace mrtdf
