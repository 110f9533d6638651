// Fused decode phases (bf16, one CFG pair: at most 2 rows per step).
//
// A decoder layer of temporal_step / depth_step (DecoderLayer::forward,
// modules.cpp:384-446) runs as three launches in the temporal stack and two
// in the depth stack instead of one launch per projection:
//
//   self phase   pre-norm, q/k/v, self-attention with relative-position bias,
//                o_proj                    (one 8-CTA cluster per head)
//   cross phase  pre-norm, cross q, cross-attention over the encoder K/V,
//                cross o_proj              (one 8-CTA cluster per row x head)
//   ffn phase    pre-norm, wi_0 / wi_1, gated GELU, wo
//                                          (8-CTA clusters over the GPU)
//
// Each phase ends in a projection whose inputs are split across CTAs (the
// heads of o_proj, the d_ff units of wo). Every CTA adds its share of the
// fp32 outputs into an int64 accumulator (value x 2^32, rounded) with
// red.global.add: integer addition does not depend on the order in which
// the CTAs arrive, so the sum is the same on every run. The NEXT phase reads
// the accumulator while it loads its input and applies the reference's
// rounding there: x = R(residual + R(sum / 2^32)) (the o_proj / wo output
// rounded to bf16, then the rounded residual add, modules.cpp:401-408).
//
// The weight rows a CTA multiplies are one contiguous range of a padded
// copy (row stride d * 2 + 16 bytes, the shared-memory stride that keeps the
// ldmatrix reads conflict free), fetched with a single TMA bulk copy: issuing
// one bulk copy per row cost about 35 ns each.
//
// Three accumulators rotate: a phase reads one (acc), adds into the next
// (acc_out), and zeroes the third (acc_clear), which the phase before it
// read; kernels of a stream are serialised by their dependency waits, so a
// buffer is zero again two phases after its last reader.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace mrtdf {

constexpr int kFusedMaxRows = 2;   // one CFG pair
constexpr int kFusedCluster = 8;   // CTAs per cluster in every fused phase

// Input of a phase. x = `x` (bf16, rows x d) when acc is null, else
// x = R(x + R(acc / 2^32)) with `x` the residual stream.
struct FusedIn {
  const void* x;
  const long long* acc;
  void* x_out;           // x (bf16) is stored here for the next phase's residual when acc != null
  long long* acc_out;    // this phase's split sums (zero on entry)
  long long* acc_clear;  // zeroed by this phase, or null
  int* err;
  int B, d;
};

struct FusedSelfParams {
  FusedIn in;
  const void* wqkv;    // head-major q/k/v rows (H * 192, d), rows padded to d * 2 + 16 bytes
  const void* norm_w;  // pre_self_attn_norm (d)
  const void* wo_blk;  // o_proj blocked: [H][8][d / 8][64] = rows r*d/8 .. of W_o's columns of head h
  void* kc;            // self K/V caches (B, H, cap, 64)
  void* vc;
  const float* bias;   // relative-position bias of this query (H, bias_stride), or null
  int bias_stride;
  int H, cap, pos;
  int l2_keep;         // 1: keep the weights in L2 (evict_last), 0: stream them
};

struct FusedCrossParams {
  FusedIn in;
  const void* wcq;     // cross q_proj (H * 64, d), rows padded to d * 2 + 16 bytes
  const void* norm_w;  // pre_cross_attn_norm (d)
  const void* wco_blk; // cross o_proj blocked like wo_blk
  const void* ck;      // cross K/V caches (B, H, Smax, 64)
  const void* cv;
  int H, Smax, S;
  int l2_keep;
};

struct FusedFfnParams {
  FusedIn in;
  const void* wi;       // wi_0 / wi_1 rows interleaved (2 * ff, d), rows padded to d * 2 + 16 bytes
  const void* norm_w;   // pre_ffn_norm (d)
  const void* wout_blk; // wo blocked: [nclusters][8][d / 8][Uc], unit columns of cluster j (zero past ff)
  int ff, Uc, nclusters;
  int l2_keep;
};

// Layout of the FFN phase for a model: nclusters clusters of 8 CTAs, Uc
// d_ff units per cluster (a multiple of 32), Uc / 8 units per CTA.
struct FfnPlan {
  int nclusters = 0, Uc = 0;
};
// Chooses the plan for (d, ff) on the current device: as many clusters as
// can be resident at once (at most ceil(SMs / 8)).
cudaError_t fused_ffn_plan(int d, int ff, int num_sms, FfnPlan* out);

cudaError_t launch_fused_self(const FusedSelfParams& p, cudaStream_t s, bool pdl);
cudaError_t launch_fused_cross(const FusedCrossParams& p, cudaStream_t s, bool pdl);
cudaError_t launch_fused_ffn(const FusedFfnParams& p, cudaStream_t s, bool pdl);
// out = R(x + R(acc / 2^32)) (bf16, B x d): the hidden state after a phase,
// for the step-level entry points that return it.
cudaError_t launch_fused_materialize(const FusedIn& in, void* out, cudaStream_t s, bool pdl);
cudaError_t fused_set_smem_limits();

// Host-side check of a model shape for the fused phases.
bool fused_supported(int d, int H, int d_kv, int ff);

}  // namespace mrtdf
