// Parameter blocks and launch entry points of the encoder kernels
// (Depthformer::encode and the cross-attention K/V projection).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace mrtdf {

enum GemmEpi : int {
  kEpiStore = 0,    // out[m, n] = R(acc)
  kEpiResid = 1,    // out[m, n] = R(out[m, n] + R(acc))
  kEpiGeglu = 2,    // columns (2j, 2j+1) = (wi_0, wi_1): out[m, j] = R(gelu(R(a)) * R(b))
  kEpiCrossKV = 3,  // column n of the all-layer K/V projection -> cross cache
  // decode projections for more rows than the GEMV kernel takes (tcgen05 only)
  kEpiDecResid = 4,  // out[m, n] = R(resid[m, n] + R(acc))   (resid may alias out)
  kEpiDecQKV = 5,    // head-major q/k/v rows: q -> out (m, h*64+c), k/v -> cache at `pos`
  kEpiLogits = 6,    // float out[m, out_offset + n] = R(acc)
};

struct GemmParams {
  const void* A;  // (M, K) row-major, lda
  const void* W;  // (N, K) row-major (Linear weight layout (out, in))
  void* out;      // (M, ldo)
  int M, N, K;
  int lda, ldo;
  // kEpiCrossKV: ck / cv are (Lt, B, H, Smax, 64); row m = b * S + s
  void* ck;
  void* cv;
  int S, B, H, Smax, inner;
  // decode epilogues: residual rows (kEpiDecResid), self K/V caches (rows, H,
  // cap, 64) written at position pos (kEpiDecQKV), column offset (kEpiLogits)
  const void* resid;
  int ldr;
  int cap, pos;
  int out_offset;
  // tcgen05 only: largest split-K cluster (1, 2, 4 or 8) the launcher may
  // choose when the output tiles cannot fill the GPU (0 or 1: no split)
  int max_ksplit;
};

// fp32 GEMM on the CUDA cores (the fp32 parity mode).
cudaError_t launch_gemm_f32(int epi, const GemmParams& p, cudaStream_t s, bool pdl);
// bf16 GEMM on tcgen05 tensor cores with TMA-fed operands (gemm_tc.cu).
cudaError_t launch_gemm_tc(int epi, const GemmParams& p, int* err, cudaStream_t s, bool pdl);
cudaError_t gemm_tc_set_smem_limits();

struct EncAttnParams {
  const void* qkv;  // (B*S, 3*inner): q | k | v
  void* out;        // (B*S, inner)
  int B, S, H, inner;
  int* err;         // device error word (bounded waits of the tensor-core kernel)
};
cudaError_t launch_enc_attention(int dtype, const EncAttnParams& p, cudaStream_t s, bool pdl);
// bf16 attention on tcgen05 (enc_attn_tc.cu)
cudaError_t launch_enc_attention_tc(const EncAttnParams& p, cudaStream_t s, bool pdl);
cudaError_t enc_attn_tc_set_smem_limits();

// x[b*S+s, :] = R(emb[ids[b*S+s], :] + pe[s, :]) with pe already rounded to the dtype.
// An id outside [0, V) sets kErrBadToken in *err and reads row 0 instead.
cudaError_t launch_embed_pe(int dtype, const void* emb, const float* pe, const int32_t* ids, int rows, int S, int d,
                            int V, void* out, int* err, cudaStream_t s, bool pdl);
// out[m, :] = RMSNorm(x[m, :]) * w (rounding as in the decode path).
cudaError_t launch_rmsnorm_rows(int dtype, const void* x, const void* w, int rows, int d, void* out, cudaStream_t s,
                                bool pdl);

}  // namespace mrtdf
