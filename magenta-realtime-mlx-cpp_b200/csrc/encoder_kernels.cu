// Encoder kernels: embedding + sinusoidal position add, row RMSNorm, the
// projection GEMMs with fused epilogues, and full (unmasked) attention.
//
// Reference semantics (rhymeswithlion/magenta-realtime-mlx-cpp):
//   Depthformer::encode  depthformer/model.cpp:226-241
//   EncoderLayer         depthformer/modules.cpp:349-358 (pre-norm self
//                        attention, no mask, no bias, scale 1.0; gated FFN)
//   project_kv           modules.cpp:323-333 (cross K/V, done for all 20
//                        temporal layers in one GEMM with N = Lt * 2 * inner)
// bf16 GEMMs and the bf16 attention run on tcgen05 (gemm_tc.cu,
// enc_attn_tc.cu); the fp32 GEMM and attention here run on the CUDA cores so
// the fp32 parity mode stays exact fp32.
#include <cuda_bf16.h>

#include "common.cuh"
#include "encoder_kernels.cuh"
#include "gemm_epilogue.cuh"

namespace mrtdf {

typedef __nv_bfloat16 bf16;

// ---------------------------------------------------------------------------
// fp32 GEMM on the CUDA cores: 64x64x16 tile, 256 threads, 4x4 outputs per
// thread, operands staged transposed in shared memory.
// ---------------------------------------------------------------------------
template <int EPI>
__global__ void __launch_bounds__(256) gemm_f32_kernel(const GemmParams p) {
  __shared__ float sA[16][64 + 4];
  __shared__ float sB[16][64 + 4];
  pdl_launch_dependents();
  pdl_wait();
  const int tid = threadIdx.x;
  const int bm = blockIdx.y * 64, bn = blockIdx.x * 64;
  const int tx = tid & 15, ty = tid >> 4;
  const float* A = reinterpret_cast<const float*>(p.A);
  const float* W = reinterpret_cast<const float*>(p.W);
  float acc[4][4] = {};
  for (int k0 = 0; k0 < p.K; k0 += 16) {
    for (int i = tid; i < 64 * 16; i += 256) {
      const int r = i >> 4, kk = i & 15;
      const int gm = bm + r, gn = bn + r, gk = k0 + kk;
      sA[kk][r] = (gm < p.M && gk < p.K) ? A[(size_t)gm * p.lda + gk] : 0.f;
      sB[kk][r] = (gn < p.N && gk < p.K) ? W[(size_t)gn * p.K + gk] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = sA[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = sB[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = bm + ty * 4 + i;
    epi_pair<float, EPI>(p, m, bn + tx * 4, acc[i][0], acc[i][1]);
    epi_pair<float, EPI>(p, m, bn + tx * 4 + 2, acc[i][2], acc[i][3]);
  }
}

template <typename P>
static cudaError_t launch_k(void (*kern)(const P), dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl,
                            const P& p) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

cudaError_t launch_gemm_f32(int epi, const GemmParams& p, cudaStream_t s, bool pdl) {
  if (p.M <= 0 || p.N <= 0) return cudaSuccess;
  if (p.N % 2 != 0) return cudaErrorInvalidValue;
  const dim3 grid((p.N + 63) / 64, (p.M + 63) / 64);
  switch (epi) {
    case kEpiStore: return launch_k(gemm_f32_kernel<kEpiStore>, grid, dim3(256), 0, s, pdl, p);
    case kEpiResid: return launch_k(gemm_f32_kernel<kEpiResid>, grid, dim3(256), 0, s, pdl, p);
    case kEpiGeglu: return launch_k(gemm_f32_kernel<kEpiGeglu>, grid, dim3(256), 0, s, pdl, p);
    case kEpiCrossKV: return launch_k(gemm_f32_kernel<kEpiCrossKV>, grid, dim3(256), 0, s, pdl, p);
  }
  return cudaErrorInvalidValue;
}

// fp32 encoder attention on the CUDA cores: one query per thread, K/V tiles
// of 16 keys in shared memory, online softmax per tile.
__global__ void __launch_bounds__(128) enc_attn_f32_kernel(const EncAttnParams p) {
  __shared__ float sK[16][64];
  __shared__ float sV[16][64];
  pdl_launch_dependents();
  pdl_wait();
  const int tid = threadIdx.x;
  const int qi = blockIdx.x * 128 + tid;
  const int bh = blockIdx.y, b = bh / p.H, h = bh - b * p.H;
  const int ld = 3 * p.inner;
  const float* base = reinterpret_cast<const float*>(p.qkv) + (size_t)b * p.S * ld;
  float q[64], o[64];
  const bool valid = qi < p.S;
#pragma unroll
  for (int c = 0; c < 64; ++c) {
    q[c] = valid ? base[(size_t)qi * ld + h * 64 + c] : 0.f;
    o[c] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  for (int k0 = 0; k0 < p.S; k0 += 16) {
    for (int i = tid; i < 16 * 64; i += 128) {
      const int r = i >> 6, c = i & 63;
      const int kr = k0 + r;
      sK[r][c] = kr < p.S ? base[(size_t)kr * ld + p.inner + h * 64 + c] : 0.f;
      sV[r][c] = kr < p.S ? base[(size_t)kr * ld + 2 * p.inner + h * 64 + c] : 0.f;
    }
    __syncthreads();
    const int nk = min(16, p.S - k0);
    float s[16];
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      float acc = 0.f;
#pragma unroll
      for (int c = 0; c < 64; ++c) acc = fmaf(q[c], sK[j][c], acc);
      s[j] = j < nk ? acc : -INFINITY;
      mx = fmaxf(mx, s[j]);
    }
    const float nm = fmaxf(m, mx);
    const float scale = (m == -INFINITY) ? 0.f : expf(m - nm);
    l *= scale;
#pragma unroll
    for (int c = 0; c < 64; ++c) o[c] *= scale;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float pj = (j < nk) ? expf(s[j] - nm) : 0.f;
      l += pj;
#pragma unroll
      for (int c = 0; c < 64; ++c) o[c] = fmaf(pj, sV[j][c], o[c]);
    }
    m = nm;
    __syncthreads();
  }
  if (valid) {
    float* out = reinterpret_cast<float*>(p.out) + ((size_t)b * p.S + qi) * p.inner + h * 64;
#pragma unroll
    for (int c = 0; c < 64; ++c) out[c] = o[c] / l;
  }
}

cudaError_t launch_enc_attention(int dtype, const EncAttnParams& p, cudaStream_t s, bool pdl) {
  if (dtype == 1) return launch_enc_attention_tc(p, s, pdl);  // tcgen05 (enc_attn_tc.cu)
  const dim3 grid((p.S + 127) / 128, p.B * p.H);
  return launch_k(enc_attn_f32_kernel, grid, dim3(128), 0, s, pdl, p);
}

// ---------------------------------------------------------------------------
// Embedding + position add and row RMSNorm
// ---------------------------------------------------------------------------
struct EmbedPeParams {
  const void* emb;
  const float* pe;
  const int32_t* ids;
  int rows, S, d, V;
  void* out;
  int* err;
};

template <typename T>
__global__ void embed_pe_kernel(const EmbedPeParams p) {
  pdl_launch_dependents();
  pdl_wait();
  const int r = blockIdx.x;
  const int s = r % p.S;
  int id = p.ids[r];
  if (id < 0 || id >= p.V) {  // device-resident ids are not checked on the host
    if (threadIdx.x == 0 && p.err) atomicOr(p.err, kErrBadToken);
    id = 0;
  }
  const T* e = reinterpret_cast<const T*>(p.emb) + (size_t)id * p.d;
  const float* pe = p.pe + (size_t)s * p.d;
  T* o = reinterpret_cast<T*>(p.out) + (size_t)r * p.d;
  for (int i = threadIdx.x; i < p.d; i += blockDim.x) o[i] = from_f<T>(__fadd_rn(to_f(e[i]), pe[i]));
}

cudaError_t launch_embed_pe(int dtype, const void* emb, const float* pe, const int32_t* ids, int rows, int S, int d,
                            int V, void* out, int* err, cudaStream_t s, bool pdl) {
  EmbedPeParams p{emb, pe, ids, rows, S, d, V, out, err};
  return dtype == 1 ? launch_k(embed_pe_kernel<bf16>, dim3(rows), dim3(256), 0, s, pdl, p)
                    : launch_k(embed_pe_kernel<float>, dim3(rows), dim3(256), 0, s, pdl, p);
}

struct RmsParams {
  const void* x;
  const void* w;
  int rows, d;
  void* out;
};

template <typename T>
__global__ void __launch_bounds__(256) rmsnorm_rows_kernel(const RmsParams p) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ float red[8];
  const int r = blockIdx.x;
  const T* x = reinterpret_cast<const T*>(p.x) + (size_t)r * p.d;
  const T* w = reinterpret_cast<const T*>(p.w);
  T* o = reinterpret_cast<T*>(p.out) + (size_t)r * p.d;
  float ss = 0.f;
  for (int i = threadIdx.x; i < p.d; i += 256) {
    const float v = to_f(x[i]);
    ss += v * v;
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) t += red[i];
  const float rs = __frcp_rn(__fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)p.d), 1e-6f)));
  for (int i = threadIdx.x; i < p.d; i += 256)
    o[i] = from_f<T>(__fmul_rn(to_f(w[i]), rnd<T>(__fmul_rn(to_f(x[i]), rs))));
}

cudaError_t launch_rmsnorm_rows(int dtype, const void* x, const void* w, int rows, int d, void* out, cudaStream_t s,
                                bool pdl) {
  RmsParams p{x, w, rows, d, out};
  return dtype == 1 ? launch_k(rmsnorm_rows_kernel<bf16>, dim3(rows), dim3(256), 0, s, pdl, p)
                    : launch_k(rmsnorm_rows_kernel<float>, dim3(rows), dim3(256), 0, s, pdl, p);
}

}  // namespace mrtdf
