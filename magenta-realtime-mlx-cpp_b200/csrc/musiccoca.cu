// Style path: the MusicCoCa text tower (prompt ids -> 768-d embedding) and
// the residual vector quantisation of the embedding into style tokens, in
// float32, with the C ABI of include/mrtmc.h.
//
// Reference (rhymeswithlion/magenta-realtime-mlx-cpp):
//   MusicCoCaEncoder::embed_text        src/magenta_realtime_mlx/musiccoca.cpp:272-295
//   TransformerLayer::operator()        musiccoca.cpp:195-205 (pre-LN, capped attention)
//   CoCaMHA::operator()                 musiccoca.cpp:136-176
//   AttentionPooler::operator()         musiccoca.cpp:219-226
//   LayerNorm::operator()               musiccoca.cpp:72-82
//   rvq_quantization                    rvq.cpp:24-66
//   StyleModel::style_tokens_lm         style_model.cpp:111-122
//
// Launch plan of one embed_text call (B prompts of L tokens, M = B * L rows):
// embedding -> 12 x (LayerNorm, q|k|v GEMM (N = 2304), capped masked
// attention, o_proj GEMM + residual, LayerNorm, w1 GEMM + GELU, w2 GEMM +
// residual) -> exit LayerNorm -> pooler LayerNorm -> k|v GEMM (N = 6144) ->
// pooler attention (one learned query, 12 heads x 256) -> o_proj GEMM. The
// GEMMs are float32 on the CUDA cores (the reference runs MusicCoCa in
// float32; tf32 tensor-core operands would not hold the 1e-4 parity), split
// over K into a scratch buffer when the output tiles cannot fill the GPU and
// summed in split order by the epilogue kernel (deterministic). One CUDA
// graph per (B, L).
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <utility>
#include <vector>

#include "../../include/mrtmc.h"
#include "device_errors.h"
#include "host_util.h"

using namespace mrtdf;

namespace {

#define MC_CUDA(expr)                                                                                    \
  do {                                                                                                   \
    cudaError_t e_ = (expr);                                                                             \
    if (e_ != cudaSuccess)                                                                               \
      throw Error{MRTDF_ERR_CUDA, std::string(#expr) + ": " + cudaGetErrorString(e_)};                   \
  } while (0)

// MusicCoCaConfig (musiccoca.h:151-162): the text tower's widths.
constexpr int kD = 768, kHeads = 12, kDHead = 64, kFF = 3072, kLayers = 12, kPoolDHead = 256;
constexpr int kMaxLen = MRTMC_MAX_TEXT_LEN;
constexpr int kQkv = 3 * kHeads * kDHead;         // 2304
constexpr int kPoolInner = kHeads * kPoolDHead;   // 3072
constexpr float kCap = 50.0f;                     // TransformerLayer::kAttenLogitCap
constexpr float kLnEps = 1e-5f;
constexpr int kMaxQuantRows = 1024;

// ---------------------------------------------------------------------------
// Kernels
// ---------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
// Sum over a block of blockDim.x threads (a multiple of 32, <= 1024).
__device__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
  for (int i = 0; i < nw; ++i) t += red[i];
  return t;
}

// Token embedding x sqrt(d_model) and the additive key mask pad x -1e9
// (MusicCoCaEncoder::embed_text, musiccoca.cpp:276-286).
__global__ void mc_embed_kernel(const float* __restrict__ emb, const int32_t* __restrict__ ids,
                                const float* __restrict__ pad, int M, int V, float* __restrict__ x,
                                float* __restrict__ mask, int* err) {
  const int m = blockIdx.x;
  if (m >= M) return;
  const int id = ids[m];
  const float s = sqrtf((float)kD);
  if (id < 0 || id >= V) {
    if (threadIdx.x == 0) atomicOr(err, kErrBadToken);
    for (int i = threadIdx.x; i < kD; i += blockDim.x) x[(size_t)m * kD + i] = 0.f;
  } else {
    for (int i = threadIdx.x; i < kD; i += blockDim.x) x[(size_t)m * kD + i] = emb[(size_t)id * kD + i] * s;
  }
  if (threadIdx.x == 0) mask[m] = pad[m] * -1e9f;
}

// LayerNorm (musiccoca.cpp:72-82): mean, var = mean((x - mean)^2),
// (x - mean) * rsqrt(var + eps) * w + b; one 256-thread CTA per row of 768.
__global__ void __launch_bounds__(256) mc_layernorm_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                           const float* __restrict__ b, float* __restrict__ y) {
  __shared__ float red[8];
  const size_t row = blockIdx.x;
  const float* r = x + row * kD;
  float v[3];
#pragma unroll
  for (int i = 0; i < 3; ++i) v[i] = r[threadIdx.x + 256 * i];
  const float mean = block_sum(v[0] + v[1] + v[2], red) / (float)kD;
  float c[3], q = 0.f;
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    c[i] = v[i] - mean;
    q += c[i] * c[i];
  }
  const float var = block_sum(q, red) / (float)kD;
  const float inv = 1.0f / sqrtf(var + kLnEps);
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    const int k = threadIdx.x + 256 * i;
    y[row * kD + k] = c[i] * inv * w[k] + b[k];
  }
}

// y = epi(x W^T + bias): x (M, K) row stride ldx, W (N, K), 64 x 64 output
// tile per CTA, 16-deep k slices staged in shared memory, 4 x 4 outputs per
// thread. blockIdx.z = split index: k range [z * kchunk, min(K, (z+1) kchunk));
// with ksplit > 1 the raw partial goes to part[z][M][N] for mc_splitk_epi.
enum McEpi : int { kMcStore = 0, kMcGelu = 1, kMcResid = 2 };

struct McGemm {
  const float* x;
  const float* w;
  const float* bias;
  float* y;
  float* part;
  int M, N, K, ldx, ldy, kchunk, ksplit, epi;
};

__device__ __forceinline__ float mc_epi(int epi, float acc, float bias, float prev) {
  const float v = acc + bias;
  if (epi == kMcGelu) return 0.5f * v * (1.0f + erff(v * 0.7071067811865475f));  // gelu, exact form
  if (epi == kMcResid) return prev + v;
  return v;
}

__global__ void __launch_bounds__(256) mc_gemm_kernel(const McGemm p) {
  __shared__ float sA[16][64 + 4];
  __shared__ float sB[16][64 + 4];
  const int tid = threadIdx.x;
  const int bm = blockIdx.y * 64, bn = blockIdx.x * 64;
  const int tx = tid & 15, ty = tid >> 4;
  const int k_begin = blockIdx.z * p.kchunk, k_end = min(p.K, k_begin + p.kchunk);
  float acc[4][4] = {};
  // staging: thread -> (row r = tid / 4, k quad kq = tid % 4): one float4 of A and of W
  const int lr = tid >> 2, lq = (tid & 3) * 4;
  for (int k0 = k_begin; k0 < k_end; k0 += 16) {
    const int gk = k0 + lq;
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f), bw = make_float4(0.f, 0.f, 0.f, 0.f);
    if (bm + lr < p.M && gk < k_end) a = *reinterpret_cast<const float4*>(p.x + (size_t)(bm + lr) * p.ldx + gk);
    if (bn + lr < p.N && gk < k_end) bw = *reinterpret_cast<const float4*>(p.w + (size_t)(bn + lr) * p.K + gk);
    sA[lq + 0][lr] = a.x;
    sA[lq + 1][lr] = a.y;
    sA[lq + 2][lr] = a.z;
    sA[lq + 3][lr] = a.w;
    sB[lq + 0][lr] = bw.x;
    sB[lq + 1][lr] = bw.y;
    sB[lq + 2][lr] = bw.z;
    sB[lq + 3][lr] = bw.w;
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      float av[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) av[i] = sA[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) bv[j] = sB[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = bm + ty * 4 + i;
    if (m >= p.M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = bn + tx * 4 + j;
      if (n >= p.N) continue;
      if (p.ksplit > 1) {
        p.part[((size_t)blockIdx.z * p.M + m) * p.N + n] = acc[i][j];
      } else {
        float* yp = p.y + (size_t)m * p.ldy + n;
        *yp = mc_epi(p.epi, acc[i][j], p.bias[n], p.epi == kMcResid ? *yp : 0.f);
      }
    }
  }
}

// Sum of the split-K partials in split order, then the epilogue.
__global__ void mc_splitk_epi_kernel(const McGemm p) {
  const size_t n_out = (size_t)p.M * p.N;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_out; i += (size_t)gridDim.x * blockDim.x) {
    const int m = (int)(i / p.N), n = (int)(i - (size_t)m * p.N);
    float acc = 0.f;
    for (int z = 0; z < p.ksplit; ++z) acc += p.part[(size_t)z * n_out + i];
    float* yp = p.y + (size_t)m * p.ldy + n;
    *yp = mc_epi(p.epi, acc, p.bias[n], p.epi == kMcResid ? *yp : 0.f);
  }
}

// Text-layer attention (CoCaMHA, musiccoca.cpp:136-176, d_head 64): logits
// q.k / 8, capped 50 tanh(l / 50), + the key mask, softmax, weighted values.
// qkv (M, 2304) = q | k | v rows of the layer's input; ctx (M, 768). Grid
// (B * H, ceil(L / 8)), 8 warps, one query per warp; the (b, h) keys and
// values staged in shared memory (L x 65 and L x 64 floats).
__global__ void __launch_bounds__(256) mc_attn_text_kernel(const float* __restrict__ qkv,
                                                           const float* __restrict__ mask, int L,
                                                           float* __restrict__ ctx) {
  extern __shared__ float sm[];
  float* sK = sm;                       // L x 65
  float* sV = sK + (size_t)kMaxLen * 65;  // L x 64
  float* sQ = sV + (size_t)kMaxLen * 64;  // 8 x 64
  float* sP = sQ + 8 * 64;              // 8 x 128
  const int b = blockIdx.x / kHeads, h = blockIdx.x - b * kHeads;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float* base = qkv + (size_t)b * L * kQkv;
  for (int i = threadIdx.x; i < L * 64; i += 256) {
    const int j = i >> 6, d = i & 63;
    sK[j * 65 + d] = base[(size_t)j * kQkv + kHeads * kDHead + h * kDHead + d];
    sV[j * 64 + d] = base[(size_t)j * kQkv + 2 * kHeads * kDHead + h * kDHead + d];
  }
  const int qi = blockIdx.y * 8 + warp;
  if (qi < L) {
    sQ[warp * 64 + lane] = base[(size_t)qi * kQkv + h * kDHead + lane];
    sQ[warp * 64 + lane + 32] = base[(size_t)qi * kQkv + h * kDHead + lane + 32];
  }
  __syncthreads();
  if (qi >= L) return;
  const float* mk = mask + (size_t)b * L;
  float lmax = -INFINITY;
  for (int j = lane; j < L; j += 32) {
    float s = 0.f;
#pragma unroll 16
    for (int d = 0; d < 64; ++d) s = fmaf(sQ[warp * 64 + d], sK[j * 65 + d], s);
    float l = s * 0.125f;  // 1 / sqrt(64)
    l = kCap * tanhf(l / kCap);
    l += mk[j];
    sP[warp * 128 + j] = l;
    lmax = fmaxf(lmax, l);
  }
  lmax = warp_max(lmax);
  float lsum = 0.f;
  for (int j = lane; j < L; j += 32) {
    const float e = expf(sP[warp * 128 + j] - lmax);
    sP[warp * 128 + j] = e;
    lsum += e;
  }
  lsum = warp_sum(lsum);
  __syncwarp();
  float o0 = 0.f, o1 = 0.f;
  for (int j = 0; j < L; ++j) {
    const float wgt = sP[warp * 128 + j] / lsum;
    o0 = fmaf(wgt, sV[j * 64 + lane], o0);
    o1 = fmaf(wgt, sV[j * 64 + lane + 32], o1);
  }
  float* out = ctx + ((size_t)b * L + qi) * kD + h * kDHead;
  out[lane] = o0;
  out[lane + 32] = o1;
}

// Pooler attention (AttentionPooler, musiccoca.cpp:219-226; CoCaMHA with the
// per-dimension query scale, no cap, no mask): one learned query (already
// projected and scaled, qs (3072)) over kv (M, 6144) = k | v rows; ctx
// (B, 3072). Grid B * H, 256 threads (one per head dimension).
__global__ void __launch_bounds__(256) mc_attn_pool_kernel(const float* __restrict__ qs, const float* __restrict__ kv,
                                                           int L, float* __restrict__ ctx) {
  __shared__ float sP[kMaxLen];
  __shared__ float red[8];
  const int b = blockIdx.x / kHeads, h = blockIdx.x - b * kHeads;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float* base = kv + (size_t)b * L * (2 * kPoolInner);
  const float* q = qs + h * kPoolDHead;
  for (int j = warp; j < L; j += 8) {
    const float* kr = base + (size_t)j * (2 * kPoolInner) + h * kPoolDHead;
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < kPoolDHead / 32; ++i) s = fmaf(q[lane + 32 * i], kr[lane + 32 * i], s);
    s = warp_sum(s);
    if (lane == 0) sP[j] = s * 0.0625f;  // 1 / sqrt(256)
  }
  __syncthreads();
  float m = -INFINITY;
  for (int j = 0; j < L; ++j) m = fmaxf(m, sP[j]);
  float part = 0.f;
  for (int j = threadIdx.x; j < L; j += 256) part += expf(sP[j] - m);
  const float sum = block_sum(part, red);
  const int d = threadIdx.x;
  float o = 0.f;
  for (int j = 0; j < L; ++j) {
    const float wgt = expf(sP[j] - m) / sum;
    o = fmaf(wgt, base[(size_t)j * (2 * kPoolInner) + kPoolInner + h * kPoolDHead + d], o);
  }
  ctx[(size_t)b * kPoolInner + h * kPoolDHead + d] = o;
}

// q (3072) scaled by the per-dimension factor sc (256), in place.
__global__ void mc_scale_query_kernel(float* q, const float* sc) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < kPoolInner) q[i] = q[i] * sc[i % kPoolDHead];
}

// rvq_quantization (rvq.cpp:24-66), one level: distance of every codeword of
// level k to each residual, |r|^2 - 2 r.c + |c|^2. Grid (N, ceil(C / 8)),
// one warp per codeword.
__global__ void __launch_bounds__(256) mc_rvq_dist_kernel(const float* __restrict__ r, const float* __restrict__ r2,
                                                          const float* __restrict__ cb, const float* __restrict__ c2,
                                                          int C, float* __restrict__ dist) {
  const int n = blockIdx.x, lane = threadIdx.x & 31;
  const int c = blockIdx.y * 8 + (threadIdx.x >> 5);
  if (c >= C) return;
  const float* rr = r + (size_t)n * kD;
  const float* w = cb + (size_t)c * kD;
  float s = 0.f;
#pragma unroll 4
  for (int i = lane; i < kD; i += 32) s = fmaf(rr[i], w[i], s);
  s = warp_sum(s);
  if (lane == 0) dist[(size_t)n * C + c] = (r2[n] - 2.0f * s) + c2[c];
}

// The first codeword of least distance (index order), then r -= codeword and
// |r|^2 for the next level. One 1024-thread CTA per residual.
__global__ void __launch_bounds__(1024) mc_rvq_pick_kernel(float* __restrict__ r, float* __restrict__ r2,
                                                           const float* __restrict__ cb, int C,
                                                           const float* __restrict__ dist, int32_t* tokens,
                                                           int levels, int level) {
  __shared__ float sd[32];
  __shared__ int si[32];
  __shared__ float red[32];
  const int n = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float bd = INFINITY;
  int bi = 0x7fffffff;
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    const float v = dist[(size_t)n * C + c];
    if (v < bd) {  // c increases along a thread's loop: the first of equal minima stays
      bd = v;
      bi = c;
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float od = __shfl_xor_sync(0xffffffffu, bd, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (od < bd || (od == bd && oi < bi)) {
      bd = od;
      bi = oi;
    }
  }
  if (lane == 0) {
    sd[warp] = bd;
    si[warp] = bi;
  }
  __syncthreads();
  float best_d = sd[0];
  int best = si[0];
  for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
    if (sd[w] < best_d || (sd[w] == best_d && si[w] < best)) {
      best_d = sd[w];
      best = si[w];
    }
  if (best >= C) best = 0;  // all distances NaN: the reference's argmin gives 0
  if (threadIdx.x == 0) tokens[(size_t)n * levels + level] = best;
  float q = 0.f;
  for (int i = threadIdx.x; i < kD; i += blockDim.x) {
    const float v = r[(size_t)n * kD + i] - cb[(size_t)best * kD + i];
    r[(size_t)n * kD + i] = v;
    q += v * v;
  }
  const float s = block_sum(q, red);
  if (threadIdx.x == 0) r2[n] = s;
}

// |r|^2 of the input embeddings (level 0).
__global__ void __launch_bounds__(256) mc_rvq_norm_kernel(const float* __restrict__ r, float* __restrict__ r2) {
  __shared__ float red[8];
  float q = 0.f;
  for (int i = threadIdx.x; i < kD; i += 256) {
    const float v = r[(size_t)blockIdx.x * kD + i];
    q += v * v;
  }
  const float s = block_sum(q, red);
  if (threadIdx.x == 0) r2[blockIdx.x] = s;
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
struct McLayer {
  float *ln1_w, *ln1_b, *ln2_w, *ln2_b;
  float *wqkv, *bqkv, *wo, *bo, *w1, *b1, *w2, *b2;
};

}  // namespace

struct mrtmc_model {
  int device = 0;
  int max_batch = 0;
  bool loaded = false;
  cudaStream_t s = nullptr;
  int V = 0, K = 0, C = 0;
  std::vector<void*> allocs;
  // weights
  float* emb = nullptr;
  McLayer layers[kLayers];
  float *exit_w, *exit_b, *pool_ln_w, *pool_ln_b;
  float *pool_wkv, *pool_bkv, *pool_wo, *pool_bo;
  float* pool_q = nullptr;  // projected, scaled learned query (3072)
  float* codebooks = nullptr;  // (K, C, 768)
  float* c2 = nullptr;         // (K, C) |c|^2
  // activations
  int32_t* ids = nullptr;
  float *pad = nullptr, *mask = nullptr;
  float *x = nullptr, *h = nullptr, *qkv = nullptr, *ctx = nullptr, *f = nullptr, *kv = nullptr;
  float *pctx = nullptr, *out = nullptr;
  float* part = nullptr;
  size_t part_floats = 0;
  // quantiser
  float *r = nullptr, *r2 = nullptr, *dist = nullptr;
  int32_t* tok = nullptr;
  int* err = nullptr;
  int num_sms = 148;
  std::map<std::pair<int, int>, cudaGraphExec_t> graphs;
  std::map<std::pair<int, int>, long long> graph_launches;
  long long launches = 0;  // of the plan being enqueued

  ~mrtmc_model() {
    for (auto& g : graphs) cudaGraphExecDestroy(g.second);
    for (void* p : allocs) cudaFree(p);
    if (s) cudaStreamDestroy(s);
  }
  void* alloc(size_t bytes) {
    void* q = nullptr;
    MC_CUDA(cudaMalloc(&q, bytes));
    allocs.push_back(q);
    return q;
  }
};

namespace {

void check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw Error{MRTDF_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e)};
}

// Split-K factor for an M x N x K GEMM: enough CTAs for two per SM, at most 8
// splits, each at least 64 deep.
int choose_ksplit(int M, int N, int K, int num_sms) {
  const int tiles = ((M + 63) / 64) * ((N + 63) / 64);
  int ks = 1;
  while (ks < 8 && tiles * ks < 2 * num_sms && K / (ks * 2) >= 64) ks *= 2;
  return ks;
}

size_t gemm_part_floats(int M, int N, int K, int num_sms) {
  const int ks = choose_ksplit(M, N, K, num_sms);
  return ks > 1 ? (size_t)ks * M * N : 0;
}

void gemm(mrtmc_model* m, const float* x, int ldx, const float* w, const float* bias, float* y, int ldy, int M, int N,
          int K, int epi) {
  McGemm p{};
  p.x = x;
  p.w = w;
  p.bias = bias;
  p.y = y;
  p.part = m->part;
  p.M = M;
  p.N = N;
  p.K = K;
  p.ldx = ldx;
  p.ldy = ldy;
  p.epi = epi;
  p.ksplit = choose_ksplit(M, N, K, m->num_sms);
  if ((size_t)p.ksplit * M * N > m->part_floats && p.ksplit > 1)
    throw Error{MRTDF_ERR_STATE, "style path: split-K scratch too small"};
  p.kchunk = ((K / p.ksplit + 15) / 16) * 16;
  dim3 grid((N + 63) / 64, (M + 63) / 64, p.ksplit);
  mc_gemm_kernel<<<grid, 256, 0, m->s>>>(p);
  ++m->launches;
  check_launch("style gemm");
  if (p.ksplit > 1) {
    const size_t n_out = (size_t)M * N;
    const int blocks = (int)std::min<size_t>((n_out + 255) / 256, (size_t)m->num_sms * 8);
    mc_splitk_epi_kernel<<<blocks, 256, 0, m->s>>>(p);
    ++m->launches;
    check_launch("style split-K epilogue");
  }
}

void layernorm(mrtmc_model* m, const float* x, const float* w, const float* b, float* y, int M) {
  mc_layernorm_kernel<<<M, 256, 0, m->s>>>(x, w, b, y);
  ++m->launches;
  check_launch("style layernorm");
}

size_t attn_text_smem() { return ((size_t)kMaxLen * 65 + (size_t)kMaxLen * 64 + 8 * 64 + 8 * 128) * sizeof(float); }

// The whole embed_text plan for (B, L) on m->s (ids, pad already on the device).
void enqueue_embed(mrtmc_model* m, int B, int L) {
  const int M = B * L;
  m->launches = 0;
  mc_embed_kernel<<<M, 256, 0, m->s>>>(m->emb, m->ids, m->pad, M, m->V, m->x, m->mask, m->err);
  ++m->launches;
  check_launch("style embedding");
  for (int l = 0; l < kLayers; ++l) {
    const McLayer& Ly = m->layers[l];
    // TransformerLayer::operator() (musiccoca.cpp:195-205)
    layernorm(m, m->x, Ly.ln1_w, Ly.ln1_b, m->h, M);
    gemm(m, m->h, kD, Ly.wqkv, Ly.bqkv, m->qkv, kQkv, M, kQkv, kD, kMcStore);
    mc_attn_text_kernel<<<dim3(B * kHeads, (L + 7) / 8), 256, attn_text_smem(), m->s>>>(m->qkv, m->mask, L, m->ctx);
    ++m->launches;
    check_launch("style attention");
    gemm(m, m->ctx, kD, Ly.wo, Ly.bo, m->x, kD, M, kD, kD, kMcResid);
    layernorm(m, m->x, Ly.ln2_w, Ly.ln2_b, m->h, M);
    gemm(m, m->h, kD, Ly.w1, Ly.b1, m->f, kFF, M, kFF, kD, kMcGelu);
    gemm(m, m->f, kFF, Ly.w2, Ly.b2, m->x, kD, M, kD, kFF, kMcResid);
  }
  layernorm(m, m->x, m->exit_w, m->exit_b, m->h, M);        // text_exit_ln
  layernorm(m, m->h, m->pool_ln_w, m->pool_ln_b, m->ctx, M);  // AttentionPooler::ln_
  gemm(m, m->ctx, kD, m->pool_wkv, m->pool_bkv, m->kv, 2 * kPoolInner, M, 2 * kPoolInner, kD, kMcStore);
  mc_attn_pool_kernel<<<B * kHeads, 256, 0, m->s>>>(m->pool_q, m->kv, L, m->pctx);
  ++m->launches;
  check_launch("style pooler attention");
  gemm(m, m->pctx, kPoolInner, m->pool_wo, m->pool_bo, m->out, kD, B, kD, kPoolInner, kMcStore);
}

cudaGraphExec_t embed_graph(mrtmc_model* m, int B, int L) {
  const auto key = std::make_pair(B, L);
  auto it = m->graphs.find(key);
  if (it != m->graphs.end()) return it->second;
  MC_CUDA(cudaStreamBeginCapture(m->s, cudaStreamCaptureModeThreadLocal));
  try {
    enqueue_embed(m, B, L);
  } catch (...) {
    cudaGraph_t g = nullptr;
    cudaStreamEndCapture(m->s, &g);
    if (g) cudaGraphDestroy(g);
    throw;
  }
  cudaGraph_t g = nullptr;
  MC_CUDA(cudaStreamEndCapture(m->s, &g));
  cudaGraphExec_t ge = nullptr;
  const cudaError_t e = cudaGraphInstantiate(&ge, g, 0);
  cudaGraphDestroy(g);
  MC_CUDA(e);
  m->graphs[key] = ge;
  m->graph_launches[key] = m->launches;
  return ge;
}

void sync_and_check(mrtmc_model* m) {
  MC_CUDA(cudaStreamSynchronize(m->s));
  int e = 0;
  MC_CUDA(cudaMemcpy(&e, m->err, sizeof(int), cudaMemcpyDeviceToHost));
  if (e) {
    MC_CUDA(cudaMemset(m->err, 0, sizeof(int)));
    if (e & kErrBadToken) throw Error{MRTDF_ERR_RANGE, "embed_text: a token id outside [0, vocab)"};
    throw Error{MRTDF_ERR_CUDA, "style path: device error word " + std::to_string(e)};
  }
}

void require_loaded(mrtmc_model* m) {
  if (!m) throw Error{MRTDF_ERR_INVALID, "NULL model"};
  if (!m->loaded) throw Error{MRTDF_ERR_STATE, "load the style model's weights first"};
}

// Upload ids / pad after the host-side checks; runs the embed plan.
void run_embed(mrtmc_model* m, const int32_t* ids, const float* pad, int B, int L) {
  if (!ids || !pad) throw Error{MRTDF_ERR_INVALID, "NULL argument"};
  if (B <= 0 || B > m->max_batch)
    throw Error{MRTDF_ERR_RANGE, "embed_text: B = " + std::to_string(B) + " outside [1, " +
                                     std::to_string(m->max_batch) + "]"};
  if (L <= 0 || L > kMaxLen)
    throw Error{MRTDF_ERR_RANGE, "embed_text: L = " + std::to_string(L) + " outside [1, 128]"};
  for (size_t i = 0; i < (size_t)B * L; ++i)
    if (ids[i] < 0 || ids[i] >= m->V)
      throw Error{MRTDF_ERR_RANGE, "embed_text: token id " + std::to_string(ids[i]) + " outside [0, " +
                                       std::to_string(m->V) + ")"};
  MC_CUDA(cudaMemcpyAsync(m->ids, ids, (size_t)B * L * 4, cudaMemcpyHostToDevice, m->s));
  MC_CUDA(cudaMemcpyAsync(m->pad, pad, (size_t)B * L * 4, cudaMemcpyHostToDevice, m->s));
  MC_CUDA(cudaGraphLaunch(embed_graph(m, B, L), m->s));
}

// rvq_quantization over m->r (N rows, already on the device) with `levels`.
void run_quantize(mrtmc_model* m, int N, int levels) {
  mc_rvq_norm_kernel<<<N, 256, 0, m->s>>>(m->r, m->r2);
  check_launch("style rvq norm");
  for (int k = 0; k < levels; ++k) {
    const float* cb = m->codebooks + (size_t)k * m->C * kD;
    mc_rvq_dist_kernel<<<dim3(N, (m->C + 7) / 8), 256, 0, m->s>>>(m->r, m->r2, cb, m->c2 + (size_t)k * m->C, m->C,
                                                                  m->dist);
    check_launch("style rvq distances");
    mc_rvq_pick_kernel<<<N, 1024, 0, m->s>>>(m->r, m->r2, cb, m->C, m->dist, m->tok, levels, k);
    check_launch("style rvq pick");
  }
}

void check_levels(mrtmc_model* m, int levels) {
  if (levels <= 0 || levels > m->K)
    throw Error{MRTDF_ERR_INVALID, "levels must be in [1, " + std::to_string(m->K) + "]"};
}

}  // namespace

extern "C" {

int mrtmc_create(int device, int max_batch, mrtmc_model** out) {
  return guarded([&] {
    if (!out) throw Error{MRTDF_ERR_INVALID, "NULL argument"};
    *out = nullptr;
    if (max_batch <= 0 || max_batch > 64) throw Error{MRTDF_ERR_INVALID, "max_batch must be in [1, 64]"};
    MC_CUDA(cudaSetDevice(device));
    cudaDeviceProp prop;
    MC_CUDA(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10)
      throw Error{MRTDF_ERR_CUDA, std::string("the style path needs an sm_100 (B200) device, found ") + prop.name};
    std::unique_ptr<mrtmc_model> m(new mrtmc_model());
    m->device = device;
    m->max_batch = max_batch;
    m->num_sms = prop.multiProcessorCount;
    MC_CUDA(cudaStreamCreateWithFlags(&m->s, cudaStreamNonBlocking));
    MC_CUDA(cudaFuncSetAttribute(mc_attn_text_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)attn_text_smem()));
    const size_t M = (size_t)max_batch * kMaxLen;
    m->ids = (int32_t*)m->alloc(M * 4);
    m->pad = (float*)m->alloc(M * 4);
    m->mask = (float*)m->alloc(M * 4);
    m->x = (float*)m->alloc(M * kD * 4);
    m->h = (float*)m->alloc(M * kD * 4);
    m->ctx = (float*)m->alloc(M * kD * 4);
    m->qkv = (float*)m->alloc(M * kQkv * 4);
    m->f = (float*)m->alloc(M * kFF * 4);
    m->kv = (float*)m->alloc(M * 2 * kPoolInner * 4);
    m->pctx = (float*)m->alloc((size_t)max_batch * kPoolInner * 4);
    m->out = (float*)m->alloc((size_t)max_batch * kD * 4);
    // split-K scratch: the largest partial set over the plan's GEMM shapes at
    // every row count up to capacity
    size_t part = 0;
    for (int rows = 1; rows <= (int)M; ++rows) {
      part = std::max(part, gemm_part_floats(rows, kQkv, kD, m->num_sms));
      part = std::max(part, gemm_part_floats(rows, kD, kD, m->num_sms));
      part = std::max(part, gemm_part_floats(rows, kFF, kD, m->num_sms));
      part = std::max(part, gemm_part_floats(rows, kD, kFF, m->num_sms));
      part = std::max(part, gemm_part_floats(rows, 2 * kPoolInner, kD, m->num_sms));
      part = std::max(part, gemm_part_floats(rows, kD, kPoolInner, m->num_sms));
      part = std::max(part, gemm_part_floats(rows, kPoolInner, kD, m->num_sms));
    }
    m->part_floats = std::max<size_t>(part, 1);
    m->part = (float*)m->alloc(m->part_floats * 4);
    m->r = (float*)m->alloc((size_t)kMaxQuantRows * kD * 4);
    m->r2 = (float*)m->alloc((size_t)kMaxQuantRows * 4);
    m->tok = (int32_t*)m->alloc((size_t)kMaxQuantRows * 64 * 4);
    m->err = (int*)m->alloc(sizeof(int));
    MC_CUDA(cudaMemset(m->err, 0, sizeof(int)));
    *out = m.release();
  });
}

void mrtmc_destroy(mrtmc_model* m) { delete m; }

int mrtmc_load_safetensors(mrtmc_model* m, const char* encoder_path, const char* codebooks_path) {
  return guarded([&] {
    if (!m || !encoder_path || !codebooks_path) throw Error{MRTDF_ERR_INVALID, "NULL argument"};
    MC_CUDA(cudaSetDevice(m->device));
    SafetensorsFile fe(encoder_path);
    SafetensorsFile fc(codebooks_path);
    std::vector<float> conv;
    auto get = [&](const SafetensorsFile& f, const char* path, const std::string& key,
                   const std::vector<int64_t>& shape) -> std::vector<float> {
      const TensorRef* t = f.find(key);
      if (!t) throw Error{MRTDF_ERR_KEY, "WeightBundle " + std::string(path) + ": missing key \"" + key + "\""};
      int64_t n = 1;
      for (auto d : shape) n *= d;
      if (t->numel() != n) throw Error{MRTDF_ERR_INVALID, "shape mismatch for " + key};
      std::vector<float> v((size_t)n);
      if (t->dtype == "F32") {
        std::memcpy(v.data(), t->data, (size_t)n * 4);
      } else if (t->dtype == "BF16") {
        const uint16_t* s = reinterpret_cast<const uint16_t*>(t->data);
        for (int64_t i = 0; i < n; ++i) {
          const uint32_t u = (uint32_t)s[i] << 16;
          std::memcpy(&v[(size_t)i], &u, 4);
        }
      } else {
        throw Error{MRTDF_ERR_INVALID, "unsupported dtype " + t->dtype + " for " + key};
      }
      return v;
    };
    auto up = [&](const std::vector<float>& v) {
      float* d = (float*)m->alloc(v.size() * 4);
      MC_CUDA(cudaMemcpy(d, v.data(), v.size() * 4, cudaMemcpyHostToDevice));
      return d;
    };
    auto enc = [&](const std::string& key, const std::vector<int64_t>& shape) {
      return get(fe, encoder_path, key, shape);
    };
    // one set of weights per model (create another model for another bundle)
    if (m->loaded) throw Error{MRTDF_ERR_STATE, "the style model's weights are already loaded"};
    const TensorRef* te = fe.find("token_embedding.weight");
    if (!te) throw Error{MRTDF_ERR_KEY, "WeightBundle " + std::string(encoder_path) + ": missing key \"token_embedding.weight\""};
    if (te->shape.size() != 2 || te->shape[1] != kD)
      throw Error{MRTDF_ERR_INVALID, "token_embedding.weight must be (V, 768)"};
    m->V = (int)te->shape[0];
    m->emb = up(enc("token_embedding.weight", {m->V, kD}));
    auto lin_cat = [&](const std::string& p, const char* const* names, int parts, int out, int in, float** w,
                       float** b) {
      std::vector<float> W, Bv;
      for (int i = 0; i < parts; ++i) {
        const auto wi = enc(p + names[i] + ".weight", {out, in});
        const auto bi = enc(p + names[i] + ".bias", {out});
        W.insert(W.end(), wi.begin(), wi.end());
        Bv.insert(Bv.end(), bi.begin(), bi.end());
      }
      *w = up(W);
      *b = up(Bv);
    };
    static const char* const kQkvNames[3] = {"q_proj", "k_proj", "v_proj"};
    static const char* const kKvNames[2] = {"k_proj", "v_proj"};
    static const char* const kO[1] = {"o_proj"};
    static const char* const kEmpty[1] = {""};
    for (int l = 0; l < kLayers; ++l) {
      const std::string p = "text_layers." + std::to_string(l) + ".";
      McLayer& Ly = m->layers[l];
      Ly.ln1_w = up(enc(p + "attn_ln.weight", {kD}));
      Ly.ln1_b = up(enc(p + "attn_ln.bias", {kD}));
      Ly.ln2_w = up(enc(p + "ffn_ln.weight", {kD}));
      Ly.ln2_b = up(enc(p + "ffn_ln.bias", {kD}));
      lin_cat(p + "attn.", kQkvNames, 3, kHeads * kDHead, kD, &Ly.wqkv, &Ly.bqkv);
      lin_cat(p + "attn.", kO, 1, kD, kHeads * kDHead, &Ly.wo, &Ly.bo);
      lin_cat(p + "ffn_w1", kEmpty, 1, kFF, kD, &Ly.w1, &Ly.b1);
      lin_cat(p + "ffn_w2", kEmpty, 1, kD, kFF, &Ly.w2, &Ly.b2);
    }
    m->exit_w = up(enc("text_exit_ln.weight", {kD}));
    m->exit_b = up(enc("text_exit_ln.bias", {kD}));
    m->pool_ln_w = up(enc("text_pooler.ln.weight", {kD}));
    m->pool_ln_b = up(enc("text_pooler.ln.bias", {kD}));
    lin_cat("text_pooler.attn.", kKvNames, 2, kPoolInner, kD, &m->pool_wkv, &m->pool_bkv);
    lin_cat("text_pooler.attn.", kO, 1, kD, kPoolInner, &m->pool_wo, &m->pool_bo);
    // the learned query is input-independent: project it once here
    // (q_proj(query) * softplus(s) / ln 2, musiccoca.cpp:144-158)
    float *wq = nullptr, *bq = nullptr;
    static const char* const kQ[1] = {"q_proj"};
    lin_cat("text_pooler.attn.", kQ, 1, kPoolInner, kD, &wq, &bq);
    const auto query = enc("text_pooler.query", {1, 1, kD});
    const auto pds = enc("text_pooler.attn._per_dim_scale", {kPoolDHead});
    std::vector<float> sc(kPoolDHead);
    for (int d = 0; d < kPoolDHead; ++d) {
      const float x = pds[d];
      const float sp = std::max(x, 0.0f) + std::log1p(std::exp(-std::fabs(x)));  // softplus (musiccoca.cpp:50-55)
      sc[d] = sp / std::log(2.0f);
    }
    float* dq = up(query);
    float* dsc = up(sc);
    m->pool_q = (float*)m->alloc((size_t)kPoolInner * 4);
    m->launches = 0;
    gemm(m, dq, kD, wq, bq, m->pool_q, kPoolInner, 1, kPoolInner, kD, kMcStore);
    mc_scale_query_kernel<<<(kPoolInner + 255) / 256, 256, 0, m->s>>>(m->pool_q, dsc);
    check_launch("style query scale");
    // codebooks (K, C, 768) and |c|^2 in index order
    const TensorRef* tc = fc.find("codebooks");
    if (!tc) throw Error{MRTDF_ERR_KEY, "WeightBundle " + std::string(codebooks_path) + ": missing key \"codebooks\""};
    if (tc->shape.size() != 3 || tc->shape[2] != kD)
      throw Error{MRTDF_ERR_INVALID, "codebooks must be (K, C, 768)"};
    m->K = (int)tc->shape[0];
    m->C = (int)tc->shape[1];
    if (m->K <= 0 || m->K > 64 || m->C <= 0) throw Error{MRTDF_ERR_INVALID, "codebooks must have 1..64 levels"};
    const auto cbv = get(fc, codebooks_path, "codebooks", {m->K, m->C, kD});
    std::vector<float> c2((size_t)m->K * m->C);
    for (size_t i = 0; i < c2.size(); ++i) {
      float s = 0.f;
      for (int k = 0; k < kD; ++k) s += cbv[i * kD + k] * cbv[i * kD + k];
      c2[i] = s;
    }
    m->codebooks = up(cbv);
    m->c2 = up(c2);
    m->dist = (float*)m->alloc((size_t)kMaxQuantRows * m->C * 4);
    MC_CUDA(cudaStreamSynchronize(m->s));
    m->loaded = true;
  });
}

int mrtmc_embed_text(mrtmc_model* m, const int32_t* ids, const float* pad, int B, int L, float* out) {
  return guarded([&] {
    require_loaded(m);
    if (!out) throw Error{MRTDF_ERR_INVALID, "NULL argument"};
    MC_CUDA(cudaSetDevice(m->device));
    run_embed(m, ids, pad, B, L);
    MC_CUDA(cudaMemcpyAsync(out, m->out, (size_t)B * kD * 4, cudaMemcpyDeviceToHost, m->s));
    sync_and_check(m);
  });
}

int mrtmc_quantize(mrtmc_model* m, const float* emb, int N, int levels, int32_t* tokens) {
  return guarded([&] {
    require_loaded(m);
    if (!emb || !tokens) throw Error{MRTDF_ERR_INVALID, "NULL argument"};
    if (N <= 0 || N > kMaxQuantRows) throw Error{MRTDF_ERR_RANGE, "quantize: N must be in [1, 1024]"};
    check_levels(m, levels);
    MC_CUDA(cudaSetDevice(m->device));
    MC_CUDA(cudaMemcpyAsync(m->r, emb, (size_t)N * kD * 4, cudaMemcpyHostToDevice, m->s));
    run_quantize(m, N, levels);
    MC_CUDA(cudaMemcpyAsync(tokens, m->tok, (size_t)N * levels * 4, cudaMemcpyDeviceToHost, m->s));
    sync_and_check(m);
  });
}

int mrtmc_style_tokens(mrtmc_model* m, const int32_t* ids, const float* pad, int B, int L,
                       int encoder_style_rvq_depth, int style_rvq_codebook_size, int vocab_style_offset,
                       int32_t* out) {
  return guarded([&] {
    require_loaded(m);
    if (!out) throw Error{MRTDF_ERR_INVALID, "NULL argument"};
    check_levels(m, encoder_style_rvq_depth);
    MC_CUDA(cudaSetDevice(m->device));
    run_embed(m, ids, pad, B, L);
    MC_CUDA(cudaMemcpyAsync(m->r, m->out, (size_t)B * kD * 4, cudaMemcpyDeviceToDevice, m->s));
    run_quantize(m, B, encoder_style_rvq_depth);
    std::vector<int32_t> tok((size_t)B * encoder_style_rvq_depth);
    MC_CUDA(cudaMemcpyAsync(tok.data(), m->tok, tok.size() * 4, cudaMemcpyDeviceToHost, m->s));
    sync_and_check(m);
    // rvq_to_llm (rvq.cpp:105-110) at the style offset
    for (int b = 0; b < B; ++b)
      for (int k = 0; k < encoder_style_rvq_depth; ++k)
        out[(size_t)b * encoder_style_rvq_depth + k] =
            vocab_style_offset + k * style_rvq_codebook_size + tok[(size_t)b * encoder_style_rvq_depth + k];
  });
}

void* mrtmc_cuda_stream(mrtmc_model* m) { return m ? (void*)m->s : nullptr; }

long long mrtmc_embed_kernels(mrtmc_model* m, int B, int L) {
  if (!m || !m->loaded || B <= 0 || B > m->max_batch || L <= 0 || L > kMaxLen) return -1;
  try {
    embed_graph(m, B, L);
    return m->graph_launches[std::make_pair(B, L)];
  } catch (...) {
    return -1;
  }
}

}  // extern "C"
