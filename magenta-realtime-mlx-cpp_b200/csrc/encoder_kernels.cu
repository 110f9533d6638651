// Encoder kernels: embedding + sinusoidal position add, row RMSNorm, the
// projection GEMMs with fused epilogues, and full (unmasked) attention.
//
// Reference semantics (rhymeswithlion/magenta-realtime-mlx-cpp):
//   Depthformer::encode  depthformer/model.cpp:226-241
//   EncoderLayer         depthformer/modules.cpp:349-358 (pre-norm self
//                        attention, no mask, no bias, scale 1.0; gated FFN)
//   project_kv           modules.cpp:323-333 (cross K/V, done for all 20
//                        temporal layers in one GEMM with N = Lt * 2 * inner)
// bf16 GEMMs run on tcgen05 (gemm_tc.cu); the fp32 GEMM here runs on the
// CUDA cores so the fp32 parity mode stays exact fp32. The encoder attention
// uses mma.sync m16n8k16 with fp32 accumulation.
#include <cuda_bf16.h>

#include "common.cuh"
#include "encoder_kernels.cuh"
#include "gemm_epilogue.cuh"

namespace mrtdf {

typedef __nv_bfloat16 bf16;

// ---------------------------------------------------------------------------
// PTX helpers of the encoder attention (cp.async, ldmatrix, mma.sync)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool pred) {
  const int src = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(gmem), "r"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void mma_bf16(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

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

// ---------------------------------------------------------------------------
// Encoder self-attention, bf16: flash-attention style. CTA = 64 queries of
// one (row, head), 4 warps x 16 query rows; K/V tiles of 64 keys
// double-buffered by cp.async; S = Q K^T and O += P V on mma.sync; online
// softmax in fp32 (scale 1.0, no mask).
// ---------------------------------------------------------------------------
__device__ __forceinline__ int swz64(int row, int chunk) { return row * 64 + ((chunk ^ (row & 7)) << 3); }

__global__ void __launch_bounds__(128) enc_attn_bf16_kernel(const EncAttnParams p) {
  __shared__ __align__(128) bf16 sQ[64 * 64];
  __shared__ __align__(128) bf16 sK[2][64 * 64];
  __shared__ __align__(128) bf16 sV[2][64 * 64];
  pdl_launch_dependents();
  pdl_wait();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int q0 = blockIdx.x * 64;
  const int bh = blockIdx.y, b = bh / p.H, h = bh - b * p.H;
  const int ld = 3 * p.inner;
  const bf16* base = reinterpret_cast<const bf16*>(p.qkv) + (size_t)b * p.S * ld;
  const bf16* Qg = base + h * 64;
  const bf16* Kg = base + p.inner + h * 64;
  const bf16* Vg = base + 2 * p.inner + h * 64;

  // Q tile
  for (int i = tid; i < 64 * 8; i += 128) {
    const int r = i >> 3, ch = i & 7;
    const int qr = q0 + r;
    cp_async16(sQ + swz64(r, ch), Qg + (size_t)min(qr, p.S - 1) * ld + ch * 8, qr < p.S);
  }
  auto load_kv = [&](int buf, int k0) {
    for (int i = tid; i < 64 * 8; i += 128) {
      const int r = i >> 3, ch = i & 7;
      const int kr = k0 + r;
      const bool ok = kr < p.S;
      const size_t off = (size_t)min(kr, p.S - 1) * ld + ch * 8;
      cp_async16(sK[buf] + swz64(r, ch), Kg + off, ok);
      cp_async16(sV[buf] + swz64(r, ch), Vg + off, ok);
    }
  };
  load_kv(0, 0);
  cp_async_commit();

  const int g = lane >> 2, t = lane & 3;
  float o[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) o[i][j] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
  uint32_t qf[4][4];
  const int nkb = (p.S + 63) / 64;
  for (int kb = 0; kb < nkb; ++kb) {
    if (kb + 1 < nkb) load_kv((kb + 1) & 1, (kb + 1) * 64);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (kb == 0) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const int row = warp * 16 + (lane & 15);
        const int ch = kk * 2 + (lane >> 4);
        ldsm_x4(qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], sQ + swz64(row, ch));
      }
    }
    const bf16* Ks = sK[kb & 1];
    const bf16* Vs = sV[kb & 1];
    float s[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[i][j] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int nj = 0; nj < 4; ++nj) {
        uint32_t b0, b1, b2, b3;
        const int row = nj * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int ch = kk * 2 + ((lane >> 3) & 1);
        ldsm_x4(b0, b1, b2, b3, Ks + swz64(row, ch));
        mma_bf16(s[2 * nj], qf[kk], b0, b1);
        mma_bf16(s[2 * nj + 1], qf[kk], b2, b3);
      }
    }
    // mask keys past the sequence end
    const int kbase = kb * 64;
#pragma unroll
    for (int ni = 0; ni < 8; ++ni) {
      const int c0 = kbase + ni * 8 + 2 * t;
      if (c0 >= p.S) { s[ni][0] = -INFINITY; s[ni][2] = -INFINITY; }
      if (c0 + 1 >= p.S) { s[ni][1] = -INFINITY; s[ni][3] = -INFINITY; }
    }
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int ni = 0; ni < 8; ++ni) {
      mx[0] = fmaxf(mx[0], fmaxf(s[ni][0], s[ni][1]));
      mx[1] = fmaxf(mx[1], fmaxf(s[ni][2], s[ni][3]));
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
    }
    float scale[2], nm[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      nm[r] = fmaxf(m_r[r], mx[r]);
      scale[r] = (m_r[r] == -INFINITY) ? 0.f : __expf(m_r[r] - nm[r]);
      m_r[r] = nm[r];
    }
    // P is split as P_hi + P_lo with both halves bf16 (P_lo = bf16(P -
    // P_hi)), and O += P_hi V + P_lo V: the probabilities keep ~16 mantissa
    // bits, so the tensor-core result matches softmax in fp32.
    float ls[2] = {0.f, 0.f};
    uint32_t pf[4][4], pl[4][4];
#pragma unroll
    for (int ni = 0; ni < 8; ++ni) {
      const float p0 = __expf(s[ni][0] - nm[0]), p1 = __expf(s[ni][1] - nm[0]);
      const float p2 = __expf(s[ni][2] - nm[1]), p3 = __expf(s[ni][3] - nm[1]);
      ls[0] += p0 + p1;
      ls[1] += p2 + p3;
      const int kk = ni >> 1;
      const int slot = (ni & 1) * 2;
      const uint32_t h01 = pack_bf16(p0, p1), h23 = pack_bf16(p2, p3);
      pf[kk][slot] = h01;
      pf[kk][slot + 1] = h23;
      const float r0 = p0 - __uint_as_float(h01 << 16), r1 = p1 - __uint_as_float(h01 & 0xffff0000u);
      const float r2 = p2 - __uint_as_float(h23 << 16), r3 = p3 - __uint_as_float(h23 & 0xffff0000u);
      pl[kk][slot] = pack_bf16(r0, r1);
      pl[kk][slot + 1] = pack_bf16(r2, r3);
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      ls[r] += __shfl_xor_sync(0xffffffffu, ls[r], 1);
      ls[r] += __shfl_xor_sync(0xffffffffu, ls[r], 2);
      l_r[r] = l_r[r] * scale[r] + ls[r];
    }
#pragma unroll
    for (int ni = 0; ni < 8; ++ni) {
      o[ni][0] *= scale[0];
      o[ni][1] *= scale[0];
      o[ni][2] *= scale[1];
      o[ni][3] *= scale[1];
    }
    // O += P V: V tile [key][dim], B operand via ldmatrix.trans
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int nj = 0; nj < 4; ++nj) {
        uint32_t b0, b1, b2, b3;
        const int krow = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
        const int ch = nj * 2 + (lane >> 4);
        ldsm_x4_t(b0, b1, b2, b3, Vs + swz64(krow, ch));
        mma_bf16(o[2 * nj], pf[kk], b0, b1);
        mma_bf16(o[2 * nj + 1], pf[kk], b2, b3);
        mma_bf16(o[2 * nj], pl[kk], b0, b1);
        mma_bf16(o[2 * nj + 1], pl[kk], b2, b3);
      }
    }
    __syncthreads();
  }
  bf16* out = reinterpret_cast<bf16*>(p.out) + (size_t)b * p.S * p.inner + h * 64;
  const int r0 = q0 + warp * 16 + g;
#pragma unroll
  for (int ni = 0; ni < 8; ++ni) {
    const int cc = ni * 8 + 2 * t;
    if (r0 < p.S) {
      out[(size_t)r0 * p.inner + cc] = __float2bfloat16_rn(o[ni][0] / l_r[0]);
      out[(size_t)r0 * p.inner + cc + 1] = __float2bfloat16_rn(o[ni][1] / l_r[0]);
    }
    if (r0 + 8 < p.S) {
      out[(size_t)(r0 + 8) * p.inner + cc] = __float2bfloat16_rn(o[ni][2] / l_r[1]);
      out[(size_t)(r0 + 8) * p.inner + cc + 1] = __float2bfloat16_rn(o[ni][3] / l_r[1]);
    }
  }
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
  if (dtype == 1) {
    const dim3 grid((p.S + 63) / 64, p.B * p.H);
    return launch_k(enc_attn_bf16_kernel, grid, dim3(128), 0, s, pdl, p);
  }
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
