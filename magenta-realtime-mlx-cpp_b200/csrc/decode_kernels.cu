// Decode-step kernels for sm_100a: the GEMV phase kernel behind every
// projection of temporal_step / depth_step, single-query attention (self
// with relative-position bias, split-K cross attention), and the fused
// CFG + vocab-mask + temperature + top-k + Gumbel-max sampler.
//
// Reference semantics (rhymeswithlion/magenta-realtime-mlx-cpp):
//   RMSNorm            depthformer/modules.cpp:72-84 (eps 1e-6, 342-346)
//   Linear             modules.cpp:98-100 (bias-free, W stored (out, in))
//   MHA (scale 1.0)    modules.cpp:243-321 (SDPA with additive bias)
//   KV append          modules.cpp:271-275, 428-429
//   Gated FFN          modules.cpp:222-226 + gelu_approx nn_ops.h:66-84
//   DecoderLayer       modules.cpp:384-408
//   sampling           decode.cpp:71-148, 465-477, 484
// In bf16 mode every op output is rounded to bf16 as MLX does; reductions
// accumulate in fp32.
#include <cuda_bf16.h>

#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "decode_device.cuh"
#include "decode_kernels.cuh"

namespace mrtdf {

constexpr int kSelfAttnMaxT = 64;  // keys of a decode self-attention (2 chunks of 32)

// ---------------------------------------------------------------------------
// GEMV phase kernel
//
// One CTA per SM. CTA c owns the contiguous unit range
// [c * units / G, (c + 1) * units / G) of the weight matrix; its rows are one
// contiguous byte range in HBM, streamed into shared memory by the TMA
// engine (cp.async.bulk) through a ring of kGemvStages buffers. The first
// stages are issued BEFORE griddepcontrol.wait, so under programmatic
// dependent launch the weight fetch overlaps the previous kernel. The input
// vector (B rows, optionally RMS-normalised) is read after the wait and kept
// in shared memory as float. Each warp reduces whole rows with 16-byte
// shared loads and a shuffle reduction; the epilogue is fused.
// ---------------------------------------------------------------------------
template <typename T, int BMAX, bool NORM, int MODE>
__global__ void __launch_bounds__(kGemvThreads) gemv_phase_kernel(const GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int RPU = (MODE == kGemvGeglu) ? 2 : 1;
  constexpr int EPC = Vec16<T>::N;
  uint8_t* stage_buf = smem;
  float* xs = reinterpret_cast<float*>(smem + kGemvStages * kGemvStageBytes);
  uint64_t* bars =
      reinterpret_cast<uint64_t*>(smem + kGemvStages * kGemvStageBytes + (((size_t)p.B * p.cols * 4 + 15) & ~15));
  __shared__ float red[kGemvThreads / 32][BMAX];
  __shared__ float rstd[BMAX];
  __shared__ int ok_flag;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = gridDim.x, c = blockIdx.x;
  const int u0 = (int)(((long long)c * p.units) / G);
  const int u1 = (int)(((long long)(c + 1) * p.units) / G);
  const int nunits = u1 - u0;
  const int unit_bytes = RPU * p.cols * (int)sizeof(T);
  const int ups = kGemvStageBytes / unit_bytes;  // host guarantees >= 1
  const int nstages = (nunits + ups - 1) / ups;
  const uint8_t* wbase = reinterpret_cast<const uint8_t*>(p.W) + (size_t)u0 * unit_bytes;

  auto issue = [&](int s) {
    const int first = s * ups;
    const int n = min(ups, nunits - first);
    const uint32_t bytes = (uint32_t)(n * unit_bytes);
    uint64_t* bar = &bars[s % kGemvStages];
    mbar_arrive_expect_tx(bar, bytes);
    bulk_g2s(stage_buf + (size_t)(s % kGemvStages) * kGemvStageBytes, wbase + (size_t)first * unit_bytes, bytes, bar);
  };

  if (tid == 0) {
    for (int i = 0; i < kGemvStages; ++i) mbar_init(&bars[i], 1);
    fence_mbar_init();
    ok_flag = 1;
  }
  __syncthreads();
  if (tid == 0) {
    for (int s = 0; s < min(kGemvStages, nstages); ++s) issue(s);
  }
  pdl_launch_dependents();
  pdl_wait();

  // ---- input vector -> shared memory (optionally RMS-normalised) ----------
  const T* x = reinterpret_cast<const T*>(p.x);
  float ss[BMAX];
#pragma unroll
  for (int b = 0; b < BMAX; ++b) ss[b] = 0.f;
#pragma unroll
  for (int b = 0; b < BMAX; ++b) {
    if (b < p.B) {
      for (int i = tid; i < p.cols; i += kGemvThreads) {
        const float v = to_f(x[(size_t)b * p.x_stride + i]);
        xs[(size_t)b * p.cols + i] = v;
        if (NORM) ss[b] += v * v;
      }
    }
  }
  if (NORM) {
#pragma unroll
    for (int b = 0; b < BMAX; ++b) {
      const float v = warp_sum(ss[b]);
      if (lane == 0) red[warp][b] = v;
    }
    __syncthreads();
    if (tid < BMAX) {
      float t = 0.f;
      for (int w = 0; w < kGemvThreads / 32; ++w) t += red[w][tid];
      rstd[tid] = __frcp_rn(__fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)p.cols), 1e-6f)));
    }
    __syncthreads();
    const T* nw = reinterpret_cast<const T*>(p.norm_w);
#pragma unroll
    for (int b = 0; b < BMAX; ++b) {
      if (b < p.B) {
        const float r = rstd[b];
        for (int i = tid; i < p.cols; i += kGemvThreads) {
          const float v = xs[(size_t)b * p.cols + i];
          xs[(size_t)b * p.cols + i] = rnd<T>(__fmul_rn(to_f(nw[i]), rnd<T>(__fmul_rn(v, r))));
        }
      }
    }
  }
  __syncthreads();

  const int nchunk = p.cols / EPC;
  for (int s = 0; s < nstages; ++s) {
    if (tid == 0) ok_flag = mbar_wait_bounded(&bars[s % kGemvStages], (uint32_t)((s / kGemvStages) & 1), p.err);
    __syncthreads();
    if (!ok_flag) break;
    const uint8_t* buf = stage_buf + (size_t)(s % kGemvStages) * kGemvStageBytes;
    const int first = s * ups;
    const int n_u = min(ups, nunits - first);
    for (int uu = warp; uu < n_u; uu += kGemvThreads / 32) {
      float acc[RPU][BMAX];
#pragma unroll
      for (int r = 0; r < RPU; ++r)
#pragma unroll
        for (int b = 0; b < BMAX; ++b) acc[r][b] = 0.f;
      const uint8_t* urow = buf + (size_t)uu * unit_bytes;
      for (int ch = lane; ch < nchunk; ch += 32) {
        float wv[RPU][EPC];
#pragma unroll
        for (int r = 0; r < RPU; ++r) {
          const uint4 raw = *reinterpret_cast<const uint4*>(urow + (size_t)r * p.cols * sizeof(T) + (size_t)ch * 16);
          Vec16<T>::unpack(raw, wv[r]);
        }
#pragma unroll
        for (int b = 0; b < BMAX; ++b) {
          if (b < p.B) {
            const float* xv = xs + (size_t)b * p.cols + (size_t)ch * EPC;
            float xr[EPC];
#pragma unroll
            for (int e = 0; e < EPC; e += 4) {
              const float4 f4 = *reinterpret_cast<const float4*>(xv + e);
              xr[e] = f4.x;
              xr[e + 1] = f4.y;
              xr[e + 2] = f4.z;
              xr[e + 3] = f4.w;
            }
#pragma unroll
            for (int r = 0; r < RPU; ++r)
#pragma unroll
              for (int e = 0; e < EPC; ++e) acc[r][b] = fmaf(wv[r][e], xr[e], acc[r][b]);
          }
        }
      }
#pragma unroll
      for (int r = 0; r < RPU; ++r)
#pragma unroll
        for (int b = 0; b < BMAX; ++b) acc[r][b] = warp_sum(acc[r][b]);

      const int u = u0 + first + uu;
#pragma unroll
      for (int b = 0; b < BMAX; ++b) {
        if (b < p.B && lane == b) {
          if (MODE == kGemvStore) {
            reinterpret_cast<T*>(p.out)[(size_t)b * p.out_stride + p.out_offset + u] = from_f<T>(acc[0][b]);
          } else if (MODE == kGemvLogits) {
            reinterpret_cast<float*>(p.out)[(size_t)b * p.out_stride + p.out_offset + u] = rnd<T>(acc[0][b]);
          } else if (MODE == kGemvResid) {
            const float rv = to_f(reinterpret_cast<const T*>(p.resid)[(size_t)b * p.resid_stride + u]);
            reinterpret_cast<T*>(p.out)[(size_t)b * p.out_stride + u] = from_f<T>(__fadd_rn(rv, rnd<T>(acc[0][b])));
          } else if (MODE == kGemvGeglu) {
            const float a = rnd<T>(acc[0][b]);
            const float g = rnd<T>(acc[1][b]);
            reinterpret_cast<T*>(p.out)[(size_t)b * p.out_stride + u] = from_f<T>(__fmul_rn(gelu_approx<T>(a), g));
          } else {  // kGemvQKV: head-major rows (h, q|k|v, 64)
            const int h = u / kQkvRowsPerHead, rr = u - h * kQkvRowsPerHead;
            const int sect = rr >> 6, cc = rr & 63;
            if (sect == 0) {
              reinterpret_cast<T*>(p.out)[(size_t)b * p.out_stride + h * 64 + cc] = from_f<T>(acc[0][b]);
            } else {
              T* cache = reinterpret_cast<T*>(sect == 1 ? p.kc : p.vc);
              cache[(((size_t)b * p.H + h) * p.cap + p.pos) * 64 + cc] = from_f<T>(acc[0][b]);
            }
          }
        }
      }
    }
    __syncthreads();  // every warp is done with this buffer
    if (tid == 0 && s + kGemvStages < nstages) issue(s + kGemvStages);
  }
  if (!ok_flag && tid == 0) {
    // Give in-flight copies a bounded chance to land before the CTA exits.
    for (int s = 0; s < nstages; ++s) mbar_wait_bounded(&bars[s % kGemvStages], (uint32_t)((s / kGemvStages) & 1), nullptr);
  }
}

// ---------------------------------------------------------------------------
// bf16 GEMV phase on the tensor cores.
//
// CTA c owns units [c * units / G, (c + 1) * units / G): R rows of W, one
// contiguous HBM range. Before griddepcontrol.wait the CTA
//   * issues one TMA bulk copy per row into shared memory with a 16-byte row
//     pad (so 8-row ldmatrix reads are bank-conflict free), all in flight at
//     once, with an L2 eviction-priority hint (depth weights kept, temporal
//     weights streamed);
//   * loads its RMSNorm scale slice into registers.
// After the wait it stages the input rows (RMS-normalised with the
// reference's rounding) as bf16 in shared memory, lets the next kernel launch
// (griddepcontrol.launch_dependents), then computes
// Y[R, B] = W_slice[R, cols] . X^T with mma.sync m16n8k16 (rows as M, the
// batch rows as N = 8, k split over the 8 warps), reduces the per-warp
// partials through shared memory and applies the fused epilogue.
// ---------------------------------------------------------------------------
constexpr int kMmaMaxRows = 32;  // 4 n8 tiles of weight rows per CTA

struct MmaLayout {
  int rstride;       // bytes per padded row (weights and inputs)
  int w_bytes;       // max_rows * rstride, rounded up to 128
  int x_bytes;       // 8 * rstride
  int red_bytes;     // 8 warps * 8 n-tiles * 8 rows * 8 batch floats
  int total;
};

__host__ __device__ inline MmaLayout mma_layout(int cols, int max_rows) {
  MmaLayout L;
  L.rstride = cols * 2 + 16;
  L.w_bytes = ((max_rows * L.rstride) + 127) & ~127;
  L.x_bytes = ((8 * L.rstride) + 127) & ~127;
  L.red_bytes = 8 * 8 * 8 * 8 * 4;
  L.total = L.w_bytes + L.x_bytes + L.red_bytes + 64;
  return L;
}

// ---- thread-block cluster helpers (kGemvQKVCluster) ----------------------
constexpr int kClusterRows = kQkvRowsPerHead / kQkvCluster;  // q/k/v rows per CTA
// Shared memory appended to the GEMV layout: the new q, k, v of the (row,
// head) this CTA attends (192 floats, written by every CTA of the cluster),
// the attention weights (kSelfAttnMaxT floats) and the head's cached keys /
// values before this position (2 x (kSelfAttnMaxT - 1) x 64 bf16).
constexpr int kClusterOffAttF = 0;
constexpr int kClusterOffP = kClusterOffAttF + 192 * 4;
constexpr int kClusterOffKVStart = kClusterOffP + kSelfAttnMaxT * 4;
constexpr int kClusterOffKV = (kClusterOffKVStart + 127) & ~127;
constexpr int kClusterKVStride = 64 * 2 + 16;  // padded row: conflict-free per-lane key rows
constexpr int kClusterKVBytes = (kSelfAttnMaxT - 1) * kClusterKVStride;
constexpr int kClusterExtra = kClusterOffKV + 2 * kClusterKVBytes;

__host__ __device__ inline int cluster_ext_offset(int total) { return (total + 127) & ~127; }

template <int BMAX, int NT, bool NORM, int MODE>
__global__ void __launch_bounds__(256, 2) gemv_mma_kernel(const GemvParams p, const int max_rows) {
  typedef __nv_bfloat16 T;
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int RPU = (MODE == kGemvGeglu) ? 2 : 1;
  const MmaLayout L = mma_layout(p.cols, max_rows);
  uint8_t* wsm = smem;
  uint8_t* xsm = smem + L.w_bytes;
  float* red = reinterpret_cast<float*>(smem + L.w_bytes + L.x_bytes);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L.w_bytes + L.x_bytes + L.red_bytes);
  uint8_t* cl_ext = smem + cluster_ext_offset(L.total);  // kGemvQKVCluster only
  float* cl_recv = reinterpret_cast<float*>(cl_ext + kClusterOffAttF);
  __shared__ float wred[8][BMAX];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = gridDim.x, c = blockIdx.x;
  const int u0 = (int)(((long long)c * p.units) / G);
  const int u1 = (int)(((long long)(c + 1) * p.units) / G);
  const int R = (u1 - u0) * RPU;
  const int row_bytes = p.cols * 2;
  const int nchunk = p.cols >> 3;  // 16-byte chunks per row

  // constant RMSNorm scale slice -> registers first, ahead of the weight burst
  uint4 nw_reg[2];
  const T* x_ptr = reinterpret_cast<const T*>(p.x);
  if (NORM) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int ch = tid + i * 256;
      nw_reg[i] = ch < nchunk ? reinterpret_cast<const uint4*>(p.norm_w)[ch] : make_uint4(0, 0, 0, 0);
    }
  }
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (warp == 0 && R > 0) {
    const uint64_t pol = l2_policy(p.l2_keep != 0);
    if (lane == 0) mbar_arrive_expect_tx(bar, (uint32_t)(R * row_bytes));
    __syncwarp();
    const uint8_t* src = reinterpret_cast<const uint8_t*>(p.W) + (size_t)u0 * RPU * row_bytes;
    for (int r = lane; r < R; r += 32) bulk_g2s_hint(wsm + (size_t)r * L.rstride, src + (size_t)r * row_bytes,
                                                    (uint32_t)row_bytes, bar, pol);
  }
  // kGemvQKVCluster: the relative-position bias of this query (a table
  // written at weight load) is read ahead of the dependency wait
  float cl_bias0 = 0.f, cl_bias1 = 0.f;
  if constexpr (MODE == kGemvQKVCluster) {
    if (warp == 0 && p.bias) {
      const float* bias = p.bias + (size_t)(c / kQkvCluster) * p.bias_stride;
      if (lane < p.pos + 1) cl_bias0 = bias[lane];
      if (32 + lane < p.pos + 1) cl_bias1 = bias[32 + lane];
    }
  }
  // ---- every global load of this phase, issued back to back -------------
  // inputs: thread owns 16-byte chunks ch = tid + 256 i (i < 2: cols <= 4096)
  uint4 xin[BMAX][2];
  // RMSNorm without a CTA-wide reduction (B <= 2, cols <= 1024, a multiple
  // of 256): every warp also loads the whole rows (L1 hits after the first
  // warp) and reduces the sum of squares with shuffles alone.
  constexpr int kWJ = 4;  // row chunks per lane
  constexpr int kWB = (NORM && BMAX <= 2) ? BMAX : 1;
  uint4 wx[kWB][kWJ];
  const bool wnorm = NORM && BMAX <= 2 && (nchunk & 31) == 0 && nchunk <= 32 * kWJ && !p.acc;
  pdl_wait();
#pragma unroll
  for (int b = 0; b < BMAX; ++b)
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int ch = tid + i * 256;
      xin[b][i] = (b < p.B && ch < nchunk) ? *reinterpret_cast<const uint4*>(x_ptr + (size_t)b * p.x_stride + ch * 8)
                                          : make_uint4(0, 0, 0, 0);
    }
  if constexpr (NORM && BMAX <= 2) {
    if (wnorm) {
#pragma unroll
      for (int b = 0; b < kWB; ++b)
#pragma unroll
        for (int j = 0; j < kWJ; ++j) {
          const int ch = lane + 32 * j;
          wx[b][j] = (b < p.B && ch < nchunk) ? *reinterpret_cast<const uint4*>(x_ptr + (size_t)b * p.x_stride + ch * 8)
                                              : make_uint4(0, 0, 0, 0);
        }
    }
  }
  if (p.acc) {
    // x = R(residual + R(acc / 2^32)): the hidden state the fused decode
    // phases leave (rows of x_stride elements in both buffers)
#pragma unroll
    for (int b = 0; b < BMAX; ++b)
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int ch = tid + i * 256;
        if (b < p.B && ch < nchunk) {
          float f[8];
          Vec16<T>::unpack(xin[b][i], f);
          const longlong2* ap = reinterpret_cast<const longlong2*>(p.acc + (size_t)b * p.x_stride + ch * 8);
          uint32_t o[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const longlong2 a = ap[q];
            const float v0 = rnd<T>(__fadd_rn(f[2 * q], rnd<T>(fixed_to_float(a.x))));
            const float v1 = rnd<T>(__fadd_rn(f[2 * q + 1], rnd<T>(fixed_to_float(a.y))));
            const __nv_bfloat162 pr = __floats2bfloat162_rn(v0, v1);
            o[q] = *reinterpret_cast<const uint32_t*>(&pr);
          }
          xin[b][i] = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
  }
  // residual values of the epilogue (same thread -> (unit, row) mapping)
  const int nunits = u1 - u0;
  float resv[2];
  if (MODE == kGemvResid) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int idx = tid + i * 256;
      resv[i] = 0.f;
      if (idx < nunits * p.B) {
        const int uu = idx / p.B, b = idx - uu * p.B;
        const T* rp = reinterpret_cast<const T*>(p.resid) + (size_t)b * p.resid_stride + u0 + uu;
        resv[i] = to_f(*rp);
      }
    }
  }

  // kGemvQKVCluster: CTA rank b < B of head h's cluster attends row b; its
  // cached keys / values (positions < pos, written by earlier launches)
  // stream into shared memory while the product runs.
  if constexpr (MODE == kGemvQKVCluster) {
    const int crank = (int)cluster_ctarank(), h = c / kQkvCluster;
    if (crank < p.B) {
      const size_t base = (((size_t)crank * p.H + h) * p.cap) * 64;
      const uint8_t* Kc = reinterpret_cast<const uint8_t*>(reinterpret_cast<const T*>(p.kc) + base);
      const uint8_t* Vc = reinterpret_cast<const uint8_t*>(reinterpret_cast<const T*>(p.vc) + base);
      const int n16 = p.pos * 8;  // 16-byte chunks of pos rows of 64 bf16
      for (int i = tid; i < 2 * n16; i += 256) {
        const int k = i < n16 ? i : i - n16, row = k >> 3, part = k & 7;
        uint8_t* dst = cl_ext + kClusterOffKV + (i < n16 ? 0 : kClusterKVBytes) + row * kClusterKVStride + part * 16;
        cp_async16(dst, (i < n16 ? Kc : Vc) + (size_t)k * 16);
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  }

  // ---- inputs -> shared memory as bf16 (RMS-normalised when NORM) --------
  bool staged = false;
  if constexpr (NORM && BMAX <= 2) {
    if (wnorm) {
#pragma unroll
      for (int b = 0; b < kWB; ++b) {
        if (b < p.B) {
          float ssw = 0.f;
#pragma unroll
          for (int j = 0; j < kWJ; ++j) {
            float f[8];
            Vec16<T>::unpack(wx[b][j], f);
#pragma unroll
            for (int e = 0; e < 8; ++e) ssw = fmaf(f[e], f[e], ssw);
          }
          ssw = warp_sum(ssw);
          const float r = __frcp_rn(__fsqrt_rn(__fadd_rn(__fdiv_rn(ssw, (float)p.cols), 1e-6f)));
          const int ch = tid;  // nchunk <= 128: one chunk per thread, xin[b][0]
          if (ch < nchunk) {
            float f[8], w[8];
            Vec16<T>::unpack(xin[b][0], f);
            Vec16<T>::unpack(nw_reg[0], w);
            uint32_t o[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float a0 = rnd<T>(__fmul_rn(w[2 * e], rnd<T>(__fmul_rn(f[2 * e], r))));
              const float a1 = rnd<T>(__fmul_rn(w[2 * e + 1], rnd<T>(__fmul_rn(f[2 * e + 1], r))));
              const __nv_bfloat162 pr = __floats2bfloat162_rn(a0, a1);
              o[e] = *reinterpret_cast<const uint32_t*>(&pr);
            }
            *reinterpret_cast<uint4*>(xsm + (size_t)b * L.rstride + ch * 16) = make_uint4(o[0], o[1], o[2], o[3]);
          }
        }
      }
      staged = true;
    }
  }
  if (NORM && !staged) {
    float ss[BMAX];
#pragma unroll
    for (int b = 0; b < BMAX; ++b) {
      ss[b] = 0.f;
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        float f[8];
        Vec16<T>::unpack(xin[b][i], f);
#pragma unroll
        for (int e = 0; e < 8; ++e) ss[b] = fmaf(f[e], f[e], ss[b]);
      }
      ss[b] = warp_sum(ss[b]);
    }
    if (lane < BMAX) {
      float v = ss[0];
#pragma unroll
      for (int b = 1; b < BMAX; ++b) v = lane == b ? ss[b] : v;
      wred[warp][lane] = v;
    }
    __syncthreads();
#pragma unroll
    for (int b = 0; b < BMAX; ++b) {
      if (b < p.B) {
        float t2 = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) t2 += wred[w][b];
        const float r = __frcp_rn(__fsqrt_rn(__fadd_rn(__fdiv_rn(t2, (float)p.cols), 1e-6f)));
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int ch = tid + i * 256;
          if (ch < nchunk) {
            float f[8], w[8];
            Vec16<T>::unpack(xin[b][i], f);
            Vec16<T>::unpack(nw_reg[i], w);
            uint32_t o[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float a0 = rnd<T>(__fmul_rn(w[2 * e], rnd<T>(__fmul_rn(f[2 * e], r))));
              const float a1 = rnd<T>(__fmul_rn(w[2 * e + 1], rnd<T>(__fmul_rn(f[2 * e + 1], r))));
              const __nv_bfloat162 pr = __floats2bfloat162_rn(a0, a1);
              o[e] = *reinterpret_cast<const uint32_t*>(&pr);
            }
            *reinterpret_cast<uint4*>(xsm + (size_t)b * L.rstride + ch * 16) = make_uint4(o[0], o[1], o[2], o[3]);
          }
        }
      }
    }
  } else if (!NORM) {
#pragma unroll
    for (int b = 0; b < BMAX; ++b)
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int ch = tid + i * 256;
        if (b < p.B && ch < nchunk) *reinterpret_cast<uint4*>(xsm + (size_t)b * L.rstride + ch * 16) = xin[b][i];
      }
  }
  __syncthreads();
  // Let the next kernel launch only now: its weight prefetch then overlaps
  // this kernel's product and epilogue instead of queueing in front of the
  // latency-critical input loads above.
  pdl_launch_dependents();

  // ---- tensor-core product --------------------------------------------
  // D[16 x 8] = X[16 x 16] . W^T[16 x 8] per k-step: the batch rows are M
  // (rows >= B are zero), eight weight rows are N, so one ldmatrix.x4 of W
  // gives the B fragments of two k-steps. Warp w takes k-steps
  // [w*KS/8, (w+1)*KS/8), two k-step pairs per iteration with every load of
  // the iteration issued before its mma.
  // NT (n-tiles of 8 weight rows) is a compile-time constant: runtime
  // guards around the ldmatrix / mma blocks split the loop into small basic
  // blocks and cost ~3x in this loop. Rows past R are clamped (their results
  // are never read).
  const int KS = p.cols >> 4;
  const int k0 = (warp * KS) >> 3, k1 = ((warp + 1) * KS) >> 3;
  const int g = lane >> 2, t = lane & 3;
  const bool gval = g < p.B;
  const uint32_t xrow = smem_u32(xsm) + (uint32_t)(g * L.rstride) + (uint32_t)(4 * t);
  // Every thread waits for the weight rows itself, so no CTA barrier follows.
  // A timed-out copy is reported in the error word and the CTA carries on
  // with whatever shared memory holds (control flow stays uniform; the
  // cluster variant must reach its cluster barrier anyway).
  if (R > 0) mbar_wait_bounded(bar, 0, p.err);
  if (MODE != kGemvQKVCluster && R == 0) return;
  float acc[NT][4];
#pragma unroll
  for (int i = 0; i < NT; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  const uint32_t wbase = smem_u32(wsm);
  uint32_t rowaddr[NT];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
    rowaddr[nt] = wbase + (uint32_t)(min(nt * 8 + (lane & 7), R - 1) * L.rstride + (lane >> 3) * 16);
  // Rows g >= B of the A operand only feed rows of D that are never read,
  // so every lane loads unconditionally.
  // Software pipeline over groups of two k-steps (one ldmatrix.x4 per n-tile
  // holds both k-steps' B fragments): the loads of group i + 1 are issued
  // before the MMAs of group i, two register buffers in turn. The load after
  // the last group re-reads that group (clamped index) instead of branching.
  const int ngr = (k1 - k0) >> 1;
  uint32_t bA[NT][4], xA[4], bB[NT][4], xB[4];
  auto load_group = [&](uint32_t(&b)[NT][4], uint32_t(&x)[4], int kk) {
    const uint32_t xo = xrow + (uint32_t)(kk * 32);
    asm volatile("ld.shared.b32 %0, [%1];" : "=r"(x[0]) : "r"(xo));
    asm volatile("ld.shared.b32 %0, [%1];" : "=r"(x[1]) : "r"(xo + 16));
    asm volatile("ld.shared.b32 %0, [%1];" : "=r"(x[2]) : "r"(xo + 32));
    asm volatile("ld.shared.b32 %0, [%1];" : "=r"(x[3]) : "r"(xo + 48));
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) ldsm_x4_g(b[nt], rowaddr[nt] + (uint32_t)(kk * 32));
  };
  auto mma_group = [&](const uint32_t(&b)[NT][4], const uint32_t(&x)[4]) {
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const uint32_t a[4] = {x[2 * q], 0u, x[2 * q + 1], 0u};
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) mma_m16n8k16(acc[nt], a, b[nt][2 * q], b[nt][2 * q + 1]);
    }
  };
  if (ngr > 0) load_group(bA, xA, k0);
  int gi = 0;
  for (; gi + 2 <= ngr; gi += 2) {
    load_group(bB, xB, k0 + 2 * (gi + 1));
    mma_group(bA, xA);
    load_group(bA, xA, k0 + 2 * min(gi + 2, ngr - 1));
    mma_group(bB, xB);
  }
  if (gi < ngr) mma_group(bA, xA);
  if ((k1 - k0) & 1) {  // one k-step left
    const int ks = k1 - 1;
    uint32_t xa0, xa1;
    const uint32_t xo = xrow + (uint32_t)(ks * 32);
    asm volatile("ld.shared.b32 %0, [%1];" : "=r"(xa0) : "r"(xo));
    asm volatile("ld.shared.b32 %0, [%1];" : "=r"(xa1) : "r"(xo + 16));
    const uint32_t a[4] = {xa0, 0u, xa1, 0u};
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      uint32_t bw[4];
      ldsm_x4_g(bw, rowaddr[nt] + (uint32_t)(ks * 32));  // k-steps ks, ks + 1 (the second is unused)
      mma_m16n8k16(acc[nt], a, bw[0], bw[1]);
    }
  }
  // thread (g, t), g < B, holds D[g][2t], D[g][2t+1] of each n-tile
  if (gval) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      float* rp = red + ((size_t)(warp * 8 + nt) * 8) * BMAX;
      rp[(2 * t) * BMAX + g] = acc[nt][0];
      rp[(2 * t + 1) * BMAX + g] = acc[nt][1];
    }
  }
  __syncthreads();

  // ---- cross-warp reduction + fused epilogue: one thread per (unit, row b)
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int idx = tid + i * 256;
    if (idx >= nunits * p.B) break;
    const int uu = idx / p.B, b = idx - uu * p.B;
    float v[RPU];
#pragma unroll
    for (int q = 0; q < RPU; ++q) {
      const int rr = uu * RPU + q;
      const int nt = rr >> 3, col = rr & 7;
      float sacc = 0.f;
#pragma unroll
      for (int w = 0; w < 8; ++w) sacc += red[((w * 8 + nt) * 8 + col) * BMAX + b];
      v[q] = sacc;
    }
    const int u = u0 + uu;
    if (MODE == kGemvStore) {
      reinterpret_cast<T*>(p.out)[(size_t)b * p.out_stride + p.out_offset + u] = from_f<T>(v[0]);
    } else if (MODE == kGemvLogits) {
      reinterpret_cast<float*>(p.out)[(size_t)b * p.out_stride + p.out_offset + u] = rnd<T>(v[0]);
    } else if (MODE == kGemvResid) {
      reinterpret_cast<T*>(p.out)[(size_t)b * p.out_stride + u] = from_f<T>(__fadd_rn(resv[i], rnd<T>(v[0])));
    } else if (MODE == kGemvGeglu) {
      const float a = rnd<T>(v[0]);
      const float gg = rnd<T>(v[RPU - 1]);
      reinterpret_cast<T*>(p.out)[(size_t)b * p.out_stride + u] = from_f<T>(__fmul_rn(gelu_approx<T>(a), gg));
    } else {  // kGemvQKV / QKVAttn / QKVCluster: head-major rows (h, q|k|v, 64)
      const int h = u / kQkvRowsPerHead, rr = u - h * kQkvRowsPerHead;
      const int sect = rr >> 6, cc = rr & 63;
      const T val = from_f<T>(v[0]);
      if (sect == 0) {
        reinterpret_cast<T*>(p.out)[(size_t)b * p.out_stride + h * 64 + cc] = val;
      } else {
        T* cache = reinterpret_cast<T*>(sect == 1 ? p.kc : p.vc);
        cache[(((size_t)b * p.H + h) * p.cap + p.pos) * 64 + cc] = val;
      }
      // the head's q/k/v of row b go to CTA rank b of the cluster, which attends (b, h)
      if (MODE == kGemvQKVCluster) st_cluster_f32(cl_recv + rr, (uint32_t)b, to_f(val));
    }
  }
  if constexpr (MODE == kGemvQKVCluster) {
    // Every CTA of the head's cluster has stored its q/k/v rows of batch row
    // b into CTA rank b (distributed shared memory); after the barrier, CTA
    // b < B runs attn_self_kernel's arithmetic for (b, h) with its cached
    // keys / values. No CTA reads another's shared memory after the barrier,
    // so the others may exit.
    // each thread's cached-key copies have landed; the cluster barrier
    // (release / acquire, all threads of all CTAs) then publishes them and
    // the pushed q/k/v rows to the attending warp
    asm volatile("cp.async.wait_all;" ::: "memory");
    cluster_sync();
    const int crank = (int)cluster_ctarank(), h = c / kQkvCluster;
    if (crank < p.B && warp == 0) {
      const int b = crank, nkeys = p.pos + 1;
      const float* qn = cl_recv;
      const float* kn = cl_recv + 64;
      const float* vn = cl_recv + 128;
      float* pk = reinterpret_cast<float*>(cl_ext + kClusterOffP);
      const T* Kold = reinterpret_cast<const T*>(cl_ext + kClusterOffKV);
      const T* Vold = reinterpret_cast<const T*>(cl_ext + kClusterOffKV + kClusterKVBytes);
      const bool has_bias = p.bias != nullptr;
      float sc[2];
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const int j = cc * 32 + lane;
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        if (j < nkeys) {
#pragma unroll
          for (int ch = 0; ch < 8; ++ch) {
            float kf[8];
            if (j == nkeys - 1) {
#pragma unroll
              for (int e = 0; e < 8; ++e) kf[e] = kn[ch * 8 + e];
            } else {
              Vec16<T>::unpack(
                  reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(Kold) + (size_t)j * kClusterKVStride)[ch],
                  kf);
            }
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[e & 3] = fmaf(qn[ch * 8 + e], kf[e], acc[e & 3]);
          }
        }
        float a = (acc[0] + acc[1]) + (acc[2] + acc[3]);
        if (has_bias) a += (cc == 0 ? cl_bias0 : cl_bias1);
        sc[cc] = j < nkeys ? a : -INFINITY;
      }
      const float m = warp_max(fmaxf(sc[0], sc[1]));
      const float p0 = lane < nkeys ? expf(sc[0] - m) : 0.f;
      const float p1 = 32 + lane < nkeys ? expf(sc[1] - m) : 0.f;
      const float l = warp_sum(p0 + p1);
      pk[lane] = p0;
      pk[32 + lane] = p1;
      __syncwarp();
      // o = sum_j p_j v_j in key order (the order of attn_self_kernel)
      float o0 = 0.f, o1 = 0.f;
      const uint32_t* vrow = reinterpret_cast<const uint32_t*>(Vold) + lane;
      constexpr int kVw = kClusterKVStride / 4;  // 32-bit words per padded row
      int jv = 0;
      for (; jv + 4 <= nkeys - 1; jv += 4) {
        uint32_t bits[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) bits[q] = vrow[(size_t)(jv + q) * kVw];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float pw = pk[jv + q];
          o0 = fmaf(pw, __uint_as_float(bits[q] << 16), o0);
          o1 = fmaf(pw, __uint_as_float(bits[q] & 0xffff0000u), o1);
        }
      }
      for (; jv < nkeys - 1; ++jv) {
        const uint32_t bits = vrow[(size_t)jv * kVw];
        const float pw = pk[jv];
        o0 = fmaf(pw, __uint_as_float(bits << 16), o0);
        o1 = fmaf(pw, __uint_as_float(bits & 0xffff0000u), o1);
      }
      {  // the newest key
        const float pw = pk[nkeys - 1];
        o0 = fmaf(pw, vn[2 * lane], o0);
        o1 = fmaf(pw, vn[2 * lane + 1], o1);
      }
      T* out = reinterpret_cast<T*>(p.attn_out) + (size_t)b * p.inner + h * 64;
      out[2 * lane] = from_f<T>(o0 / l);
      out[2 * lane + 1] = from_f<T>(o1 / l);
    }
  }
}

// Grid for the tensor-core GEMV: at least one CTA per SM when there are
// enough units, and no CTA with more rows than fit its shared memory.
static void mma_plan(int units, int rpu, int cols, int num_sms, int* grid, int* max_rows) {
  const int rstride = cols * 2 + 16;
  int cap_rows = (190 * 1024) / rstride;
  cap_rows = min(cap_rows, kMmaMaxRows);
  cap_rows -= cap_rows % rpu;
  int G = min(units, num_sms);
  const int need = (units * rpu + cap_rows - 1) / cap_rows;
  if (need > G) G = need;
  *grid = G;
  *max_rows = ((units + G - 1) / G) * rpu;
}

template <int BMAX, int NT, bool NORM, int MODE>
static cudaError_t launch_mma_nt(const GemvParams& p, int grid, int max_rows, cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = mma_layout(p.cols, max_rows).total;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, gemv_mma_kernel<BMAX, NT, NORM, MODE>, p, max_rows);
}

// kGemvQKVCluster: one cluster of kQkvCluster CTAs per head, kClusterRows
// q/k/v rows each (three 8-row n-tiles).
template <int BMAX>
static cudaError_t launch_mma_cluster(const GemvParams& p, cudaStream_t s, bool pdl) {
  if (p.units != p.H * kQkvRowsPerHead || p.pos + 1 > kSelfAttnMaxT || !p.attn_out || p.B > kQkvCluster)
    return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.H * kQkvCluster);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = cluster_ext_offset(mma_layout(p.cols, kClusterRows).total) + kClusterExtra;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kQkvCluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, gemv_mma_kernel<BMAX, 3, true, kGemvQKVCluster>, p, kClusterRows);
}

template <int BMAX, bool NORM, int MODE>
static cudaError_t launch_mma_t(const GemvParams& p, int num_sms, cudaStream_t s, bool pdl) {
  int grid, max_rows;
  mma_plan(p.units, MODE == kGemvGeglu ? 2 : 1, p.cols, num_sms, &grid, &max_rows);
  if (max_rows > kMmaMaxRows || grid <= 0) return cudaErrorInvalidValue;
  switch ((max_rows + 7) / 8) {
    case 1: return launch_mma_nt<BMAX, 1, NORM, MODE>(p, grid, max_rows, s, pdl);
    case 2: return launch_mma_nt<BMAX, 2, NORM, MODE>(p, grid, max_rows, s, pdl);
    case 3: return launch_mma_nt<BMAX, 3, NORM, MODE>(p, grid, max_rows, s, pdl);
    default: return launch_mma_nt<BMAX, 4, NORM, MODE>(p, grid, max_rows, s, pdl);
  }
}

template <int BMAX>
static cudaError_t launch_gemv_mma_b(int mode, bool norm, const GemvParams& p, int num_sms, cudaStream_t s, bool pdl) {
  switch (mode) {
    case kGemvStore:
      return norm ? launch_mma_t<BMAX, true, kGemvStore>(p, num_sms, s, pdl)
                  : launch_mma_t<BMAX, false, kGemvStore>(p, num_sms, s, pdl);
    case kGemvResid:
      return norm ? launch_mma_t<BMAX, true, kGemvResid>(p, num_sms, s, pdl)
                  : launch_mma_t<BMAX, false, kGemvResid>(p, num_sms, s, pdl);
    case kGemvQKV:
      return launch_mma_t<BMAX, true, kGemvQKV>(p, num_sms, s, pdl);
    case kGemvQKVCluster:
      return launch_mma_cluster<BMAX>(p, s, pdl);
    case kGemvGeglu:
      return launch_mma_t<BMAX, true, kGemvGeglu>(p, num_sms, s, pdl);
    case kGemvLogits:
      return launch_mma_t<BMAX, true, kGemvLogits>(p, num_sms, s, pdl);
  }
  return cudaErrorInvalidValue;
}

static cudaError_t launch_gemv_mma(int mode, bool norm, const GemvParams& p, int num_sms, cudaStream_t s, bool pdl) {
  if (p.cols % 16 != 0 || p.cols > 4096 || p.B > kGemvMaxB || p.B <= 0) return cudaErrorInvalidValue;
  if (p.acc && (p.B > 2 || (p.x_stride & 7) != 0)) return cudaErrorInvalidValue;
  if (p.B <= 2) return launch_gemv_mma_b<2>(mode, norm, p, num_sms, s, pdl);
  if (p.B <= 4) return launch_gemv_mma_b<4>(mode, norm, p, num_sms, s, pdl);
  return launch_gemv_mma_b<8>(mode, norm, p, num_sms, s, pdl);
}

template <int BMAX, int NT>
static cudaError_t set_mma_limits_bn() {
  cudaError_t e = cudaSuccess;
  auto set = [&](const void* f) {
    cudaError_t r = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (r != cudaSuccess) e = r;
  };
  set((const void*)gemv_mma_kernel<BMAX, NT, true, kGemvStore>);
  set((const void*)gemv_mma_kernel<BMAX, NT, false, kGemvStore>);
  set((const void*)gemv_mma_kernel<BMAX, NT, true, kGemvResid>);
  set((const void*)gemv_mma_kernel<BMAX, NT, false, kGemvResid>);
  set((const void*)gemv_mma_kernel<BMAX, NT, true, kGemvQKV>);
  if (NT == 3) set((const void*)gemv_mma_kernel<BMAX, 3, true, kGemvQKVCluster>);
  set((const void*)gemv_mma_kernel<BMAX, NT, true, kGemvGeglu>);
  set((const void*)gemv_mma_kernel<BMAX, NT, true, kGemvLogits>);
  return e;
}

template <int BMAX>
static cudaError_t set_mma_limits_b() {
  cudaError_t e = set_mma_limits_bn<BMAX, 1>();
  if (e == cudaSuccess) e = set_mma_limits_bn<BMAX, 2>();
  if (e == cudaSuccess) e = set_mma_limits_bn<BMAX, 3>();
  if (e == cudaSuccess) e = set_mma_limits_bn<BMAX, 4>();
  return e;
}

static cudaError_t set_mma_limits() {
  cudaError_t e = set_mma_limits_b<2>();
  if (e == cudaSuccess) e = set_mma_limits_b<4>();
  if (e == cudaSuccess) e = set_mma_limits_b<8>();
  return e;
}

size_t gemv_smem_bytes(int B, int cols) {
  return (size_t)kGemvStages * kGemvStageBytes + (((size_t)B * cols * 4 + 15) & ~(size_t)15) + kGemvStages * 8;
}

template <typename T, int BMAX, bool NORM, int MODE>
static cudaError_t launch_gemv_t(const GemvParams& p, int grid, cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kGemvThreads);
  cfg.dynamicSmemBytes = gemv_smem_bytes(p.B, p.cols);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, gemv_phase_kernel<T, BMAX, NORM, MODE>, p);
}

template <typename T, int BMAX>
static cudaError_t dispatch_mode(int mode, bool norm, const GemvParams& p, int grid, cudaStream_t s, bool pdl) {
  switch (mode) {
    case kGemvStore:
      return norm ? launch_gemv_t<T, BMAX, true, kGemvStore>(p, grid, s, pdl)
                  : launch_gemv_t<T, BMAX, false, kGemvStore>(p, grid, s, pdl);
    case kGemvResid:
      return norm ? launch_gemv_t<T, BMAX, true, kGemvResid>(p, grid, s, pdl)
                  : launch_gemv_t<T, BMAX, false, kGemvResid>(p, grid, s, pdl);
    case kGemvQKV:
      return launch_gemv_t<T, BMAX, true, kGemvQKV>(p, grid, s, pdl);
    case kGemvGeglu:
      return launch_gemv_t<T, BMAX, true, kGemvGeglu>(p, grid, s, pdl);
    case kGemvLogits:
      return launch_gemv_t<T, BMAX, true, kGemvLogits>(p, grid, s, pdl);
  }
  return cudaErrorInvalidValue;
}

template <typename T>
static cudaError_t dispatch_b(int mode, bool norm, const GemvParams& p, int grid, cudaStream_t s, bool pdl) {
  if (p.B <= 1) return dispatch_mode<T, 1>(mode, norm, p, grid, s, pdl);
  if (p.B <= 2) return dispatch_mode<T, 2>(mode, norm, p, grid, s, pdl);
  if (p.B <= 4) return dispatch_mode<T, 4>(mode, norm, p, grid, s, pdl);
  if (p.B <= 8) return dispatch_mode<T, 8>(mode, norm, p, grid, s, pdl);
  return cudaErrorInvalidValue;
}

cudaError_t launch_gemv(int dtype, int mode, bool norm, const GemvParams& p, int num_sms, cudaStream_t s, bool pdl) {
  if (p.units <= 0) return cudaSuccess;
  if (dtype == 1) return launch_gemv_mma(mode, norm, p, num_sms, s, pdl);
  if (p.acc) return cudaErrorInvalidValue;
  const int rpu = mode == kGemvGeglu ? 2 : 1;
  if (p.cols % 4 != 0 || rpu * p.cols * 4 > kGemvStageBytes) return cudaErrorInvalidValue;
  const int grid = p.units < num_sms ? p.units : num_sms;
  return dispatch_b<float>(mode, norm, p, grid, s, pdl);
}

template <typename T, int BMAX>
static cudaError_t set_limits_b() {
  const int mx = (int)gemv_smem_bytes(BMAX, 4096);
  cudaError_t e = cudaSuccess;
  auto set = [&](const void* f) {
    cudaError_t r = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
    if (r != cudaSuccess) e = r;
  };
  set((const void*)gemv_phase_kernel<T, BMAX, true, kGemvStore>);
  set((const void*)gemv_phase_kernel<T, BMAX, false, kGemvStore>);
  set((const void*)gemv_phase_kernel<T, BMAX, true, kGemvResid>);
  set((const void*)gemv_phase_kernel<T, BMAX, false, kGemvResid>);
  set((const void*)gemv_phase_kernel<T, BMAX, true, kGemvQKV>);
  set((const void*)gemv_phase_kernel<T, BMAX, true, kGemvGeglu>);
  set((const void*)gemv_phase_kernel<T, BMAX, true, kGemvLogits>);
  return e;
}

template <typename T>
static cudaError_t set_limits_t() {
  cudaError_t e;
  if ((e = set_limits_b<T, 1>()) != cudaSuccess) return e;
  if ((e = set_limits_b<T, 2>()) != cudaSuccess) return e;
  if ((e = set_limits_b<T, 4>()) != cudaSuccess) return e;
  return set_limits_b<T, 8>();
}

cudaError_t gemv_set_smem_limits() {
  cudaError_t e = set_mma_limits();
  if (e != cudaSuccess) return e;
  return set_limits_t<float>();
}

// ---------------------------------------------------------------------------
// Self-attention for one new query (decode), one warp per (row, head),
// at most 64 keys (2 chunks of 32). Every load is issued right after the
// dependency wait - q, key row j for lane j, and each lane's two value
// columns of every key - so the kernel pays one L2 round trip; then lane j
// scores key j, a warp softmax, and lane l accumulates output dims 2l, 2l+1.
// Scale 1.0, additive bias (relative-position bias of this query position,
// in the compute dtype's values).
// ---------------------------------------------------------------------------

template <typename T>
__device__ __forceinline__ uint32_t load_pair_bits(const T* p);
template <>
__device__ __forceinline__ uint32_t load_pair_bits<__nv_bfloat16>(const __nv_bfloat16* p) {
  return *reinterpret_cast<const uint32_t*>(p);
}
template <typename T>
__device__ __forceinline__ float2 pair_from_bits(uint32_t v);
template <>
__device__ __forceinline__ float2 pair_from_bits<__nv_bfloat16>(uint32_t v) {
  return make_float2(__uint_as_float(v << 16), __uint_as_float(v & 0xffff0000u));
}

template <typename T>
struct PairReg {  // two consecutive elements kept in registers
  typedef typename std::conditional<sizeof(T) == 2, uint32_t, float2>::type type;
};

template <typename T>
__device__ __forceinline__ typename PairReg<T>::type load_pair(const T* p) {
  if constexpr (sizeof(T) == 2) return load_pair_bits<T>(p);
  else return *reinterpret_cast<const float2*>(p);
}
template <typename T>
__device__ __forceinline__ float2 unpack_pair(typename PairReg<T>::type v) {
  if constexpr (sizeof(T) == 2) return pair_from_bits<T>(v);
  else return v;
}

template <typename T>
__global__ void __launch_bounds__(128) attn_self_kernel(const AttnParams p) {
  pdl_wait();
  __shared__ float qs[4][64];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gw = blockIdx.x * 4 + warp;
  const bool active = gw < p.B * p.H;
  const int b = active ? gw / p.H : 0, h = active ? gw - b * p.H : 0;
  const size_t base = ((size_t)b * p.H + h) * p.cap * 64;
  const T* K = reinterpret_cast<const T*>(p.K) + base;
  const T* V = reinterpret_cast<const T*>(p.V) + base;
  constexpr int EPC = Vec16<T>::N;
  // ---- all loads ----
  const float2 qv = unpack_pair<T>(load_pair<T>(reinterpret_cast<const T*>(p.q) + (size_t)b * p.inner + h * 64 + 2 * lane));
  uint4 kr[2][64 / EPC];
  typename PairReg<T>::type vr[2][32];
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    const int j = c * 32 + lane;
    const bool kv = active && j < p.T;
#pragma unroll
    for (int ch = 0; ch < 64 / EPC; ++ch)
      kr[c][ch] = kv ? reinterpret_cast<const uint4*>(K + (size_t)j * 64)[ch] : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int jj = 0; jj < 32; ++jj) {
      const int jv = c * 32 + jj;
      vr[c][jj] = (active && jv < p.T) ? load_pair<T>(V + (size_t)jv * 64 + 2 * lane) : typename PairReg<T>::type{};
    }
  }
  const float bias0 = (active && p.bias && lane < p.T) ? p.bias[(size_t)h * p.bias_stride + lane] : 0.f;
  const float bias1 = (active && p.bias && 32 + lane < p.T) ? p.bias[(size_t)h * p.bias_stride + 32 + lane] : 0.f;
  pdl_launch_dependents();
  if (!active) return;
  qs[warp][2 * lane] = qv.x;
  qs[warp][2 * lane + 1] = qv.y;
  __syncwarp();
  // ---- scores: lane j <-> key j of each chunk ----
  float sc[2];
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    const int j = c * 32 + lane;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int ch = 0; ch < 64 / EPC; ++ch) {
      float kf[EPC];
      Vec16<T>::unpack(kr[c][ch], kf);
#pragma unroll
      for (int e = 0; e < EPC; ++e) acc[e & 3] = fmaf(qs[warp][ch * EPC + e], kf[e], acc[e & 3]);
    }
    float a = (acc[0] + acc[1]) + (acc[2] + acc[3]);
    if (p.bias) a += (c == 0 ? bias0 : bias1);
    sc[c] = j < p.T ? a : -INFINITY;
  }
  const float m = warp_max(fmaxf(sc[0], sc[1]));
  const float p0 = lane < p.T ? expf(sc[0] - m) : 0.f;
  const float p1 = 32 + lane < p.T ? expf(sc[1] - m) : 0.f;
  const float l = warp_sum(p0 + p1);
  float o0 = 0.f, o1 = 0.f;
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    const float pc = c == 0 ? p0 : p1;
#pragma unroll
    for (int jj = 0; jj < 32; ++jj) {
      const float pw = __shfl_sync(0xffffffffu, pc, jj);
      const float2 v = unpack_pair<T>(vr[c][jj]);
      o0 = fmaf(pw, v.x, o0);
      o1 = fmaf(pw, v.y, o1);
    }
  }
  T* out = reinterpret_cast<T*>(p.out) + (size_t)b * p.inner + h * 64;
  out[2 * lane] = from_f<T>(o0 / l);
  out[2 * lane + 1] = from_f<T>(o1 / l);
}

// ---------------------------------------------------------------------------
// Cross-attention for one new query over the cached encoder K/V: grid
// (B*H, nsplit), 4 warps per CTA, the nsplit CTAs of a (row, head) one
// thread-block cluster. Each CTA reduces its key slice to a partial (max,
// sum, o[64]) and stores it into rank 0's shared memory; rank 0 combines.
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(128) attn_cross_kernel(const AttnParams p) {
  pdl_wait();
  __shared__ float qs[4][64];
  __shared__ float wm[4], wl[4], wo[4][64];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int bh = blockIdx.x, sp = blockIdx.y;
  const int b = bh / p.H, h = bh - b * p.H;
  const size_t base = ((size_t)b * p.H + h) * p.cap * 64;
  const T* K = reinterpret_cast<const T*>(p.K) + base;
  const T* V = reinterpret_cast<const T*>(p.V) + base;
  const int k0 = (int)(((long long)sp * p.T) / p.nsplit), k1 = (int)(((long long)(sp + 1) * p.T) / p.nsplit);
  constexpr int EPC = Vec16<T>::N;
  float m = -INFINITY, l = 0.f, o0 = 0.f, o1 = 0.f;
  bool first = true;
  for (int j0 = k0 + warp * 32; j0 < k1; j0 += 128) {
    // ---- every load of this 32-key chunk (and q), back to back ----
    const int j = j0 + lane;
    const int nj = min(32, k1 - j0);
    uint4 kr[64 / EPC];
#pragma unroll
    for (int ch = 0; ch < 64 / EPC; ++ch)
      kr[ch] = j < k1 ? reinterpret_cast<const uint4*>(K + (size_t)j * 64)[ch] : make_uint4(0, 0, 0, 0);
    typename PairReg<T>::type vr[32];
#pragma unroll
    for (int jj = 0; jj < 32; ++jj)
      vr[jj] = jj < nj ? load_pair<T>(V + (size_t)(j0 + jj) * 64 + 2 * lane) : typename PairReg<T>::type{};
    if (first) {
      const float2 qv =
          unpack_pair<T>(load_pair<T>(reinterpret_cast<const T*>(p.q) + (size_t)b * p.inner + h * 64 + 2 * lane));
      qs[warp][2 * lane] = qv.x;
      qs[warp][2 * lane + 1] = qv.y;
      __syncwarp();
      first = false;
    }
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int ch = 0; ch < 64 / EPC; ++ch) {
      float kf[EPC];
      Vec16<T>::unpack(kr[ch], kf);
#pragma unroll
      for (int e = 0; e < EPC; ++e) acc[e & 3] = fmaf(qs[warp][ch * EPC + e], kf[e], acc[e & 3]);
    }
    const float sc = j < k1 ? (acc[0] + acc[1]) + (acc[2] + acc[3]) : -INFINITY;
    const float cm = warp_max(sc);
    const float nm = fmaxf(m, cm);
    const float scale = (m == -INFINITY) ? 0.f : expf(m - nm);
    const float pj = (j < k1) ? expf(sc - nm) : 0.f;
    l = l * scale + warp_sum(pj);
    o0 *= scale;
    o1 *= scale;
#pragma unroll
    for (int jj = 0; jj < 32; ++jj) {
      const float pw = __shfl_sync(0xffffffffu, pj, jj);
      const float2 v = unpack_pair<T>(vr[jj]);
      o0 = fmaf(pw, v.x, o0);
      o1 = fmaf(pw, v.y, o1);
    }
    m = nm;
  }
  pdl_launch_dependents();
  if (lane == 0) {
    wm[warp] = m;
    wl[warp] = l;
  }
  wo[warp][2 * lane] = o0;
  wo[warp][2 * lane + 1] = o1;
  __syncthreads();
  float part_m = -INFINITY, part_l = 0.f, part_o = 0.f;
  if (threadIdx.x < 64) {
    float M = -INFINITY;
    for (int w = 0; w < 4; ++w) M = fmaxf(M, wm[w]);
    float L = 0.f, O = 0.f;
    for (int w = 0; w < 4; ++w) {
      if (wm[w] == -INFINITY) continue;
      const float f = expf(wm[w] - M);
      L += wl[w] * f;
      O += wo[w][threadIdx.x] * f;
    }
    part_m = M;
    part_l = L;
    part_o = O;
  }
  // The nsplit CTAs of this (row, head) are one thread-block cluster: each
  // pushes its partial (max, sum, o[64]) into slot `sp` of rank 0, which
  // combines the slots in split order after one cluster barrier.
  __shared__ float slots[kCrossSplit][66];
  if (threadIdx.x < 64) {
    st_cluster_f32(&slots[sp][2 + threadIdx.x], 0, part_o);
    if (threadIdx.x == 0) {
      st_cluster_f32(&slots[sp][0], 0, part_m);
      st_cluster_f32(&slots[sp][1], 0, part_l);
    }
  }
  cluster_sync();
  if (cluster_ctarank() != 0 || threadIdx.x >= 64) return;
  float M = -INFINITY;
  for (int s2 = 0; s2 < p.nsplit; ++s2) M = fmaxf(M, slots[s2][0]);
  float L = 0.f, O = 0.f;
  for (int s2 = 0; s2 < p.nsplit; ++s2) {
    const float ms = slots[s2][0];
    if (ms == -INFINITY) continue;
    const float f = expf(ms - M);
    L += slots[s2][1] * f;
    O += slots[s2][2 + threadIdx.x] * f;
  }
  reinterpret_cast<T*>(p.out)[(size_t)b * p.inner + h * 64 + threadIdx.x] = from_f<T>(O / L);
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

cudaError_t launch_attn_self(int dtype, const AttnParams& p, cudaStream_t s, bool pdl) {
  if (p.T > kSelfAttnMaxT) return cudaErrorInvalidValue;
  const dim3 grid((p.B * p.H + 3) / 4);
  return dtype == 1 ? launch_k(attn_self_kernel<__nv_bfloat16>, grid, dim3(128), 0, s, pdl, p)
                    : launch_k(attn_self_kernel<float>, grid, dim3(128), 0, s, pdl, p);
}

cudaError_t launch_attn_cross(int dtype, const AttnParams& p, cudaStream_t s, bool pdl) {
  if (p.nsplit != 1 && p.nsplit != 2 && p.nsplit != 4 && p.nsplit != kCrossSplit) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.B * p.H, p.nsplit);
  cfg.blockDim = dim3(128);
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = p.nsplit;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  return dtype == 1 ? cudaLaunchKernelEx(&cfg, attn_cross_kernel<__nv_bfloat16>, p)
                    : cudaLaunchKernelEx(&cfg, attn_cross_kernel<float>, p);
}

// ---------------------------------------------------------------------------
// Sampler: one CTA of 256 threads per sequence.
//   guided = CFG mix of the sequence's two rows (fp32), restricted to the
//   candidate range [lo, hi) (the level's vocab mask); temperature 0 ->
//   argmax (first index on ties); else scaled = guided / T, threshold = the
//   top_k-th largest scaled value (exact radix select over order-preserving
//   keys, 8 bits per pass, warp-aggregated shared histogram; ties at the
//   threshold survive), token = argmax(scaled + Gumbel(u)) over the
//   survivors. Then the embedding of the token becomes the next depth input
//   of every row of the sequence and is added into the frame sum; on the
//   last level the next temporal input R(sum / depth) is written.
// ---------------------------------------------------------------------------
constexpr int kSampleThreads = 256;

__device__ __forceinline__ void argmax_combine(float& v, int& i, float v2, int i2) {
  if (v2 > v || (v2 == v && i2 < i)) {
    v = v2;
    i = i2;
  }
}

template <typename T>
__global__ void __launch_bounds__(kSampleThreads) sample_kernel(const SampleParams p) {
  pdl_wait();
  pdl_launch_dependents();
  extern __shared__ __align__(16) float vals[];
  __shared__ unsigned hist[256];
  __shared__ unsigned sel_prefix, sel_k;
  __shared__ float rv[kSampleThreads / 32];
  __shared__ int ri[kSampleThreads / 32];
  __shared__ int tok_s;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int seq = blockIdx.x;
  const int n = p.hi - p.lo;
  const int r0 = seq * p.rows_per_seq;

  // The frame's running embedding sum does not depend on the token: its
  // loads go out first, next to the logits loads (one round trip for both).
  constexpr int EPC = Vec16<T>::N;
  const int nchunk = p.d / EPC;
  constexpr int kFsumRegs = 2;  // chunks per thread held in registers (d <= 2 x 256 x EPC)
  uint4 fs_pre[2][kFsumRegs];
  const bool fs_in_regs = !p.is_first && p.rows_per_seq <= 2 && nchunk <= kFsumRegs * kSampleThreads;
  if (fs_in_regs) {
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
      for (int q = 0; q < kFsumRegs; ++q) {
        const int ch = tid + q * kSampleThreads;
        fs_pre[r][q] = (r < p.rows_per_seq && ch < nchunk)
                           ? reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.fsum) +
                                                            (size_t)(r0 + r) * p.d)[ch]
                           : make_uint4(0, 0, 0, 0);
      }
  }

  int token;
  if (p.forced) {
    token = p.forced[seq];
  } else {
    const float* l0 = p.logits + (size_t)r0 * p.logits_stride + (p.lo - p.col_offset);
    const float* l1 = l0 + p.logits_stride;
    // four strides of candidates per pass: all eight loads in flight at once
    constexpr int U = 4;
    for (int i0 = 0; i0 < n; i0 += U * kSampleThreads) {
      float a[U], b[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = i0 + u * kSampleThreads + tid;
        a[u] = i < n ? l0[i] : 0.f;
        b[u] = (i < n && p.rows_per_seq == 2) ? l1[i] : 0.f;
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = i0 + u * kSampleThreads + tid;
        if (i < n) {
          float g = (p.rows_per_seq == 2) ? cfg_mix(a[u], b[u], p.w) : a[u];
          if (p.temperature != 0.0f) g = __fdiv_rn(g, p.temperature);
          vals[i] = g;
        }
      }
    }
    if (tid == 0) {
      sel_prefix = 0u;
      sel_k = (unsigned)p.top_k;
    }
    __syncthreads();
    float thr = -INFINITY;
    if (p.temperature != 0.0f && p.top_k > 0 && p.top_k < n) {
      unsigned mask = 0u;
      for (int pass = 0; pass < 4; ++pass) {
        const int shift = 24 - 8 * pass;
        hist[tid] = 0u;
        __syncthreads();
        const unsigned prefix = sel_prefix;
        for (int i0 = 0; i0 < n; i0 += kSampleThreads) {
          const int i = i0 + tid;
          const unsigned key = i < n ? float_order_key(vals[i]) : 0u;
          const bool in = i < n && (key & mask) == prefix;
          const unsigned dg = in ? ((key >> shift) & 255u) : 256u + (unsigned)lane;  // unique no-op digit
          // lanes holding the same digit add once, through their leader
          const unsigned peers = __match_any_sync(0xffffffffu, dg);
          if (in && lane == (__ffs(peers) - 1)) atomicAdd(&hist[dg], (unsigned)__popc(peers));
        }
        __syncthreads();
        if (warp == 0) {
          // lane L owns digits 255-8L ... 248-8L (descending)
          unsigned cnt[8], tot = 0;
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            cnt[q] = hist[255 - 8 * lane - q];
            tot += cnt[q];
          }
          unsigned incl = tot;
#pragma unroll
          for (int o = 1; o < 32; o <<= 1) {
            const unsigned t2 = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += t2;
          }
          const unsigned excl = incl - tot;
          const unsigned kk = sel_k;
          if (excl < kk && incl >= kk) {
            unsigned cum = excl;
            int dg = 255 - 8 * lane;
            for (int q = 0; q < 8; ++q) {
              if (cum + cnt[q] >= kk) {
                dg = 255 - 8 * lane - q;
                break;
              }
              cum += cnt[q];
            }
            sel_prefix = prefix | ((unsigned)dg << shift);
            sel_k = kk - cum;
          }
        }
        mask |= 255u << shift;
        __syncthreads();
      }
      thr = float_from_order_key(sel_prefix);
    }
    float best = -INFINITY;
    int bi = 0x7fffffff;
    const float* uni = p.uniforms ? p.uniforms + (size_t)seq * p.uni_seq_stride : nullptr;
    const uint64_t seed = p.seeds ? p.seeds[seq] : p.seed_value;
    for (int i = tid; i < n; i += kSampleThreads) {
      float v = vals[i];
      if (p.temperature != 0.0f) {
        if (v < thr || v == -INFINITY) {
          v = -INFINITY;
        } else {
          const int vid = p.lo + i;
          const float u = uni ? uni[vid] : philox_uniform(seed, p.step, (uint32_t)vid);
          v = __fadd_rn(v, gumbel_from_uniform(u));
        }
      }
      argmax_combine(best, bi, v, i);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float v2 = __shfl_xor_sync(0xffffffffu, best, o);
      const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
      argmax_combine(best, bi, v2, i2);
    }
    if (lane == 0) {
      rv[warp] = best;
      ri[warp] = bi;
    }
    __syncthreads();
    if (tid == 0) {
      best = rv[0];
      bi = ri[0];
      for (int w = 1; w < kSampleThreads / 32; ++w) argmax_combine(best, bi, rv[w], ri[w]);
      tok_s = bi == 0x7fffffff ? -1 : p.lo + bi;  // -1: no candidate survived (NaN logits, empty range)
    }
    __syncthreads();
    token = tok_s;
  }
  int out_token = token;
  if (token < 0 || token >= p.V) {
    if (tid == 0 && p.err) atomicOr(p.err, kErrBadToken);
    out_token = p.bad_token;
    token = 0;  // the embedding rows stay defined
  }
  if (tid == 0 && p.tokens) p.tokens[(size_t)seq * p.tok_stride + p.tok_index] = out_token;

  // embedding feedback, 16 bytes per thread per row
  const uint4* e = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.emb) + (size_t)token * p.d);
  for (int ch = tid, q_reg = 0; ch < nchunk; ch += kSampleThreads, ++q_reg) {
    const uint4 ev = e[ch];
    float ef[EPC];
    Vec16<T>::unpack(ev, ef);
    for (int r = 0; r < p.rows_per_seq; ++r) {
      const size_t off = (size_t)(r0 + r) * p.d + (size_t)ch * EPC;
      *reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.din) + off) = ev;
      T* fs = reinterpret_cast<T*>(p.fsum) + off;
      T* tin = reinterpret_cast<T*>(p.tin) + off;
      float prev[EPC];
      if (!p.is_first) {
        if (fs_in_regs) {
          uint4 pv = make_uint4(0, 0, 0, 0);
#pragma unroll
          for (int qq = 0; qq < kFsumRegs; ++qq)
#pragma unroll
            for (int rr = 0; rr < 2; ++rr)
              if (qq == q_reg && rr == r) pv = fs_pre[rr][qq];
          Vec16<T>::unpack(pv, prev);
        } else {
#pragma unroll
          for (int q = 0; q < EPC; ++q) prev[q] = to_f(fs[q]);
        }
      }
      T outv[EPC];
#pragma unroll
      for (int q = 0; q < EPC; ++q) {
        const float sum = p.is_first ? ef[q] : rnd<T>(__fadd_rn(prev[q], ef[q]));
        outv[q] = from_f<T>(sum);
        if (p.is_last) tin[q] = from_f<T>(__fdiv_rn(sum, (float)p.depth));
      }
#pragma unroll
      for (int q = 0; q < EPC; ++q) fs[q] = outv[q];
    }
  }
}

// ---------------------------------------------------------------------------
// Sampler for at most 1024 candidates (a level's vocab mask holds one
// codebook): one CTA of 1024 threads per sequence, thread i owns candidate
// lo + i. Same arithmetic and result as sample_kernel, organised for short
// dependency chains:
//   * the Gumbel noise of every candidate (Philox draw + two logs) does not
//     depend on the logits, so it is computed while their loads are in flight;
//   * the top-k threshold (the k-th largest order key, ties counted with
//     their multiplicity as the radix select counts them) comes from two
//     1024-bin histogram levels (key bits 31..22, then 21..12 inside the
//     boundary bin; shared-memory atomics and block scans) and an exact
//     rank count among the candidates left in the final bin.
// ---------------------------------------------------------------------------
constexpr int kSampleSmallThreads = 1024;

// Inclusive prefix sum of v over the 1024 threads (thread order); wsum is
// 32 words of shared scratch. Two barriers.
__device__ __forceinline__ unsigned block_scan_1024(unsigned v, unsigned* wsum) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) wsum[warp] = x;
  __syncthreads();
  if (warp == 0) {
    unsigned w = wsum[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    wsum[lane] = w;
  }
  __syncthreads();
  return x + (warp > 0 ? wsum[warp - 1] : 0u);
}

template <typename T>
__global__ void __launch_bounds__(kSampleSmallThreads) sample_small_kernel(const SampleParams p) {
  __shared__ unsigned hist[1024];
  __shared__ unsigned wsum[32];
  __shared__ uint32_t cand[1024];
  __shared__ unsigned sel_bin, sel_above, ncand;
  __shared__ uint32_t kth;
  __shared__ float rv[32];
  __shared__ int ri[32];
  __shared__ int tok_s;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int seq = blockIdx.x;
  const int n = p.hi - p.lo;
  const int r0 = seq * p.rows_per_seq;
  constexpr int EPC = Vec16<T>::N;
  const int nchunk = p.d / EPC;

  // Before the dependency wait (none of it is written by the kernel ahead,
  // the lm_head launch): the Gumbel noise of every candidate (seeds and
  // injected draws are inputs of the chunk) and the frame's running
  // embedding sum (written by the previous level's sampler, which completed
  // before the kernel ahead passed its own wait).
  const bool fs_pre_ok = !p.is_first && tid < p.rows_per_seq * nchunk;
  uint4 fs_pre = make_uint4(0, 0, 0, 0);
  if (fs_pre_ok) {
    const int r = tid / nchunk, ch = tid - r * nchunk;
    fs_pre = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.fsum) + (size_t)(r0 + r) * p.d)[ch];
  }
  const bool has = tid < n;
  const bool sampled = p.temperature != 0.0f;
  float gum = 0.f;
  if (!p.forced && has && sampled) {
    const float u = p.uniforms ? p.uniforms[(size_t)seq * p.uni_seq_stride + p.lo + tid]
                               : philox_uniform(p.seeds ? p.seeds[seq] : p.seed_value, p.step, (uint32_t)(p.lo + tid));
    gum = gumbel_from_uniform(u);
  }
  pdl_wait();
  pdl_launch_dependents();

  int token;
  if (p.forced) {
    token = p.forced[seq];
  } else {
    float a = 0.f, b = 0.f;
    if (has) {
      const float* l0 = p.logits + (size_t)r0 * p.logits_stride + (p.lo - p.col_offset);
      a = l0[tid];
      if (p.rows_per_seq == 2) b = l0[p.logits_stride + tid];
    }
    float v = -INFINITY;
    if (has) {
      float g = p.rows_per_seq == 2 ? cfg_mix(a, b, p.w) : a;
      if (sampled) g = __fdiv_rn(g, p.temperature);
      v = g;
    }
    float thr = -INFINITY;
    if (sampled && p.top_k > 0 && p.top_k < n) {
      const uint32_t key = float_order_key(v);
      // level 1: bins of key bits 31..22
      hist[tid] = 0u;
      if (tid == 0) ncand = 0u;
      __syncthreads();
      if (has) atomicAdd(&hist[key >> 22], 1u);
      __syncthreads();
      unsigned c = hist[1023 - tid];  // thread t <-> bin 1023 - t: descending keys
      unsigned incl = block_scan_1024(c, wsum);
      if (incl - c < (unsigned)p.top_k && incl >= (unsigned)p.top_k) {
        sel_bin = 1023u - (unsigned)tid;
        sel_above = incl - c;
      }
      __syncthreads();
      const unsigned bin1 = sel_bin, above1 = sel_above;
      // level 2: bins of key bits 21..12 inside bin1
      hist[tid] = 0u;
      __syncthreads();
      const bool in1 = has && (key >> 22) == bin1;
      if (in1) atomicAdd(&hist[(key >> 12) & 1023u], 1u);
      __syncthreads();
      c = hist[1023 - tid];
      incl = block_scan_1024(c, wsum);
      const unsigned k2 = (unsigned)p.top_k - above1;
      if (incl - c < k2 && incl >= k2) {
        sel_bin = 1023u - (unsigned)tid;
        sel_above = above1 + incl - c;
      }
      __syncthreads();
      const unsigned bin2 = sel_bin, above2 = sel_above;
      // the final bin: exact ranks among its members
      const bool in2 = in1 && ((key >> 12) & 1023u) == bin2;
      if (in2) cand[atomicAdd(&ncand, 1u)] = key;
      __syncthreads();
      if (in2) {
        const unsigned k3 = (unsigned)p.top_k - above2, m = ncand;
        unsigned gt = 0, ge = 0;
        for (unsigned j = 0; j < m; ++j) {
          const uint32_t kj = cand[j];
          gt += kj > key;
          ge += kj >= key;
        }
        if (gt < k3 && k3 <= ge) kth = key;  // every writer holds the same key
      }
      __syncthreads();
      thr = float_from_order_key(kth);
    }
    float best = -INFINITY;
    int bi = 0x7fffffff;
    if (has) {
      float val = v;
      if (sampled) val = (val < thr || val == -INFINITY) ? -INFINITY : __fadd_rn(val, gum);
      argmax_combine(best, bi, val, tid);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float v2 = __shfl_xor_sync(0xffffffffu, best, o);
      const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
      argmax_combine(best, bi, v2, i2);
    }
    if (lane == 0) {
      rv[warp] = best;
      ri[warp] = bi;
    }
    __syncthreads();
    if (warp == 0) {
      best = rv[lane];
      bi = ri[lane];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float v2 = __shfl_xor_sync(0xffffffffu, best, o);
        const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
        argmax_combine(best, bi, v2, i2);
      }
      if (lane == 0) tok_s = bi == 0x7fffffff ? -1 : p.lo + bi;  // -1: no candidate survived
    }
    __syncthreads();
    token = tok_s;
  }
  int out_token = token;
  if (token < 0 || token >= p.V) {
    if (tid == 0 && p.err) atomicOr(p.err, kErrBadToken);
    out_token = p.bad_token;
    token = 0;  // the embedding rows stay defined
  }
  if (tid == 0 && p.tokens) p.tokens[(size_t)seq * p.tok_stride + p.tok_index] = out_token;

  // embedding feedback: work item (row r, 16-byte chunk ch)
  const uint4* e = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.emb) + (size_t)token * p.d);
  for (int w = tid; w < p.rows_per_seq * nchunk; w += kSampleSmallThreads) {
    const int r = w / nchunk, ch = w - r * nchunk;
    const uint4 ev = e[ch];
    float ef[EPC];
    Vec16<T>::unpack(ev, ef);
    const size_t off = (size_t)(r0 + r) * p.d + (size_t)ch * EPC;
    *reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.din) + off) = ev;
    T* fs = reinterpret_cast<T*>(p.fsum) + off;
    T* tin = reinterpret_cast<T*>(p.tin) + off;
    float prev[EPC];
    if (!p.is_first) {
      if (w == tid && fs_pre_ok) {
        Vec16<T>::unpack(fs_pre, prev);
      } else {
#pragma unroll
        for (int q = 0; q < EPC; ++q) prev[q] = to_f(fs[q]);
      }
    }
    T outv[EPC];
#pragma unroll
    for (int q = 0; q < EPC; ++q) {
      const float sum = p.is_first ? ef[q] : rnd<T>(__fadd_rn(prev[q], ef[q]));
      outv[q] = from_f<T>(sum);
      if (p.is_last) tin[q] = from_f<T>(__fdiv_rn(sum, (float)p.depth));
    }
#pragma unroll
    for (int q = 0; q < EPC; ++q) fs[q] = outv[q];
  }
}

size_t sample_smem_bytes(int n_candidates) { return (size_t)n_candidates * 4; }

cudaError_t sample_set_smem_limits() {
  cudaError_t e = cudaFuncSetAttribute(sample_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       kSampleMaxSmem);
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(sample_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSampleMaxSmem);
}

cudaError_t launch_sample(int dtype, const SampleParams& p, int num_seq, cudaStream_t s, bool pdl) {
  const int n = p.hi - p.lo;
  if (n >= 1 && n <= kSampleSmallThreads)
    return dtype == 1 ? launch_k(sample_small_kernel<__nv_bfloat16>, dim3(num_seq), dim3(kSampleSmallThreads), 0, s,
                                 pdl, p)
                      : launch_k(sample_small_kernel<float>, dim3(num_seq), dim3(kSampleSmallThreads), 0, s, pdl, p);
  const size_t smem = sample_smem_bytes(n);
  if (smem > (size_t)kSampleMaxSmem) return cudaErrorInvalidValue;
  return dtype == 1 ? launch_k(sample_kernel<__nv_bfloat16>, dim3(num_seq), dim3(kSampleThreads), smem, s, pdl, p)
                    : launch_k(sample_kernel<float>, dim3(num_seq), dim3(kSampleThreads), smem, s, pdl, p);
}

// ---------------------------------------------------------------------------
// Allocation-free sampling (mrtdf_sample_noalloc): the three
// embedding-feedback rows the sampler writes live in this fixed device array
// instead of cudaMalloc'd buffers. Every GPU that loads the library holds
// these 64 KiB until process exit; all calls on a device share them, so
// calls that overlap on the GPU race. Nothing in it has to start at zero:
// the kernel writes the feedback rows without reading them (first level, not
// last). The seed travels by value in the launch parameters and a failed
// draw is reported through the token itself (-1), so no word here is read.
// ---------------------------------------------------------------------------
static __device__ __align__(256) unsigned char g_sample_scratch[kSampleScratchBytes];

cudaError_t sample_scratch_address(int device, void** out) {
  // One lookup per device, made with that device current: in host code the
  // array's name is only a stand-in, its device address comes from the runtime.
  static std::mutex mu;
  static void* addr[128] = {};
  if (device < 0 || device >= 128) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[device]) {
    int prev = 0;
    cudaError_t e = cudaGetDevice(&prev);
    if (e != cudaSuccess) return e;
    if (prev != device && (e = cudaSetDevice(device)) != cudaSuccess) return e;
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_sample_scratch);
    if (prev != device) cudaSetDevice(prev);
    if (e != cudaSuccess) return e;
    addr[device] = p;
  }
  *out = addr[device];
  return cudaSuccess;
}

// ---------------------------------------------------------------------------
// Read bandwidth probe: every thread streams 16-byte loads (L1 bypassed) over
// a grid-strided range and folds them into one word per CTA, so the loads
// cannot be elided.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) l2_read_kernel(const uint4* buf, size_t n16, unsigned* sink) {
  unsigned acc = 0;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (; i + 3 * stride < n16; i += 4 * stride) {
    const uint4 a = __ldcg(buf + i), b = __ldcg(buf + i + stride), c = __ldcg(buf + i + 2 * stride),
                d = __ldcg(buf + i + 3 * stride);
    acc ^= a.x ^ a.y ^ a.z ^ a.w ^ b.x ^ b.y ^ b.z ^ b.w ^ c.x ^ c.y ^ c.z ^ c.w ^ d.x ^ d.y ^ d.z ^ d.w;
  }
  for (; i < n16; i += stride) {
    const uint4 a = __ldcg(buf + i);
    acc ^= a.x ^ a.y ^ a.z ^ a.w;
  }
  acc = __reduce_xor_sync(0xffffffffu, acc);
  if ((threadIdx.x & 31) == 0) atomicXor(sink + (blockIdx.x & 4095), acc);
}

cudaError_t launch_l2_read(const void* buf, size_t bytes, unsigned* sink, int num_sms, cudaStream_t s) {
  l2_read_kernel<<<num_sms * 4, 256, 0, s>>>(reinterpret_cast<const uint4*>(buf), bytes / 16, sink);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Failure-detection check: the production bounded wait on an mbarrier whose
// phase never completes (count 1, no arrival, no copy in flight), with a
// caller-chosen bound. The CTA gives up, reports kErrMbarTimeout and exits.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(32) wait_timeout_probe_kernel(int* err, unsigned long long timeout_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait_bounded(&bar, 0, err, timeout_ns);
}

cudaError_t launch_wait_timeout_probe(int* err, unsigned long long timeout_ns, cudaStream_t s) {
  wait_timeout_probe_kernel<<<1, 32, 0, s>>>(err, timeout_ns);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Small helpers
// ---------------------------------------------------------------------------
struct EmbedParams {
  const void* emb;
  const int32_t* ids;
  int rows, d;
  void* out;
};

template <typename T>
__global__ void embed_rows_kernel(const EmbedParams p) {
  pdl_launch_dependents();
  pdl_wait();
  const int r = blockIdx.x;
  const int id = p.ids ? p.ids[r] : 0;
  const T* e = reinterpret_cast<const T*>(p.emb) + (size_t)id * p.d;
  T* o = reinterpret_cast<T*>(p.out) + (size_t)r * p.d;
  for (int i = threadIdx.x; i < p.d; i += blockDim.x) o[i] = e[i];
}

cudaError_t launch_embed_rows(int dtype, const void* emb, const int32_t* ids, int rows, int d, void* out,
                              cudaStream_t s, bool pdl) {
  EmbedParams p{emb, ids, rows, d, out};
  return dtype == 1 ? launch_k(embed_rows_kernel<__nv_bfloat16>, dim3(rows), dim3(256), 0, s, pdl, p)
                    : launch_k(embed_rows_kernel<float>, dim3(rows), dim3(256), 0, s, pdl, p);
}

struct ConvParams {
  const void* src;
  size_t n;
  void* dst;
};

template <typename T>
__global__ void f32_to_act_kernel(const ConvParams p) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < p.n; i += (size_t)gridDim.x * blockDim.x)
    reinterpret_cast<T*>(p.dst)[i] = from_f<T>(reinterpret_cast<const float*>(p.src)[i]);
}
template <typename T>
__global__ void act_to_f32_kernel(const ConvParams p) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < p.n; i += (size_t)gridDim.x * blockDim.x)
    reinterpret_cast<float*>(p.dst)[i] = to_f(reinterpret_cast<const T*>(p.src)[i]);
}

cudaError_t launch_f32_to_act(int dtype, const float* src, size_t n, void* out, cudaStream_t s) {
  ConvParams p{src, n, out};
  const int grid = (int)std::min<size_t>((n + 255) / 256, 4096);
  if (grid == 0) return cudaSuccess;
  if (dtype == 1) f32_to_act_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(p);
  else f32_to_act_kernel<float><<<grid, 256, 0, s>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_act_to_f32(int dtype, const void* src, size_t n, float* out, cudaStream_t s) {
  ConvParams p{src, n, out};
  const int grid = (int)std::min<size_t>((n + 255) / 256, 4096);
  if (grid == 0) return cudaSuccess;
  if (dtype == 1) act_to_f32_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(p);
  else act_to_f32_kernel<float><<<grid, 256, 0, s>>>(p);
  return cudaGetLastError();
}

}  // namespace mrtdf
