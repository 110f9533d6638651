// Fused decode phases for one CFG pair in bf16 (fused_decode.cuh): a decoder
// layer as three launches (temporal stack) or two (depth stack), each ending
// in a split-K projection summed in an int64 fixed-point accumulator.
//
// Reference semantics (rhymeswithlion/magenta-realtime-mlx-cpp):
//   DecoderLayer::forward  depthformer/modules.cpp:384-446 (pre-norm
//                          sub-blocks, residual adds rounded to bf16)
//   RMSNorm                modules.cpp:72-84 (eps 1e-6)
//   MHA, scale 1.0         modules.cpp:243-321 (SDPA with additive bias;
//                          cross attention without bias over the cached
//                          encoder K/V, modules.cpp:258-261)
//   Gated FFN              modules.cpp:222-226 + gelu_approx nn_ops.h:66-84
// Rounding points as MLX in bf16: every projection output, the attention
// output and each residual sum rounded to bf16; reductions in fp32. The
// split-K sums of o_proj / wo are exact integer sums of the fp32 partials
// scaled by 2^32, rounded to fp32 and then to bf16 by the consumer.
#include <cuda_bf16.h>

#include <algorithm>

#include "common.cuh"
#include "decode_device.cuh"
#include "decode_kernels.cuh"
#include "device_errors.h"
#include "fused_decode.cuh"

namespace mrtdf {

namespace {

typedef __nv_bfloat16 bf16;
constexpr int kThreads = 256;
constexpr int kSelfMaxKeys = 64;                     // keys of a decode self-attention
constexpr int kCrossMaxKeysPerCta = 128;             // 4 warps x 32 keys
constexpr int kBlkRow = 64 * 2 + 16;                 // padded row of an o_proj block (64 bf16 + 8 zero)

__host__ __device__ inline int align128(int v) { return (v + 127) & ~127; }

// acc += round(v * 2^32) with a relaxed 64-bit atomic add (no return value).
// NaN or |v| >= 2^30 cannot be represented: the error word gets
// kErrFixedRange and 0 is added instead.
__device__ __forceinline__ void red_add_fixed(long long* addr, float v, int* err) {
  if (!(fabsf(v) < 1073741824.0f)) {
    if (err) atomicOr(err, kErrFixedRange);
    v = 0.f;
  }
  const long long q = __double2ll_rn((double)v * 4294967296.0);
  asm volatile("red.relaxed.gpu.global.add.u64 [%0], %1;" ::"l"(addr), "l"(q) : "memory");
}

__device__ __forceinline__ void st_cluster_u16(void* local, uint32_t rank, uint16_t v) {
  uint32_t ra;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(smem_u32(local)), "r"(rank));
  asm volatile("st.shared::cluster.u16 [%0], %1;" ::"r"(ra), "h"(v) : "memory");
}

// This thread's norm-weight chunks for its input-stage work items
// w = tid + 256 i (chunk w % nch); loaded before the dependency wait.
__device__ __forceinline__ void load_norm_chunks(const void* norm_w, int nch, int nrows, uint4 (&nw)[2]) {
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int w = threadIdx.x + kThreads * i;
    nw[i] = w < nrows * nch ? reinterpret_cast<const uint4*>(norm_w)[w % nch] : make_uint4(0, 0, 0, 0);
  }
}

// The phase input for rows r0 .. r0 + nrows - 1 (nrows <= 2): x (the plain
// input, or R(residual + R(acc / 2^32))), stored as bf16 to in.x_out when
// `write_x` (accumulator input only), and R(w * R(x * rstd)) staged as bf16
// rows `rs` bytes apart in xs. Ends with a CTA barrier.
__device__ __forceinline__ void stage_input(const FusedIn& in, int r0, int nrows, const uint4 (&nw)[2], uint8_t* xs,
                                            int rs, bool write_x, float* red16) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nch = in.d >> 3;
  float f[2][8];
  int rowi[2] = {0, 0}, chi[2] = {0, 0};
  bool act[2];
  float ss0 = 0.f, ss1 = 0.f;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int w = tid + kThreads * i;
    act[i] = w < nrows * nch;
    if (!act[i]) continue;
    const int rb = w / nch, ch = w - rb * nch;
    rowi[i] = rb;
    chi[i] = ch;
    const size_t off = (size_t)(r0 + rb) * in.d + (size_t)ch * 8;
    Vec16<bf16>::unpack(*reinterpret_cast<const uint4*>(reinterpret_cast<const bf16*>(in.x) + off), f[i]);
    if (in.acc) {
      const longlong2* ap = reinterpret_cast<const longlong2*>(in.acc + off);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const longlong2 a = ap[q];
        f[i][2 * q] = rnd<bf16>(__fadd_rn(f[i][2 * q], rnd<bf16>(fixed_to_float(a.x))));
        f[i][2 * q + 1] = rnd<bf16>(__fadd_rn(f[i][2 * q + 1], rnd<bf16>(fixed_to_float(a.y))));
      }
      if (write_x && in.x_out) {
        uint32_t o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const __nv_bfloat162 pr = __floats2bfloat162_rn(f[i][2 * e], f[i][2 * e + 1]);
          o[e] = *reinterpret_cast<const uint32_t*>(&pr);
        }
        *reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(in.x_out) + off) = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
    float s = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) s = fmaf(f[i][e], f[i][e], s);
    if (rb == 0) ss0 += s;
    else ss1 += s;
  }
  ss0 = warp_sum(ss0);
  ss1 = warp_sum(ss1);
  if (lane == 0) {
    red16[warp * 2] = ss0;
    red16[warp * 2 + 1] = ss1;
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    if (!act[i]) continue;
    const int rb = rowi[i];
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) t += red16[w * 2 + rb];
    const float r = __frcp_rn(__fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)in.d), 1e-6f)));
    float wv[8];
    Vec16<bf16>::unpack(nw[i], wv);
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float a0 = rnd<bf16>(__fmul_rn(wv[2 * e], rnd<bf16>(__fmul_rn(f[i][2 * e], r))));
      const float a1 = rnd<bf16>(__fmul_rn(wv[2 * e + 1], rnd<bf16>(__fmul_rn(f[i][2 * e + 1], r))));
      const __nv_bfloat162 pr = __floats2bfloat162_rn(a0, a1);
      o[e] = *reinterpret_cast<const uint32_t*>(&pr);
    }
    *reinterpret_cast<uint4*>(xs + (size_t)rb * rs + chi[i] * 16) = make_uint4(o[0], o[1], o[2], o[3]);
  }
  __syncthreads();
}

// CTA `cta` of `ncta` zeroes its share of the n accumulator words.
__device__ __forceinline__ void zero_share(long long* p, int n, int cta, int ncta) {
  if (!p) return;
  const int a = (int)(((long long)cta * n) / ncta), b = (int)(((long long)(cta + 1) * n) / ncta);
  for (int i = a + (int)threadIdx.x; i < b; i += kThreads) p[i] = 0;
}

// Y[rr][b] = sum_k W[rr][k] * X[b][k] for the R weight rows in shared memory
// (padded rows rs bytes apart, 8 * NT rows at most) and nrows input rows:
// mma.sync m16n8k16 with the input rows as M and eight weight rows per
// n-tile, k split over the 8 warps; every warp's partial lands in `red`
// (sum it over warps with mma_rows_result after a CTA barrier).
template <int NT>
__device__ __forceinline__ void mma_rows(uint32_t wbase, int R, uint32_t xbase, int rs, int nrows, int cols,
                                         float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int KS = cols >> 4;
  const int k0 = (warp * KS) >> 3, k1 = ((warp + 1) * KS) >> 3;
  const int g = lane >> 2, t = lane & 3;
  const uint32_t xrow = xbase + (uint32_t)(min(g, nrows - 1) * rs) + (uint32_t)(4 * t);
  float acc[NT][4];
#pragma unroll
  for (int i = 0; i < NT; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  uint32_t rowaddr[NT];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
    rowaddr[nt] = wbase + (uint32_t)(min(nt * 8 + (lane & 7), R - 1) * rs + (lane >> 3) * 16);
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
      ldsm_x4_g(bw, rowaddr[nt] + (uint32_t)(ks * 32));
      mma_m16n8k16(acc[nt], a, bw[0], bw[1]);
    }
  }
  if (g < nrows) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      float* rp = red + ((size_t)(warp * NT + nt) * 8) * 2;
      rp[(2 * t) * 2 + g] = acc[nt][0];
      rp[(2 * t + 1) * 2 + g] = acc[nt][1];
    }
  }
}

template <int NT>
__device__ __forceinline__ float mma_rows_result(const float* red, int rr, int b) {
  float s = 0.f;
#pragma unroll
  for (int w = 0; w < 8; ++w) s += red[((w * NT + (rr >> 3)) * 8 + (rr & 7)) * 2 + b];
  return s;
}

// out[b * out_stride + n0 + n] += sum_k A[b][k] * Wt[n][k] (n < 8 * ntiles,
// b < nrows) into the fixed-point accumulator: Wt rows in shared memory
// (rs_w bytes apart), A rows bf16 in shared memory (rs_a bytes apart),
// K a multiple of 32. Warp w takes n-tiles w, w + 8, ...
__device__ __forceinline__ void proj_red(uint32_t wt, int rs_w, int ntiles, uint32_t a, int rs_a, int nrows, int K,
                                         long long* out, int out_stride, int n0, int* err) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const uint32_t xrow = a + (uint32_t)(min(g, nrows - 1) * rs_a) + (uint32_t)(4 * t);
  for (int nt = warp; nt < ntiles; nt += 8) {
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    const uint32_t ra = wt + (uint32_t)((nt * 8 + (lane & 7)) * rs_w + (lane >> 3) * 16);
    for (int kk = 0; kk < (K >> 4); kk += 2) {
      uint32_t b[4], x[4];
      ldsm_x4_g(b, ra + (uint32_t)(kk * 32));
      const uint32_t xo = xrow + (uint32_t)(kk * 32);
      asm volatile("ld.shared.b32 %0, [%1];" : "=r"(x[0]) : "r"(xo));
      asm volatile("ld.shared.b32 %0, [%1];" : "=r"(x[1]) : "r"(xo + 16));
      asm volatile("ld.shared.b32 %0, [%1];" : "=r"(x[2]) : "r"(xo + 32));
      asm volatile("ld.shared.b32 %0, [%1];" : "=r"(x[3]) : "r"(xo + 48));
      const uint32_t a0[4] = {x[0], 0u, x[1], 0u};
      const uint32_t a1[4] = {x[2], 0u, x[3], 0u};
      mma_m16n8k16(acc, a0, b[0], b[1]);
      mma_m16n8k16(acc, a1, b[2], b[3]);
    }
    if (g < nrows) {
      long long* o = out + (size_t)g * out_stride + n0 + nt * 8 + 2 * t;
      red_add_fixed(o, acc[0], err);
      red_add_fixed(o + 1, acc[1], err);
    }
  }
}

__device__ __forceinline__ uint16_t bf16_bits_dev(float v) {
  const bf16 h = __float2bfloat16_rn(v);
  return *reinterpret_cast<const uint16_t*>(&h);
}

// ---------------------------------------------------------------------------
// Shared-memory layouts (the host sizes the launch with the same function)
// ---------------------------------------------------------------------------
struct SelfLayout {
  int rs, wsm, xsm, wob, kv, recv, osm, pk, red, red16, bar, total;
};
__host__ __device__ inline SelfLayout self_layout(int d, int nkv) {
  SelfLayout L;
  L.rs = d * 2 + 16;
  int o = 0;
  // the o_proj block is copied into the q/k/v rows' space once the q/k/v
  // product is done (during the attention): a depth-stack self phase then
  // fits beside an FFN phase on one SM, so the FFN's weights load while the
  // self phase runs and the other way round
  L.wsm = o;
  L.wob = o;
  o = align128(o + max((kQkvRowsPerHead / kFusedCluster) * L.rs, (d / kFusedCluster) * kBlkRow));
  L.xsm = o;
  o = align128(o + 2 * L.rs);
  L.kv = o;
  o = align128(o + 2 * 2 * nkv * kBlkRow);
  L.recv = o;
  o += 2 * kQkvRowsPerHead * 4;
  L.osm = o;
  o += 2 * kBlkRow;
  L.pk = o;
  o += 2 * kSelfMaxKeys * 4;
  L.red = o;
  o += 8 * 3 * 8 * 2 * 4;
  L.red16 = o;
  o += 16 * 4;
  L.bar = o;
  o += 16;
  L.total = o;
  return L;
}

struct CrossLayout {
  int rs, wq, xsm, wob, qbuf, slots, wpart, osm, red, red16, bar, total;
};
__host__ __device__ inline CrossLayout cross_layout(int d) {
  CrossLayout L;
  L.rs = d * 2 + 16;
  int o = 0;
  L.wq = o;
  o = align128(o + 8 * L.rs);
  L.xsm = o;
  o = align128(o + L.rs);
  L.wob = o;
  o = align128(o + (d / kFusedCluster) * kBlkRow);
  L.qbuf = o;
  o += 64 * 4;
  L.slots = o;
  o += kFusedCluster * 66 * 4;
  L.wpart = o;
  o += 4 * 66 * 4;
  L.osm = o;
  o += kBlkRow;
  L.red = o;
  o += 8 * 1 * 8 * 2 * 4;
  L.red16 = o;
  o += 16 * 4;
  L.bar = o;
  o += 16;
  L.total = o;
  return L;
}

struct FfnLayout {
  int rs, rsw, wsm, xsm, wob, hbuf, hloc, red, red16, bar, total;
};
// n-tiles of 8 weight rows the FFN kernel needs for Uc units per cluster
__host__ __device__ inline int ffn_ntiles(int Uc) { return (2 * (Uc / kFusedCluster) + 7) / 8; }

// nt: the kernel's n-tile count (its template parameter), which sizes `red`
__host__ __device__ inline FfnLayout ffn_layout(int d, int Uc, int nt) {
  FfnLayout L;
  L.rs = d * 2 + 16;
  L.rsw = Uc * 2 + 16;
  const int upc = Uc / kFusedCluster;
  int o = 0;
  L.wsm = o;
  o = align128(o + 2 * upc * L.rs);
  L.xsm = o;
  o = align128(o + 2 * L.rs);
  L.wob = o;
  o = align128(o + (d / kFusedCluster) * L.rsw);
  L.hbuf = o;
  o = align128(o + 2 * L.rsw);
  L.hloc = o;
  o += 2 * upc * 4;
  L.red = o;
  o += 8 * nt * 8 * 2 * 4;
  L.red16 = o;
  o += 16 * 4;
  L.bar = o;
  o += 16;
  L.total = o;
  return L;
}

// ---------------------------------------------------------------------------
// Self phase: one 8-CTA cluster per head h; CTA r holds q/k/v rows
// h * 192 + 24 r .. + 24 and the o_proj block of output dims
// r * d/8 .. + d/8 for head h's 64 attention columns. Every CTA pushes its
// q/k/v values of both rows to all eight CTAs, so each one runs both rows'
// attention itself (one cluster barrier) and then its o_proj block.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads, 1) fused_self_kernel(const FusedSelfParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int d = p.in.d, B = p.in.B, dpc = d / kFusedCluster, nch = d >> 3;
  const int h = blockIdx.x / kFusedCluster;
  const int r = (int)cluster_ctarank();
  const int pos = p.pos, nkv = pos;  // cached keys before this position
  const SelfLayout L = self_layout(d, nkv);
  constexpr int RQ = kQkvRowsPerHead / kFusedCluster;  // 24
  uint8_t* wsm = smem + L.wsm;
  uint8_t* xsm = smem + L.xsm;
  uint8_t* wob = smem + L.wob;
  uint8_t* kvs = smem + L.kv;
  float* recv = reinterpret_cast<float*>(smem + L.recv);
  uint8_t* osm = smem + L.osm;
  float* pk = reinterpret_cast<float*>(smem + L.pk);
  float* red = reinterpret_cast<float*>(smem + L.red);
  float* red16 = reinterpret_cast<float*>(smem + L.red16);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L.bar);

  cluster_arrive_relaxed();
  uint4 nw[2];
  load_norm_chunks(p.norm_w, nch, B, nw);
  if (tid == 0) {
    mbar_init(bar, 1);      // q/k/v rows
    mbar_init(bar + 1, 1);  // o_proj block
    fence_mbar_init();
  }
  __syncthreads();
  const uint64_t pol = l2_policy(p.l2_keep != 0);
  if (tid == 0) {
    mbar_arrive_expect_tx(bar, (uint32_t)(RQ * L.rs));
    const uint8_t* src =
        reinterpret_cast<const uint8_t*>(p.wqkv) + ((size_t)h * kQkvRowsPerHead + (size_t)r * RQ) * L.rs;
    bulk_g2s_hint(wsm, src, (uint32_t)(RQ * L.rs), bar, pol);
  }
  // relative-position bias of this query for head h (a table written at load)
  float bias0 = 0.f, bias1 = 0.f;
  if (warp < B && p.bias) {
    const float* bp = p.bias + (size_t)h * p.bias_stride;
    if (lane <= pos) bias0 = bp[lane];
    if (32 + lane <= pos) bias1 = bp[32 + lane];
  }
  // cached keys / values of both rows at positions < pos: written by the
  // layer's earlier steps, which completed before the kernel ahead of this
  // one passed its own dependency wait
  {
    const int n16 = nkv * 8;  // 16-byte chunks of nkv rows of 64 bf16
    for (int i = tid; i < B * 2 * n16; i += kThreads) {
      const int bsel = i / n16, k = i - bsel * n16, b = bsel >> 1, sel = bsel & 1;
      const int row = k >> 3, part = k & 7;
      const uint8_t* src = reinterpret_cast<const uint8_t*>(sel ? p.vc : p.kc) +
                           ((((size_t)b * p.H + h) * p.cap + row) * 64) * 2 + part * 16;
      cp_async16(kvs + ((size_t)bsel * nkv + row) * kBlkRow + part * 16, src);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
  pdl_wait();
  stage_input(p.in, 0, B, nw, xsm, L.rs, blockIdx.x == 0, red16);
  zero_share(p.in.acc_clear, B * d, blockIdx.x, gridDim.x);
  pdl_launch_dependents();

  mbar_wait_bounded(bar, 0, p.in.err);
  mma_rows<3>(smem_u32(wsm), RQ, smem_u32(xsm), L.rs, B, d, red);
  __syncthreads();
  // the q/k/v rows are consumed: the o_proj block goes into their space (the
  // proxy fence orders the reads above before the copy's writes)
  if (tid == 0) {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    mbar_arrive_expect_tx(bar + 1, (uint32_t)(dpc * kBlkRow));
    bulk_g2s_hint(wob, reinterpret_cast<const uint8_t*>(p.wo_blk) + ((size_t)h * kFusedCluster + r) * dpc * kBlkRow,
                  (uint32_t)(dpc * kBlkRow), bar + 1, pol);
  }
  // q/k/v epilogue: k / v appended to the caches at `pos`; every value of
  // both rows pushed to all eight CTAs (recv[b][head row])
  cluster_wait();
  for (int idx = tid; idx < RQ * B; idx += kThreads) {
    const int rr = idx / B, b = idx - rr * B;
    const float v = rnd<bf16>(mma_rows_result<3>(red, rr, b));
    const int hr = r * RQ + rr, sect = hr >> 6, c = hr & 63;
    if (sect > 0) {
      bf16* cache = reinterpret_cast<bf16*>(sect == 1 ? p.kc : p.vc);
      cache[(((size_t)b * p.H + h) * p.cap + pos) * 64 + c] = __float2bfloat16_rn(v);
    }
#pragma unroll
    for (int q = 0; q < kFusedCluster; ++q) st_cluster_f32(recv + b * kQkvRowsPerHead + hr, (uint32_t)q, v);
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  cluster_sync();

  // self-attention of row b = warp (scale 1.0, additive bias), the
  // arithmetic of the separate attention kernel in the same order
  if (warp < B) {
    const int b = warp, nkeys = pos + 1;
    const float* qn = recv + b * kQkvRowsPerHead;
    const float* kn = qn + 64;
    const float* vn = qn + 128;
    const uint8_t* Kold = kvs + (size_t)(b * 2) * nkv * kBlkRow;
    const uint8_t* Vold = kvs + (size_t)(b * 2 + 1) * nkv * kBlkRow;
    float* pw = pk + b * kSelfMaxKeys;
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
            Vec16<bf16>::unpack(reinterpret_cast<const uint4*>(Kold + (size_t)j * kBlkRow)[ch], kf);
          }
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[e & 3] = fmaf(qn[ch * 8 + e], kf[e], acc[e & 3]);
        }
      }
      float a = (acc[0] + acc[1]) + (acc[2] + acc[3]);
      if (p.bias) a += (cc == 0 ? bias0 : bias1);
      sc[cc] = j < nkeys ? a : -INFINITY;
    }
    const float m = warp_max(fmaxf(sc[0], sc[1]));
    const float p0 = lane < nkeys ? expf(sc[0] - m) : 0.f;
    const float p1 = 32 + lane < nkeys ? expf(sc[1] - m) : 0.f;
    const float l = warp_sum(p0 + p1);
    pw[lane] = p0;
    pw[32 + lane] = p1;
    __syncwarp();
    float o0 = 0.f, o1 = 0.f;
    const uint32_t* vrow = reinterpret_cast<const uint32_t*>(Vold) + lane;
    constexpr int kVw = kBlkRow / 4;
    int jv = 0;
    for (; jv + 4 <= nkeys - 1; jv += 4) {
      uint32_t bits[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) bits[q] = vrow[(size_t)(jv + q) * kVw];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float pq = pw[jv + q];
        o0 = fmaf(pq, __uint_as_float(bits[q] << 16), o0);
        o1 = fmaf(pq, __uint_as_float(bits[q] & 0xffff0000u), o1);
      }
    }
    for (; jv < nkeys - 1; ++jv) {
      const uint32_t bits = vrow[(size_t)jv * kVw];
      const float pq = pw[jv];
      o0 = fmaf(pq, __uint_as_float(bits << 16), o0);
      o1 = fmaf(pq, __uint_as_float(bits & 0xffff0000u), o1);
    }
    {
      const float pq = pw[nkeys - 1];
      o0 = fmaf(pq, vn[2 * lane], o0);
      o1 = fmaf(pq, vn[2 * lane + 1], o1);
    }
    const __nv_bfloat162 pr = __floats2bfloat162_rn(o0 / l, o1 / l);
    reinterpret_cast<uint32_t*>(osm + b * kBlkRow)[lane] = *reinterpret_cast<const uint32_t*>(&pr);
  }
  __syncthreads();
  // o_proj block: output dims r * dpc .. + dpc of both rows
  mbar_wait_bounded(bar + 1, 0, p.in.err);
  proj_red(smem_u32(wob), kBlkRow, dpc / 8, smem_u32(osm), kBlkRow, B, 64, p.in.acc_out, d, r * dpc, p.in.err);
}

// ---------------------------------------------------------------------------
// Cross phase: one 8-CTA cluster per (row b, head h); CTA r computes cross q
// rows h * 64 + 8 r .. + 8 and attends keys [r S / 8, (r + 1) S / 8) (their K
// rows and V columns are loaded into registers before the dependency wait:
// the cache was written by encode). The eight (max, sum, out) partials are
// exchanged, every CTA combines them in rank order and runs its cross o_proj
// block.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads, 2) fused_cross_kernel(const FusedCrossParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int d = p.in.d, dpc = d / kFusedCluster, nch = d >> 3;
  const int bh = blockIdx.x / kFusedCluster, b = bh / p.H, h = bh - b * p.H;
  const int r = (int)cluster_ctarank();
  const CrossLayout L = cross_layout(d);
  uint8_t* wq = smem + L.wq;
  uint8_t* xsm = smem + L.xsm;
  uint8_t* wob = smem + L.wob;
  float* qbuf = reinterpret_cast<float*>(smem + L.qbuf);
  float* slots = reinterpret_cast<float*>(smem + L.slots);
  float* wpart = reinterpret_cast<float*>(smem + L.wpart);
  uint8_t* osm = smem + L.osm;
  float* red = reinterpret_cast<float*>(smem + L.red);
  float* red16 = reinterpret_cast<float*>(smem + L.red16);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L.bar);

  cluster_arrive_relaxed();
  uint4 nw[2];
  load_norm_chunks(p.norm_w, nch, 1, nw);
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (warp == 0) {
    const uint64_t pol = l2_policy(p.l2_keep != 0);
    if (lane == 0) mbar_arrive_expect_tx(bar, (uint32_t)(8 * L.rs + dpc * kBlkRow));
    __syncwarp();
    const uint8_t* src = reinterpret_cast<const uint8_t*>(p.wcq) + ((size_t)h * 64 + (size_t)r * 8) * L.rs;
    if (lane == 0) bulk_g2s_hint(wq, src, (uint32_t)(8 * L.rs), bar, pol);
    if (lane == 1)
      bulk_g2s_hint(wob, reinterpret_cast<const uint8_t*>(p.wco_blk) + ((size_t)h * kFusedCluster + r) * dpc * kBlkRow,
                    (uint32_t)(dpc * kBlkRow), bar, pol);
  }
  // this CTA's key slice: warp w < 4 holds keys k0 + 32 w + lane (K row) and
  // the V columns 2 lane, 2 lane + 1 of its 32 keys
  const int k0 = (int)(((long long)r * p.S) / kFusedCluster), k1 = (int)(((long long)(r + 1) * p.S) / kFusedCluster);
  const size_t base = ((size_t)b * p.H + h) * p.Smax * 64;
  const bf16* Kc = reinterpret_cast<const bf16*>(p.ck) + base;
  const bf16* Vc = reinterpret_cast<const bf16*>(p.cv) + base;
  const int j0 = k0 + warp * 32;
  const int nj = warp < 4 ? max(0, min(32, k1 - j0)) : 0;
  uint4 kr[8];
  uint32_t vr[32];
#pragma unroll
  for (int ch = 0; ch < 8; ++ch)
    kr[ch] = lane < nj ? reinterpret_cast<const uint4*>(Kc + (size_t)(j0 + lane) * 64)[ch] : make_uint4(0, 0, 0, 0);
#pragma unroll
  for (int jj = 0; jj < 32; ++jj)
    vr[jj] = jj < nj ? *reinterpret_cast<const uint32_t*>(Vc + (size_t)(j0 + jj) * 64 + 2 * lane) : 0u;

  pdl_wait();
  stage_input(p.in, b, 1, nw, xsm, L.rs, h == 0 && r == 0, red16);
  zero_share(p.in.acc_clear, p.in.B * d, blockIdx.x, gridDim.x);
  pdl_launch_dependents();

  mbar_wait_bounded(bar, 0, p.in.err);
  mma_rows<1>(smem_u32(wq), 8, smem_u32(xsm), L.rs, 1, d, red);
  __syncthreads();
  cluster_wait();
  if (tid < 8) {
    const float q = rnd<bf16>(mma_rows_result<1>(red, tid, 0));
#pragma unroll
    for (int c = 0; c < kFusedCluster; ++c) st_cluster_f32(qbuf + r * 8 + tid, (uint32_t)c, q);
  }
  cluster_sync();

  // partial attention over this CTA's keys: warp w < 4, lane = key
  if (warp < 4) {
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int ch = 0; ch < 8; ++ch) {
      float kf[8];
      Vec16<bf16>::unpack(kr[ch], kf);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e & 3] = fmaf(qbuf[ch * 8 + e], kf[e], acc[e & 3]);
    }
    const float sc = lane < nj ? (acc[0] + acc[1]) + (acc[2] + acc[3]) : -INFINITY;
    const float m = warp_max(sc);
    const float pj = (lane < nj) ? expf(sc - m) : 0.f;
    const float l = warp_sum(pj);
    float o0 = 0.f, o1 = 0.f;
#pragma unroll
    for (int jj = 0; jj < 32; ++jj) {
      const float pw = __shfl_sync(0xffffffffu, pj, jj);
      o0 = fmaf(pw, __uint_as_float(vr[jj] << 16), o0);
      o1 = fmaf(pw, __uint_as_float(vr[jj] & 0xffff0000u), o1);
    }
    float* wp = wpart + warp * 66;
    if (lane == 0) {
      wp[0] = nj > 0 ? m : -INFINITY;
      wp[1] = l;
    }
    wp[2 + 2 * lane] = o0;
    wp[3 + 2 * lane] = o1;
  }
  __syncthreads();
  // combine the warps in order, push this CTA's partial to every CTA
  if (tid < 64) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, wpart[w * 66]);
    float Ls = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float mw = wpart[w * 66];
      if (mw == -INFINITY) continue;
      const float f = expf(mw - M);
      Ls += wpart[w * 66 + 1] * f;
      O += wpart[w * 66 + 2 + tid] * f;
    }
#pragma unroll
    for (int c = 0; c < kFusedCluster; ++c) {
      st_cluster_f32(slots + r * 66 + 2 + tid, (uint32_t)c, O);
      if (tid == 0) {
        st_cluster_f32(slots + r * 66, (uint32_t)c, M);
        st_cluster_f32(slots + r * 66 + 1, (uint32_t)c, Ls);
      }
    }
  }
  cluster_sync();
  if (tid < 64) {
    float M = -INFINITY;
#pragma unroll
    for (int s2 = 0; s2 < kFusedCluster; ++s2) M = fmaxf(M, slots[s2 * 66]);
    float Ls = 0.f, O = 0.f;
#pragma unroll
    for (int s2 = 0; s2 < kFusedCluster; ++s2) {
      const float ms = slots[s2 * 66];
      if (ms == -INFINITY) continue;
      const float f = expf(ms - M);
      Ls += slots[s2 * 66 + 1] * f;
      O += slots[s2 * 66 + 2 + tid] * f;
    }
    reinterpret_cast<uint16_t*>(osm)[tid] = bf16_bits_dev(O / Ls);
  }
  __syncthreads();
  proj_red(smem_u32(wob), kBlkRow, dpc / 8, smem_u32(osm), kBlkRow, 1, 64, p.in.acc_out + (size_t)b * d, d, r * dpc,
           p.in.err);
}

// ---------------------------------------------------------------------------
// FFN phase: clusters of 8 CTAs; cluster j owns d_ff units
// [j Uc, (j + 1) Uc) (padded past ff), CTA r units j Uc + r Uc / 8 .. of it:
// wi_0 / wi_1 rows, gated GELU, the hidden values pushed to every CTA of the
// cluster; then CTA r runs wo for output dims r * d/8 .. + d/8 over the
// cluster's Uc units.
// ---------------------------------------------------------------------------
template <int NT>
__global__ void __launch_bounds__(kThreads, 1) fused_ffn_kernel(const FusedFfnParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int d = p.in.d, B = p.in.B, dpc = d / kFusedCluster, nch = d >> 3;
  const int j = blockIdx.x / kFusedCluster;
  const int r = (int)cluster_ctarank();
  const FfnLayout L = ffn_layout(d, p.Uc, NT);
  const int upc = p.Uc / kFusedCluster;
  const int u0 = j * p.Uc + r * upc;
  const int nu = max(0, min(upc, p.ff - u0));
  const int R = 2 * nu;
  uint8_t* wsm = smem + L.wsm;
  uint8_t* xsm = smem + L.xsm;
  uint8_t* wob = smem + L.wob;
  uint8_t* hbuf = smem + L.hbuf;
  float* hloc = reinterpret_cast<float*>(smem + L.hloc);
  float* red = reinterpret_cast<float*>(smem + L.red);
  float* red16 = reinterpret_cast<float*>(smem + L.red16);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L.bar);
  (void)hloc;

  cluster_arrive_relaxed();
  uint4 nw[2];
  load_norm_chunks(p.norm_w, nch, B, nw);
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  const int blk_bytes = dpc * L.rsw;
  if (warp == 0) {
    const uint64_t pol = l2_policy(p.l2_keep != 0);
    if (lane == 0) mbar_arrive_expect_tx(bar, (uint32_t)(R * L.rs + blk_bytes));
    __syncwarp();
    const uint8_t* src = reinterpret_cast<const uint8_t*>(p.wi) + (size_t)2 * u0 * L.rs;
    if (lane == 0 && R > 0) bulk_g2s_hint(wsm, src, (uint32_t)(R * L.rs), bar, pol);
    if (lane == 1)
      bulk_g2s_hint(wob, reinterpret_cast<const uint8_t*>(p.wout_blk) + ((size_t)j * kFusedCluster + r) * blk_bytes,
                    (uint32_t)blk_bytes, bar, pol);
  }
  pdl_wait();
  stage_input(p.in, 0, B, nw, xsm, L.rs, blockIdx.x == 0, red16);
  zero_share(p.in.acc_clear, B * d, blockIdx.x, gridDim.x);
  pdl_launch_dependents();

  mbar_wait_bounded(bar, 0, p.in.err);
  if (R > 0) mma_rows<NT>(smem_u32(wsm), R, smem_u32(xsm), L.rs, B, d, red);
  __syncthreads();
  // gated GELU of this CTA's units, pushed to every CTA of the cluster
  // (hbuf[b][unit of the cluster], bf16; units past ff are 0)
  cluster_wait();
  for (int idx = tid; idx < upc * B; idx += kThreads) {
    const int i = idx / B, b = idx - i * B;
    float v = 0.f;
    if (i < nu) {
      const float a = rnd<bf16>(mma_rows_result<NT>(red, 2 * i, b));
      const float g = rnd<bf16>(mma_rows_result<NT>(red, 2 * i + 1, b));
      v = __fmul_rn(gelu_approx<bf16>(a), g);
    }
    const uint16_t bits = bf16_bits_dev(v);
    uint8_t* dst = hbuf + (size_t)b * L.rsw + (size_t)(r * upc + i) * 2;
#pragma unroll
    for (int c = 0; c < kFusedCluster; ++c) st_cluster_u16(dst, (uint32_t)c, bits);
  }
  cluster_sync();
  proj_red(smem_u32(wob), L.rsw, dpc / 8, smem_u32(hbuf), L.rsw, B, p.Uc, p.in.acc_out, d, r * dpc, p.in.err);
}

// out = R(x + R(acc / 2^32)), or x when acc is null.
__global__ void __launch_bounds__(kThreads) fused_materialize_kernel(const FusedIn in, void* out) {
  pdl_wait();
  const int n = in.B * in.d;
  for (int i = blockIdx.x * kThreads + threadIdx.x; i < n; i += gridDim.x * kThreads) {
    float v = __bfloat162float(reinterpret_cast<const bf16*>(in.x)[i]);
    if (in.acc) v = rnd<bf16>(__fadd_rn(v, rnd<bf16>(fixed_to_float(in.acc[i]))));
    reinterpret_cast<bf16*>(out)[i] = __float2bfloat16_rn(v);
  }
}

template <typename P>
cudaError_t launch_cluster(void (*kern)(const P), int grid, size_t smem, cudaStream_t s, bool pdl, const P& p) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kFusedCluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

bool in_ok(const FusedIn& in) {
  return in.x && in.acc_out && in.B >= 1 && in.B <= kFusedMaxRows && in.d % 64 == 0 && in.d <= 2048 &&
         (in.acc == nullptr || in.acc != in.acc_out);
}

}  // namespace

bool fused_supported(int d, int H, int d_kv, int ff) {
  return d_kv == 64 && d % 64 == 0 && d >= 64 && d <= 2048 && H >= 1 && ff >= 16;
}

cudaError_t fused_ffn_plan(int d, int ff, int num_sms, FfnPlan* out) {
  int nc = (num_sms + kFusedCluster - 1) / kFusedCluster;
  for (; nc >= 1; --nc) {
    int uc = (ff + nc - 1) / nc;
    uc = (uc + 31) & ~31;
    const int nt = ffn_ntiles(uc);
    if (nt > 6) return cudaErrorInvalidValue;  // d_ff too large for one pass
    const FfnLayout L = ffn_layout(d, uc, nt);
    if (L.total > 227 * 1024) return cudaErrorInvalidValue;
    // how many clusters of this kernel fit on the GPU at once
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(nc * kFusedCluster);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = L.total;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kFusedCluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int fit = 0;
    cudaError_t e;
    switch (nt) {
      case 1: e = cudaOccupancyMaxActiveClusters(&fit, fused_ffn_kernel<1>, &cfg); break;
      case 2: e = cudaOccupancyMaxActiveClusters(&fit, fused_ffn_kernel<2>, &cfg); break;
      case 3: e = cudaOccupancyMaxActiveClusters(&fit, fused_ffn_kernel<3>, &cfg); break;
      case 4: e = cudaOccupancyMaxActiveClusters(&fit, fused_ffn_kernel<4>, &cfg); break;
      case 5: e = cudaOccupancyMaxActiveClusters(&fit, fused_ffn_kernel<5>, &cfg); break;
      default: e = cudaOccupancyMaxActiveClusters(&fit, fused_ffn_kernel<6>, &cfg); break;
    }
    if (e != cudaSuccess) return e;
    if (fit >= nc) {
      out->nclusters = nc;
      out->Uc = uc;
      return cudaSuccess;
    }
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_fused_self(const FusedSelfParams& p, cudaStream_t s, bool pdl) {
  if (!in_ok(p.in) || p.pos < 0 || p.pos + 1 > kSelfMaxKeys || p.pos >= p.cap || !p.wqkv || !p.wo_blk)
    return cudaErrorInvalidValue;
  const SelfLayout L = self_layout(p.in.d, p.pos);
  return launch_cluster(fused_self_kernel, p.H * kFusedCluster, (size_t)L.total, s, pdl, p);
}

cudaError_t launch_fused_cross(const FusedCrossParams& p, cudaStream_t s, bool pdl) {
  if (!in_ok(p.in) || p.S < 1 || p.S > p.Smax || (p.S + kFusedCluster - 1) / kFusedCluster > kCrossMaxKeysPerCta)
    return cudaErrorInvalidValue;
  const CrossLayout L = cross_layout(p.in.d);
  return launch_cluster(fused_cross_kernel, p.in.B * p.H * kFusedCluster, (size_t)L.total, s, pdl, p);
}

cudaError_t launch_fused_ffn(const FusedFfnParams& p, cudaStream_t s, bool pdl) {
  if (!in_ok(p.in) || p.Uc % 32 != 0 || p.nclusters < 1 || p.nclusters * p.Uc < p.ff) return cudaErrorInvalidValue;
  const int nt = ffn_ntiles(p.Uc);
  const FfnLayout L = ffn_layout(p.in.d, p.Uc, nt);
  const int grid = p.nclusters * kFusedCluster;
  switch (nt) {
    case 1: return launch_cluster(fused_ffn_kernel<1>, grid, (size_t)L.total, s, pdl, p);
    case 2: return launch_cluster(fused_ffn_kernel<2>, grid, (size_t)L.total, s, pdl, p);
    case 3: return launch_cluster(fused_ffn_kernel<3>, grid, (size_t)L.total, s, pdl, p);
    case 4: return launch_cluster(fused_ffn_kernel<4>, grid, (size_t)L.total, s, pdl, p);
    case 5: return launch_cluster(fused_ffn_kernel<5>, grid, (size_t)L.total, s, pdl, p);
    case 6: return launch_cluster(fused_ffn_kernel<6>, grid, (size_t)L.total, s, pdl, p);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_fused_materialize(const FusedIn& in, void* out, cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((in.B * in.d + kThreads - 1) / kThreads);
  cfg.blockDim = dim3(kThreads);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, fused_materialize_kernel, in, out);
}

cudaError_t fused_set_smem_limits() {
  const int mx = 227 * 1024;
  cudaError_t e = cudaFuncSetAttribute(fused_self_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(fused_cross_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(fused_ffn_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(fused_ffn_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(fused_ffn_kernel<3>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(fused_ffn_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(fused_ffn_kernel<5>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(fused_ffn_kernel<6>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
  return e;
}

}  // namespace mrtdf
