// SpectroStream decode phase on the device (see codec_kernels.cuh).
//
// Reference (rhymeswithlion/magenta-realtime-mlx-cpp):
//   rvq_dequantization                 src/magenta_realtime_mlx/rvq.cpp:68-87
//   WNConv2d / WNConvTranspose2d       spectrostream.cpp:125-157
//   Res1x1Block / Res3x3Block          spectrostream.cpp:163-199
//   DecoderResBlock                    spectrostream.cpp:202-267
//   SpectroStreamDecoder::operator()   spectrostream.cpp:365-419
//   istft_postprocess                  spectrostream.cpp:593-681
//   elu                                nn_ops.h:31-39
//
// conv_tc_kernel: implicit-GEMM convolution on the 5th-generation tensor
// cores. One 128-position x BN-channel output tile per CTA, 128 threads:
//   warp 0 lane 0  TMA producer: per k-tile (tap, 32 input channels) one 4-D
//                  tiled load of the input (box 32 channels x wt x ht
//                  positions, 128-byte swizzle; out-of-range coordinates
//                  read zero, which is the convolution's padding) and one
//                  2-D load of the weight tile, into a 4-stage ring;
//   warp 1 lane 0  MMA issuer: 4 x tcgen05.mma kind::tf32 (M 128, N BN,
//                  K 8) per stage into a BN-column TMEM accumulator;
//   all 4 warps    epilogue: tcgen05.ld of the thread's accumulator row,
//                  bias, ELU, residual, then 64-byte stores per 16 channels.
// No multicast. Every mbarrier wait is bounded (error word, CTA exits after
// releasing its TMEM).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "codec_kernels.cuh"
#include "common.cuh"
#include "device_errors.h"

namespace mrtdf {

namespace cv {

constexpr int BM = 128, BK = kConvBK, STAGES = 4;
constexpr int A_BYTES = BM * BK * 4;  // 16 KB, 1024-byte multiple (swizzle atoms)

template <int BN>
struct Cfg {
  static constexpr int B_BYTES = BN * BK * 4;
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int SMEM = STAGES * STAGE + 1024 /* alignment slack */ + 256 /* barriers */;
  // instruction descriptor: D f32 (bit 4), A / B tf32 (format 2 at bits 7 /
  // 10), both K-major, N >> 3 at bit 17, M >> 4 at bit 24
  static constexpr uint32_t IDESC = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(BN >> 3) << 17) |
                                    ((uint32_t)(BM >> 4) << 24);
  static_assert(B_BYTES % 1024 == 0, "weight tile must keep the 1024-byte swizzle alignment");
};

__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// elu with alpha 1 (nn_ops.h:31-39)
__device__ __forceinline__ float elu1(float v) { return v > 0.f ? v : expf(v) - 1.0f; }

template <int BN>
__global__ void __launch_bounds__(128, 1)
    conv_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const ConvParams p, int* err) {
  typedef Cfg<BN> C;
  extern __shared__ uint8_t cv_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(cv_smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * C::STAGE);
  uint64_t* empty = full + STAGES;
  uint64_t* done = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  __shared__ int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  int t = blockIdx.x;
  const int tile_x = t % p.tiles_x;
  t /= p.tiles_x;
  const int tile_y = t % p.tiles_y;
  const int img = t / p.tiles_y;
  const int qy0 = p.q0y + tile_y * p.ht, qx0 = p.q0x + tile_x * p.wt;
  const int bn = blockIdx.y * BN;
  const int kc = p.cin / BK;  // k-tiles per tap
  const int KT = p.ntaps * kc;
  const uint32_t tx_bytes = (uint32_t)(BK * 4 * p.wt * p.ht + C::B_BYTES);

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"((uint32_t)BN)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 32) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    fence_mbar_init();
    abort_flag = 0;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  pdl_launch_dependents();
  pdl_wait();

  if (warp == 0 && lane == 0) {
    // ---- TMA producer ----
    for (int kt = 0; kt < KT; ++kt) {
      const int s = kt % STAGES, round = kt / STAGES;
      if (round > 0 && !mbar_wait_bounded(&empty[s], (uint32_t)((round - 1) & 1), err)) {
        abort_flag = 1;
        break;
      }
      const int tap = kt / kc, c0 = (kt - tap * kc) * BK;
      const int ty = tap / p.ntx, tx = tap - ty * p.ntx;
      uint8_t* sa = smem + s * C::STAGE;
      mbar_arrive_expect_tx(&full[s], tx_bytes);
      tma_load_4d(sa, &tmA, c0, qx0 + p.ax0 + tx * p.adx, qy0 + p.ay0 + ty * p.ady, img, &full[s]);
      tma_load_2d(sa + A_BYTES, &tmB, kt * BK, bn, &full[s]);
    }
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer ----
    for (int kt = 0; kt < KT; ++kt) {
      const int s = kt % STAGES, round = kt / STAGES;
      if (!mbar_wait_bounded(&full[s], (uint32_t)(round & 1), err)) {
        abort_flag = 1;
        break;
      }
      tc_fence_after();
      const uint32_t sa = smem_u32(smem + s * C::STAGE);
      const uint32_t sb = sa + A_BYTES;
#pragma unroll
      for (int j = 0; j < BK / 8; ++j)  // K 8 per instruction = 32 bytes along the swizzled row
        mma_tf32(tmem, smem_desc_sw128(sa + j * 32), smem_desc_sw128(sb + j * 32), C::IDESC, (kt | j) != 0);
      mma_commit(&empty[s]);
    }
    mma_commit(done);
  }
  __syncwarp();
  // the TMEM loads below are .sync.aligned: decide CTA-uniformly
  const bool ok = __syncthreads_and(mbar_wait_bounded(done, 0, err) ? 1 : 0) && !abort_flag;
  tc_fence_after();
  if (ok) {
    // accumulator row r (TMEM lane) = tile position (r / wt, r % wt)
    const int r = warp * 32 + lane;
    const int ly = r / p.wt, lx = r - ly * p.wt;
    const int qy = qy0 + ly, qx = qx0 + lx;
    const int oy = qy * p.osy + p.ory, ox = qx * p.osx + p.orx;
    const bool valid = r < p.wt * p.ht && qy < p.q0y + p.hq && qx < p.q0x + p.wq && oy >= 0 && oy < p.ho &&
                       ox >= 0 && ox < p.wo;
    const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
#pragma unroll 1
    for (int c = 0; c < BN; c += 16) {
      uint32_t v[16];
      tmem_ld16(lane_base + (uint32_t)c, v);
      tmem_wait_ld();
      if (!valid) continue;
      const int n = bn + c;
      float f[16];
#pragma unroll
      for (int q = 0; q < 16; q += 4) {
        const float4 b4 = *reinterpret_cast<const float4*>(p.bias + n + q);
        f[q] = __uint_as_float(v[q]) + b4.x;
        f[q + 1] = __uint_as_float(v[q + 1]) + b4.y;
        f[q + 2] = __uint_as_float(v[q + 2]) + b4.z;
        f[q + 3] = __uint_as_float(v[q + 3]) + b4.w;
      }
      if (p.elu_acc) {
#pragma unroll
        for (int q = 0; q < 16; ++q) f[q] = elu1(f[q]);
      }
      if (p.resid) {
        const float* rp = p.resid + (((size_t)img * p.rh + oy / p.rsy) * p.rw + ox / p.rsx) * p.cout + n;
#pragma unroll
        for (int q = 0; q < 16; q += 4) {
          const float4 r4 = *reinterpret_cast<const float4*>(rp + q);
          f[q] += r4.x;
          f[q + 1] += r4.y;
          f[q + 2] += r4.z;
          f[q + 3] += r4.w;
        }
      }
      int oimg = img, oc = p.cout, nn = n;
      if (p.split > 0) {
        oimg = (n / p.split) * p.n_img + img;
        nn = n - (n / p.split) * p.split;
        oc = p.split;
      }
      const size_t off = (((size_t)oimg * p.ho + oy) * p.wo + ox) * oc + nn;
      if (p.out_raw) {
        float4* dst = reinterpret_cast<float4*>(p.out_raw + off);
#pragma unroll
        for (int q = 0; q < 4; ++q) dst[q] = make_float4(f[4 * q], f[4 * q + 1], f[4 * q + 2], f[4 * q + 3]);
      }
      if (p.out_elu) {
        float4* dst = reinterpret_cast<float4*>(p.out_elu + off);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          dst[q] = make_float4(elu1(f[4 * q]), elu1(f[4 * q + 1]), elu1(f[4 * q + 2]), elu1(f[4 * q + 3]));
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)BN) : "memory");
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

// Input activation (in_n, in_h, in_w, cin) as a 4-D map {cin, in_w, in_h,
// in_n}: box 32 channels x wt x ht x 1, 128-byte swizzle, zero fill.
bool make_map_act(CUtensorMap* m, const ConvParams& p) {
  auto fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[4] = {(cuuint64_t)p.cin, (cuuint64_t)p.in_w, (cuuint64_t)p.in_h, (cuuint64_t)p.in_n};
  const cuuint64_t strides[3] = {(cuuint64_t)p.cin * 4, (cuuint64_t)p.in_w * p.cin * 4,
                                 (cuuint64_t)p.in_h * p.in_w * p.cin * 4};
  const cuuint32_t box[4] = {(cuuint32_t)BK, (cuuint32_t)p.wt, (cuuint32_t)p.ht, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float*>(p.in), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Weights (cout, ntaps * cin) row-major: box 32 x bn rows.
bool make_map_wgt(CUtensorMap* m, const ConvParams& p, int bn) {
  auto fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t K = (cuuint64_t)p.ntaps * p.cin;
  const cuuint64_t dims[2] = {K, (cuuint64_t)p.cout};
  const cuuint64_t strides[1] = {K * 4};
  const cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)bn};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(p.wgt), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN>
cudaError_t launch_bn(const ConvParams& p, int* err, cudaStream_t s, bool pdl) {
  CUtensorMap a, b;
  if (!make_map_act(&a, p) || !make_map_wgt(&b, p, BN)) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(p.tiles_x * p.tiles_y * p.n_img), (unsigned)(p.cout / BN), 1);
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = Cfg<BN>::SMEM;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  int n = 0;
  if (pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, conv_tc_kernel<BN>, a, b, p, err);
}

// ---- output convolution 7x7, 64 -> 2 (SIMT) --------------------------------
// Block (32, 8): thread (tx, ty) computes output column ox0 + tx and rows
// r0 + 4 ty + i (i < 4) of a 32 x 32 tile, both output channels. Input rows
// and columns of the tile (+6 rows above, +3 columns each side: the causal
// padding of causal_same_pad(x, {7, 7}, {1, 1})) are staged 8 channels at a
// time in shared memory with a 12-float pixel stride (conflict-free 16-byte
// loads); the weights sit in shared memory whole and are read as broadcasts.
constexpr int kOcTile = 32, kOcRows = 4, kOcCh = 8, kOcStride = 12, kOcSpan = kOcTile + 6;
constexpr int kOcXFloats = kOcSpan * kOcSpan * kOcStride;
constexpr int kOcWFloats = 2 * 49 * 64;
constexpr int kOcSmem = (kOcXFloats + kOcWFloats) * 4;

__global__ void __launch_bounds__(256) out_conv_kernel(const OutConvParams p) {
  extern __shared__ float oc_sm[];
  float* xs = oc_sm;
  float* ws = oc_sm + kOcXFloats;
  const int tx = threadIdx.x, ty = threadIdx.y, tid = ty * 32 + tx;
  const int img = blockIdx.z;
  const int ox0 = blockIdx.x * kOcTile;
  const int r0 = blockIdx.y * kOcTile;  // first output row after the crop
  const int oy0 = r0 + p.crop;          // the same row before the crop
  for (int i = tid; i < kOcWFloats / 4; i += 256)
    reinterpret_cast<float4*>(ws)[i] = reinterpret_cast<const float4*>(p.wgt)[i];
  float acc[kOcRows][2];
#pragma unroll
  for (int i = 0; i < kOcRows; ++i) {
    acc[i][0] = p.bias[0];
    acc[i][1] = p.bias[1];
  }
  pdl_wait();
  for (int c0 = 0; c0 < 64; c0 += kOcCh) {
    __syncthreads();  // the previous chunk is consumed (and the weights are staged)
    for (int i = tid; i < kOcSpan * kOcSpan * 2; i += 256) {
      const int pix = i >> 1, half = i & 1;
      const int ly = pix / kOcSpan, lx = pix - ly * kOcSpan;
      const int y = oy0 - 6 + ly, x = ox0 - 3 + lx;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (y >= 0 && y < p.H && x >= 0 && x < p.W)
        v = *reinterpret_cast<const float4*>(p.in + (((size_t)img * p.H + y) * p.W + x) * 64 + c0 + half * 4);
      *reinterpret_cast<float4*>(xs + pix * kOcStride + half * 4) = v;
    }
    __syncthreads();
#pragma unroll 1
    for (int dx = 0; dx < 7; ++dx) {
#pragma unroll
      for (int rr = 0; rr < kOcRows + 6; ++rr) {
        const float* xp = xs + ((ty * kOcRows + rr) * kOcSpan + tx + dx) * kOcStride;
        const float4 a = *reinterpret_cast<const float4*>(xp);
        const float4 b = *reinterpret_cast<const float4*>(xp + 4);
#pragma unroll
        for (int i = 0; i < kOcRows; ++i) {
          const int dy = rr - i;
          if (dy < 0 || dy > 6) continue;
#pragma unroll
          for (int o = 0; o < 2; ++o) {
            const float* wp = ws + ((o * 7 + dy) * 7 + dx) * 64 + c0;
            const float4 w0 = *reinterpret_cast<const float4*>(wp);
            const float4 w1 = *reinterpret_cast<const float4*>(wp + 4);
            float s = acc[i][o];
            s = fmaf(a.x, w0.x, s);
            s = fmaf(a.y, w0.y, s);
            s = fmaf(a.z, w0.z, s);
            s = fmaf(a.w, w0.w, s);
            s = fmaf(b.x, w1.x, s);
            s = fmaf(b.y, w1.y, s);
            s = fmaf(b.z, w1.z, s);
            s = fmaf(b.w, w1.w, s);
            acc[i][o] = s;
          }
        }
      }
    }
  }
  // stereo recombine: image s * B + b -> spec[b, row, col, 2 s + o]
  const int st = img / p.B, b = img - st * p.B;
  const int ox = ox0 + tx;
  const int Hc = p.H - p.crop;
#pragma unroll
  for (int i = 0; i < kOcRows; ++i) {
    const int r = r0 + ty * kOcRows + i;
    if (r < Hc && ox < p.W) {
      float2* dst = reinterpret_cast<float2*>(p.spec + (((size_t)b * Hc + r) * p.W + ox) * 4 + 2 * st);
      *dst = make_float2(acc[i][0], acc[i][1]);
    }
  }
}

// ---- iSTFT: irfft (n 960) + synthesis window + overlap-add -----------------
// Block (hop i, stereo s, batch b) writes samples [480 i, 480 (i + 1)) of
// channel s: frame i at n = j plus frame i - 1 at n = j + 480. Each frame
// sample is the real inverse DFT of its 480 bins and a zero Nyquist bin,
// x[n] = (X_0.re + 2 sum_{k=1}^{479} (X_k.re cos(2 pi k n / 960) -
// X_k.im sin(2 pi k n / 960))) / 960, with the twiddle index k n mod 960
// stepped incrementally and sin read from the cosine table shifted by 720.
constexpr int kFft = 960, kHop = 480;

__device__ __forceinline__ float irfft_sample(const float2* X, const float* cs, int n) {
  float acc = 0.f;
  int m = 0;
#pragma unroll 4
  for (int k = 1; k < kHop; ++k) {
    m += n;
    if (m >= kFft) m -= kFft;
    int ms = m + 720;
    if (ms >= kFft) ms -= kFft;
    acc = fmaf(X[k].x, cs[m], acc);
    acc = fmaf(-X[k].y, cs[ms], acc);
  }
  return (X[0].x + 2.0f * acc) / (float)kFft;
}

__global__ void __launch_bounds__(256) istft_kernel(const IstftParams p) {
  __shared__ float cs[kFft];
  __shared__ float2 Xa[kHop], Xb[kHop];
  const int i = blockIdx.x, s = blockIdx.y, b = blockIdx.z, tid = threadIdx.x;
  for (int m = tid; m < kFft; m += 256) cs[m] = p.cosv[m];
  pdl_wait();
  for (int k = tid; k < kHop; k += 256) {
    float2 a = make_float2(0.f, 0.f), c = make_float2(0.f, 0.f);
    if (i < p.frames) a = *reinterpret_cast<const float2*>(p.spec + (((size_t)b * p.frames + i) * kHop + k) * 4 + 2 * s);
    if (i >= 1)
      c = *reinterpret_cast<const float2*>(p.spec + (((size_t)b * p.frames + i - 1) * kHop + k) * 4 + 2 * s);
    Xa[k] = a;
    Xb[k] = c;
  }
  __syncthreads();
  for (int j = tid; j < kHop; j += 256) {
    const int t = i * kHop + j;
    if (t >= p.target) continue;
    float v = 0.f;
    if (i < p.frames) v = irfft_sample(Xa, cs, j) * p.synth[j];
    if (i >= 1) v += irfft_sample(Xb, cs, j + kHop) * p.synth[j + kHop];
    p.audio[((size_t)b * p.target + t) * 2 + s] = v;
  }
}

// ---- RVQ dequantisation ------------------------------------------------------
// Block (frame s, batch b), thread d: sum over levels k = 0, 1, ... of
// codebooks[k][code][d] in float32 (the reference's order); frames >= S
// (the decoder's appended zero frame) are written as zeros. A code outside
// [0, C) sets kErrBadToken and contributes codebook row 0.
__global__ void dequant_kernel(const DequantParams p) {
  const int s = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
  pdl_wait();
  float acc = 0.f;
  if (s < p.S) {
    for (int k = 0; k < p.levels; ++k) {
      int code = p.codes[((size_t)b * p.S + s) * p.levels + k];
      if (code < 0 || code >= p.C) {
        if (d == 0) atomicOr(p.err, kErrBadToken);
        code = 0;
      }
      acc += p.codebooks[((size_t)k * p.C + code) * p.D + d];
    }
  }
  p.out[((size_t)b * (p.S + p.pad_frames) + s) * p.D + d] = acc;
}

template <typename K, typename P>
cudaError_t launch_simple(K kernel, dim3 grid, dim3 block, size_t smem, const P& p, cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  int n = 0;
  if (pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, p);
}

}  // namespace cv

cudaError_t conv_tc_set_smem_limits() {
  cudaError_t e = cudaFuncSetAttribute(cv::conv_tc_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       cv::Cfg<64>::SMEM);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(cv::conv_tc_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             cv::Cfg<128>::SMEM);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(cv::out_conv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, cv::kOcSmem);
  return e;
}

cudaError_t launch_conv_tc(const ConvParams& p, int* err, cudaStream_t s, bool pdl) {
  // shapes the kernel relies on: 32-channel k-tiles, whole BN-column tiles,
  // 16-channel epilogue chunks, a tile of at most 128 positions inside one
  // TMA box (<= 256 per dimension), 16-byte aligned operands and outputs
  if (p.cin <= 0 || p.cin % cv::BK || p.ntaps <= 0 || p.ntx <= 0 || p.cout % 64) return cudaErrorInvalidValue;
  if (p.wt <= 0 || p.ht <= 0 || p.wt * p.ht > cv::BM || p.wt > 256 || p.ht > 256) return cudaErrorInvalidValue;
  if (p.tiles_x <= 0 || p.tiles_y <= 0 || p.n_img <= 0 || p.osy <= 0 || p.osx <= 0) return cudaErrorInvalidValue;
  if (p.split > 0 && (p.split % 16 || p.cout % p.split)) return cudaErrorInvalidValue;
  if (p.resid && (p.rsy <= 0 || p.rsx <= 0)) return cudaErrorInvalidValue;
  auto mis = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) != 0; };
  if (mis(p.in) || mis(p.wgt) || mis(p.bias) || (p.resid && mis(p.resid)) || (p.out_raw && mis(p.out_raw)) ||
      (p.out_elu && mis(p.out_elu)))
    return cudaErrorInvalidValue;
  if (p.cout % 128 == 0) return cv::launch_bn<128>(p, err, s, pdl);
  return cv::launch_bn<64>(p, err, s, pdl);
}

cudaError_t launch_out_conv(const OutConvParams& p, cudaStream_t s, bool pdl) {
  if (p.H <= p.crop || p.W <= 0 || p.B <= 0) return cudaErrorInvalidValue;
  const dim3 grid((p.W + cv::kOcTile - 1) / cv::kOcTile, (p.H - p.crop + cv::kOcTile - 1) / cv::kOcTile, 2 * p.B);
  return cv::launch_simple(cv::out_conv_kernel, grid, dim3(32, 8), cv::kOcSmem, p, s, pdl);
}

cudaError_t launch_istft(const IstftParams& p, cudaStream_t s, bool pdl) {
  if (p.B <= 0 || p.frames <= 0 || p.target <= 0 || p.target > (p.frames + 1) * cv::kHop) return cudaErrorInvalidValue;
  const dim3 grid((p.target + cv::kHop - 1) / cv::kHop, 2, p.B);
  return cv::launch_simple(cv::istft_kernel, grid, dim3(256), 0, p, s, pdl);
}

cudaError_t launch_dequant(const DequantParams& p, cudaStream_t s, bool pdl) {
  if (p.B <= 0 || p.S <= 0 || p.levels <= 0 || p.D <= 0 || p.D > 1024 || p.pad_frames < 0) return cudaErrorInvalidValue;
  return cv::launch_simple(cv::dequant_kernel, dim3(p.S + p.pad_frames, p.B), dim3(p.D), 0, p, s, pdl);
}

}  // namespace mrtdf
