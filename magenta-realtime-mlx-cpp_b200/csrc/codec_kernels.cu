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
//                  2-D load of the weight tile, into a 3- or 4-stage ring;
//   warp 1 lane 0  MMA issuer: 4 x tcgen05.mma kind::tf32 (M 128, N BN,
//                  K 8) per stage into a BN-column TMEM accumulator;
//   all 4 warps    epilogue: tcgen05.ld of the thread's accumulator row,
//                  bias, ELU, residual, then 64-byte stores per 16 channels.
// No multicast. Every mbarrier wait is bounded (error word, CTA exits after
// releasing its TMEM).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "codec_kernels.cuh"
#include "common.cuh"
#include "device_errors.h"
#include "tcgen05.cuh"

namespace mrtdf {

namespace cv {

using namespace tcg;

constexpr int BM = 128, BK = kConvBK;
constexpr int A_BYTES = BM * BK * 4;  // 16 KB, 1024-byte multiple (swizzle atoms)

// Unsplit launches use a 3-stage ring (96 KB at BN 128), so two CTAs share an
// SM and one CTA's epilogue overlaps the other's mainloop; split-K launches
// keep 4 stages (their receive region leaves room for one CTA per SM).
template <int BN, int KSPLIT>
struct Cfg {
  static constexpr int STAGES = KSPLIT > 1 ? 4 : 3;
  static constexpr int B_BYTES = BN * BK * 4;
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int PART_LD = BN + 4;  // floats per partial-tile row in the split-K receive region
  static constexpr int SMEM = STAGES * STAGE + 1024 /* alignment slack */ + 256 /* barriers */ +
                              (KSPLIT > 1 ? BM * PART_LD * 4 : 0);
  // instruction descriptor: D f32 (bit 4), A / B tf32 (format 2 at bits 7 /
  // 10), both K-major, N >> 3 at bit 17, M >> 4 at bit 24
  static constexpr uint32_t IDESC = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(BN >> 3) << 17) |
                                    ((uint32_t)(BM >> 4) << 24);
  static_assert(B_BYTES % 1024 == 0, "weight tile must keep the 1024-byte swizzle alignment");
};

__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// elu with alpha 1 (nn_ops.h:31-39)
__device__ __forceinline__ float elu1(float v) { return v > 0.f ? v : expf(v) - 1.0f; }

// ---- split-K over a thread-block cluster --------------------------------------
// Layers with few output tiles and long K (the decoder's first layers: 12-140
// CTAs, up to 144 k-tiles) split K over a cluster of KSPLIT CTAs (grid z,
// cluster dims (1, 1, KSPLIT)): CTA z runs k-tiles [z KT / KSPLIT, (z + 1) KT /
// KSPLIT) into its own TMEM accumulator, pushes every row of its fp32 partial
// tile into the receive region of the CTA that owns the row (rows
// [z' 128 / KSPLIT, ...) belong to CTA z') with st.shared::cluster, and after
// one cluster barrier each CTA sums its rows over the slots in rank order
// (deterministic) and runs the epilogue on them. The receive region lies past
// the pipeline buffers, so no CTA waits for another's mainloop to push.
// Epilogue of one accumulator row r, output channels [n, n + 16): the row's
// output position, then bias, ELU, residual, stores (raw and / or ELU'd,
// the stereo split folded into the address). Rows outside the tile's valid
// positions or the output image are skipped.
__device__ __forceinline__ void epi16(const ConvParams& p, int img, int qy0, int qx0, int r, int n, float* f) {
  const int ly = r / p.wt, lx = r - ly * p.wt;
  const int qy = qy0 + ly, qx = qx0 + lx;
  const int oy = qy * p.osy + p.ory, ox = qx * p.osx + p.orx;
  if (!(r < p.wt * p.ht && qy < p.q0y + p.hq && qx < p.q0x + p.wq && oy >= 0 && oy < p.ho && ox >= 0 &&
        ox < p.wo))
    return;
#pragma unroll
  for (int q = 0; q < 16; q += 4) {
    const float4 b4 = *reinterpret_cast<const float4*>(p.bias + n + q);
    f[q] += b4.x;
    f[q + 1] += b4.y;
    f[q + 2] += b4.z;
    f[q + 3] += b4.w;
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

template <int BN, int KSPLIT>
__global__ void __launch_bounds__(128, KSPLIT > 1 ? 1 : 2)
    conv_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const ConvParams p, int* err) {
  typedef Cfg<BN, KSPLIT> C;
  constexpr int STAGES = C::STAGES;
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
  const int KT_all = p.ntaps * kc;
  const int kz = KSPLIT > 1 ? (int)blockIdx.z : 0;
  const int kt0 = kz * KT_all / KSPLIT, kt1 = (kz + 1) * KT_all / KSPLIT;
  const int KT = kt1 - kt0;
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
    for (int i = 0; i < KT; ++i) {
      const int s = i % STAGES, round = i / STAGES;
      if (round > 0 && !mbar_wait_bounded(&empty[s], (uint32_t)((round - 1) & 1), err)) {
        abort_flag = 1;
        break;
      }
      const int kt = kt0 + i;
      const int tap = kt / kc, c0 = (kt - tap * kc) * BK;
      const int ty = tap / p.ntx, tx = tap - ty * p.ntx;
      uint8_t* sa = smem + s * C::STAGE;
      mbar_arrive_expect_tx(&full[s], tx_bytes);
      tma_load_4d(sa, &tmA, c0, qx0 + p.ax0 + tx * p.adx, qy0 + p.ay0 + ty * p.ady, img, &full[s]);
      tma_load_2d(sa + A_BYTES, &tmB, kt * BK, bn, &full[s]);
    }
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer ----
    for (int i = 0; i < KT; ++i) {
      const int s = i % STAGES, round = i / STAGES;
      if (!mbar_wait_bounded(&full[s], (uint32_t)(round & 1), err)) {
        abort_flag = 1;
        break;
      }
      tc_fence_after();
      const uint32_t sa = smem_u32(smem + s * C::STAGE);
      const uint32_t sb = sa + A_BYTES;
#pragma unroll
      for (int j = 0; j < BK / 8; ++j)  // K 8 per instruction = 32 bytes along the swizzled row
        mma_tf32(tmem, smem_desc_sw128(sa + j * 32), smem_desc_sw128(sb + j * 32), C::IDESC, (i | j) != 0);
      mma_commit(&empty[s]);
    }
    mma_commit(done);
  }
  __syncwarp();
  // the TMEM loads below are .sync.aligned: decide CTA-uniformly
  const bool ok = __syncthreads_and(mbar_wait_bounded(done, 0, err) ? 1 : 0) && !abort_flag;
  tc_fence_after();
  const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
  if constexpr (KSPLIT == 1) {
    if (ok) {
      // accumulator row r (TMEM lane) = tile position (r / wt, r % wt)
      const int r = warp * 32 + lane;
#pragma unroll 1
      for (int c = 0; c < BN; c += 16) {
        uint32_t v[16];
        tmem_ld16(lane_base + (uint32_t)c, v);
        tmem_wait_ld();
        float f[16];
#pragma unroll
        for (int q = 0; q < 16; ++q) f[q] = __uint_as_float(v[q]);
        epi16(p, img, qy0, qx0, r, bn + c, f);
      }
    }
  } else {
    constexpr int RS = BM / KSPLIT;  // rows reduced by this CTA
    constexpr int LD = C::PART_LD;
    float* recv = reinterpret_cast<float*>(smem + STAGES * C::STAGE + 256);  // past the barrier words
    if (ok) {
      const int r = warp * 32 + lane;
      const uint32_t owner = (uint32_t)(r / RS);
      float* slot_row = recv + ((size_t)kz * RS + (r % RS)) * LD;  // the same offset in the owner
#pragma unroll 1
      for (int c = 0; c < BN; c += 16) {
        uint32_t v[16];
        tmem_ld16(lane_base + (uint32_t)c, v);
        tmem_wait_ld();
#pragma unroll
        for (int q = 0; q < 4; ++q)
          st_cluster_f32x4(slot_row + c + 4 * q, owner, __uint_as_float(v[4 * q]), __uint_as_float(v[4 * q + 1]),
                           __uint_as_float(v[4 * q + 2]), __uint_as_float(v[4 * q + 3]));
      }
    }
    cluster_sync_all();  // every pushed partial has landed (every CTA arrives, ok or not)
    if (ok) {
      for (int item = tid; item < RS * (BN / 16); item += 128) {
        const int rr = item / (BN / 16), c = (item - rr * (BN / 16)) * 16;
        float f[16];
#pragma unroll
        for (int q = 0; q < 16; q += 4) {
          const float4 a = *reinterpret_cast<const float4*>(recv + (size_t)rr * LD + c + q);
          f[q] = a.x;
          f[q + 1] = a.y;
          f[q + 2] = a.z;
          f[q + 3] = a.w;
        }
#pragma unroll 1
        for (int z = 1; z < KSPLIT; ++z) {
          const float* src = recv + ((size_t)z * RS + rr) * LD + c;
#pragma unroll
          for (int q = 0; q < 16; q += 4) {
            const float4 a = *reinterpret_cast<const float4*>(src + q);
            f[q] += a.x;
            f[q + 1] += a.y;
            f[q + 2] += a.z;
            f[q + 3] += a.w;
          }
        }
        epi16(p, img, qy0, qx0, kz * RS + rr, bn + c, f);
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

// Input activation (in_n, in_h, in_w, cin) as a 4-D map {cin, in_w, in_h,
// in_n}: box 32 channels x wt x ht x 1, 128-byte swizzle, zero fill.
bool make_map_act(CUtensorMap* m, const ConvParams& p) {
  auto fn = tcg::encode_tiled_fn();
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
  auto fn = tcg::encode_tiled_fn();
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

template <int BN, int KSPLIT>
cudaError_t launch_bn(const CUtensorMap& a, const CUtensorMap& b, const ConvParams& p, int* err, cudaStream_t s,
                      bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(p.tiles_x * p.tiles_y * p.n_img), (unsigned)(p.cout / BN), KSPLIT);
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = Cfg<BN, KSPLIT>::SMEM;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (KSPLIT > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = 1;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = KSPLIT;
    ++n;
  }
  if (pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, conv_tc_kernel<BN, KSPLIT>, a, b, p, err);
}

template <int BN>
cudaError_t launch_split(const ConvParams& p, int ks, int* err, cudaStream_t s, bool pdl) {
  CUtensorMap a, b;
  if (!make_map_act(&a, p) || !make_map_wgt(&b, p, BN)) return cudaErrorInvalidValue;
  switch (ks) {
    case 2: return launch_bn<BN, 2>(a, b, p, err, s, pdl);
    case 4: return launch_bn<BN, 4>(a, b, p, err, s, pdl);
    case 8: return launch_bn<BN, 8>(a, b, p, err, s, pdl);
    default: return launch_bn<BN, 1>(a, b, p, err, s, pdl);
  }
}

// Split-K factor from the layer's tile count for ONE sequence (split_tiles),
// so the summation order, and with it every output bit, does not depend on
// how many sequences share the launch: double while the split grid of one
// sequence stays within half the SMs and each CTA keeps >= 4 k-tiles.
int choose_ksplit(int split_tiles, int kt, int num_sms) {
  int k = 1;
  while (k < 8 && split_tiles * k * 2 <= num_sms && kt >= 4 * k) k *= 2;
  return k;
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

__global__ void __launch_bounds__(256, 2) out_conv_kernel(const OutConvParams p) {
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
      // the thread's 10 input rows of this column tap, 8 channels each, in
      // registers: every weight pair read below serves all 4 output rows
      float4 xa[kOcRows + 6], xb[kOcRows + 6];
#pragma unroll
      for (int rr = 0; rr < kOcRows + 6; ++rr) {
        const float* xp = xs + ((ty * kOcRows + rr) * kOcSpan + tx + dx) * kOcStride;
        xa[rr] = *reinterpret_cast<const float4*>(xp);
        xb[rr] = *reinterpret_cast<const float4*>(xp + 4);
      }
#pragma unroll
      for (int dy = 0; dy < 7; ++dy) {
#pragma unroll
        for (int o = 0; o < 2; ++o) {
          const float* wp = ws + ((o * 7 + dy) * 7 + dx) * 64 + c0;
          const float4 w0 = *reinterpret_cast<const float4*>(wp);
          const float4 w1 = *reinterpret_cast<const float4*>(wp + 4);
#pragma unroll
          for (int i = 0; i < kOcRows; ++i) {
            const float4 a = xa[i + dy], b = xb[i + dy];
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
// istft_frames_kernel: block (frame pair, stereo s, batch b) computes the
// windowed time samples of two consecutive frames, every thread four sample
// indices n, so each twiddle pair read serves two frames. A frame sample is
// the real inverse DFT of its 480 bins and a zero Nyquist bin,
// x[n] = (X_0.re + 2 sum_{k=1}^{479} (X_k.re cos(2 pi k n / 960) -
// X_k.im sin(2 pi k n / 960))) / 960, with the twiddle index k n mod 960
// stepped incrementally and sin read from the cosine table shifted by 720.
// istft_ola_kernel: the overlap-add (frame i at j plus frame i - 1 at
// j + 480), the trim to `target` and the stereo interleave.
constexpr int kFft = 960, kHop = 480, kFramesPerBlock = 2;

__global__ void __launch_bounds__(256) istft_frames_kernel(const IstftParams p) {
  __shared__ float cs[kFft];
  __shared__ float2 X[kFramesPerBlock][kHop];
  const int f0 = blockIdx.x * kFramesPerBlock, s = blockIdx.y, b = blockIdx.z, tid = threadIdx.x;
  for (int m = tid; m < kFft; m += 256) cs[m] = p.cosv[m];
  pdl_wait();
  for (int i = tid; i < kFramesPerBlock * kHop; i += 256) {
    const int f = i / kHop, k = i - f * kHop;
    float2 v = make_float2(0.f, 0.f);
    if (f0 + f < p.frames)
      v = *reinterpret_cast<const float2*>(p.spec + (((size_t)b * p.frames + f0 + f) * kHop + k) * 4 + 2 * s);
    X[f][k] = v;
  }
  __syncthreads();
  const bool four = tid + 768 < kFft;  // warps 0-5 take four sample indices, warps 6-7 three
  float acc[4][kFramesPerBlock];
  int m[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    m[j] = 0;
#pragma unroll
    for (int f = 0; f < kFramesPerBlock; ++f) acc[j][f] = 0.f;
  }
#pragma unroll 2
  for (int k = 1; k < kHop; ++k) {
    float2 x[kFramesPerBlock];
#pragma unroll
    for (int f = 0; f < kFramesPerBlock; ++f) x[f] = X[f][k];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (j == 3 && !four) break;
      m[j] += tid + 256 * j;
      if (m[j] >= kFft) m[j] -= kFft;
      int ms = m[j] + 720;
      if (ms >= kFft) ms -= kFft;
      const float c = cs[m[j]], sn = cs[ms];
#pragma unroll
      for (int f = 0; f < kFramesPerBlock; ++f) {
        acc[j][f] = fmaf(x[f].x, c, acc[j][f]);
        acc[j][f] = fmaf(-x[f].y, sn, acc[j][f]);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int n = tid + 256 * j;
    if (n >= kFft) break;
#pragma unroll
    for (int f = 0; f < kFramesPerBlock; ++f)
      if (f0 + f < p.frames)
        p.frames_buf[(((size_t)b * 2 + s) * p.frames + f0 + f) * kFft + n] =
            ((X[f][0].x + 2.0f * acc[j][f]) / (float)kFft) * p.synth[n];
  }
}

__global__ void __launch_bounds__(256) istft_ola_kernel(const IstftParams p) {
  const size_t idx = (size_t)blockIdx.x * 256 + threadIdx.x;  // (b, t, s) of the interleaved output
  pdl_wait();
  if (idx >= (size_t)p.B * p.target * 2) return;
  const int s = (int)(idx & 1);
  const size_t bt = idx >> 1;
  const int b = (int)(bt / p.target), t = (int)(bt - (size_t)b * p.target);
  const int i = t / kHop, j = t - i * kHop;
  const float* fr = p.frames_buf + ((size_t)b * 2 + s) * p.frames * kFft;
  float v = 0.f;
  if (i < p.frames) v = fr[(size_t)i * kFft + j];
  if (i >= 1) v += fr[(size_t)(i - 1) * kFft + j + kHop];
  p.audio[idx] = v;
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

template <int BN>
static void conv_limits(cudaError_t& e) {
  auto set = [&](const void* f, int bytes) {
    if (e == cudaSuccess) e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  };
  set((const void*)cv::conv_tc_kernel<BN, 1>, cv::Cfg<BN, 1>::SMEM);
  set((const void*)cv::conv_tc_kernel<BN, 2>, cv::Cfg<BN, 2>::SMEM);
  set((const void*)cv::conv_tc_kernel<BN, 4>, cv::Cfg<BN, 4>::SMEM);
  set((const void*)cv::conv_tc_kernel<BN, 8>, cv::Cfg<BN, 8>::SMEM);
}

cudaError_t conv_tc_set_smem_limits() {
  cudaError_t e = cudaSuccess;
  conv_limits<64>(e);
  conv_limits<128>(e);
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
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int bn = p.cout % 128 == 0 ? 128 : 64;
  const int ks = cv::choose_ksplit(std::max(1, p.split_tiles) * (p.cout / bn), p.ntaps * (p.cin / cv::BK), sms);
  if (bn == 128) return cv::launch_split<128>(p, ks, err, s, pdl);
  return cv::launch_split<64>(p, ks, err, s, pdl);
}

cudaError_t launch_out_conv(const OutConvParams& p, cudaStream_t s, bool pdl) {
  if (p.H <= p.crop || p.W <= 0 || p.B <= 0) return cudaErrorInvalidValue;
  const dim3 grid((p.W + cv::kOcTile - 1) / cv::kOcTile, (p.H - p.crop + cv::kOcTile - 1) / cv::kOcTile, 2 * p.B);
  return cv::launch_simple(cv::out_conv_kernel, grid, dim3(32, 8), cv::kOcSmem, p, s, pdl);
}

cudaError_t launch_istft(const IstftParams& p, cudaStream_t s, bool pdl) {
  if (p.B <= 0 || p.frames <= 0 || p.target <= 0 || p.target > (p.frames + 1) * cv::kHop || !p.frames_buf)
    return cudaErrorInvalidValue;
  const dim3 grid((p.frames + cv::kFramesPerBlock - 1) / cv::kFramesPerBlock, 2, p.B);
  cudaError_t e = cv::launch_simple(cv::istft_frames_kernel, grid, dim3(256), 0, p, s, pdl);
  if (e != cudaSuccess) return e;
  const size_t n = (size_t)p.B * p.target * 2;
  return cv::launch_simple(cv::istft_ola_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, p, s, pdl);
}

cudaError_t launch_dequant(const DequantParams& p, cudaStream_t s, bool pdl) {
  if (p.B <= 0 || p.S <= 0 || p.levels <= 0 || p.D <= 0 || p.D > 1024 || p.pad_frames < 0) return cudaErrorInvalidValue;
  return cv::launch_simple(cv::dequant_kernel, dim3(p.S + p.pad_frames, p.B), dim3(p.D), 0, p, s, pdl);
}

}  // namespace mrtdf
