// bf16 encoder GEMM on the 5th-generation tensor cores: C = A W^T with A
// (M, K) and W (N, K) both K-major, fp32 accumulation in tensor memory.
//
// One 128 x 128 output tile per CTA, 128 threads:
//   warp 0 lane 0  TMA producer: 2-D tiled loads (128 rows x 64 k, 128-byte
//                  swizzle) of A and W into a 3-stage shared-memory ring,
//                  completion counted on a `full` mbarrier per stage;
//   warp 1 lane 0  MMA issuer: 4 x tcgen05.mma (M 128, N 128, K 16) per
//                  stage into a 128-column TMEM accumulator; tcgen05.commit
//                  frees the stage (`empty` mbarrier) once the MMAs that read
//                  it retire, and signals `done` after the last k-tile;
//   all 4 warps    epilogue: tcgen05.ld (32 lanes x 16 columns per load)
//                  from the warp's TMEM lane quarter into a bf16 tile in the
//                  freed pipeline shared memory (GEGLU applied here), then
//                  16-byte stores along output rows with the fused epilogue
//                  (store / residual add / cross-K/V scatter).
// No multicast anywhere. Launches with few output tiles may split K over a
// thread-block cluster (see the split-K section below: partial tiles move
// through st.shared::cluster stores only). Every mbarrier wait is bounded and
// reports a timeout in the stream's error word; TMEM is always released.
//
// Descriptor formats follow the sm_100 UMMA definitions (CUTLASS
// cute/arch/mma_sm100_desc.hpp): shared-memory descriptor = start >> 4,
// LBO (16-byte units) at bit 16, SBO at bit 32, version 1 at bit 46,
// layout type at bit 61 (2 = 128-byte swizzle); instruction descriptor =
// D format at bit 4, A / B formats at bits 7 / 10, N >> 3 at bit 17,
// M >> 4 at bit 24.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>

#include <mutex>

#include "common.cuh"
#include "encoder_kernels.cuh"
#include "tcgen05.cuh"

namespace mrtdf {

namespace tc {

using namespace tcg;

constexpr int BM = 128, BN = 128, BK = 64, STAGES = 3;
constexpr int A_BYTES = BM * BK * 2;  // 16 KB
constexpr int B_BYTES = BN * BK * 2;  // 16 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int SMEM_PIPE = STAGES * STAGE_BYTES;  // pipeline buffers (then the epilogue tile)
constexpr int SMEM = SMEM_PIPE + 1024 /* 1024-byte alignment slack */ + 256 /* barriers */;
constexpr uint32_t TMEM_COLS = 128;
// Epilogue tile in shared memory: 128 rows x (128 + 8) bf16 (16-byte row pad).
constexpr int kTileLd = BN + 8;
static_assert(BM * kTileLd * 2 <= STAGES * STAGE_BYTES, "epilogue tile must fit the pipeline buffers");

constexpr uint32_t kIdesc = (1u << 4)              // D: f32
                            | (1u << 7)            // A: bf16
                            | (1u << 10)           // B: bf16
                            | ((uint32_t)(BN >> 3) << 17)
                            | ((uint32_t)(BM >> 4) << 24);

__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// ---- split-K over a thread-block cluster (few output tiles, long K) -------
// CTA z of a cluster (z = blockIdx.z, cluster dims (1, 1, KSPLIT)) runs k-tiles
// [z KT / KSPLIT, (z + 1) KT / KSPLIT) into its own TMEM accumulator, pushes
// each row of its fp32 partial tile into the receive region of the CTA that
// owns that row (rows [z' * 128 / KSPLIT, ...) belong to CTA z') through
// distributed shared memory and, after one cluster barrier, sums its rows
// over the KSPLIT slots in rank order before running the epilogue on them.
constexpr int kPartLd = BN + 4;                      // floats per partial-tile row
constexpr int kPartBytes = BM * kPartLd * 4;         // 66 KB receive region (split-K launches only)
constexpr int SMEM_SPLIT = SMEM + kPartBytes;
static_assert(BM * kTileLd * 2 <= SMEM_PIPE, "epilogue tile must fit the pipeline buffers");
// 16 fp32 accumulator columns [c, c + 16) of one tile row -> bf16 tile row
// (GEGLU: 8 output columns at c / 2).
template <int EPI>
__device__ __forceinline__ void tile_row_store(__nv_bfloat16* srow, int c, const float* f) {
  typedef __nv_bfloat16 T;
  if (EPI == kEpiGeglu) {
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float a0 = rnd<T>(f[4 * i]), g0 = rnd<T>(f[4 * i + 1]);
      const float a1 = rnd<T>(f[4 * i + 2]), g1 = rnd<T>(f[4 * i + 3]);
      const __nv_bfloat162 pr =
          __floats2bfloat162_rn(__fmul_rn(gelu_approx<T>(a0), g0), __fmul_rn(gelu_approx<T>(a1), g1));
      o[i] = *reinterpret_cast<const uint32_t*>(&pr);
    }
    *reinterpret_cast<uint4*>(srow + (c >> 1)) = make_uint4(o[0], o[1], o[2], o[3]);
  } else {
    uint32_t o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const __nv_bfloat162 pr = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
      o[i] = *reinterpret_cast<const uint32_t*>(&pr);
    }
    uint4* dst = reinterpret_cast<uint4*>(srow + c);
    dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
    dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
  }
}

// Phase 2 of the epilogue: 16-byte stores along output rows (8 columns per
// chunk) for tile rows [r0, r1); the bf16 values of row r sit at stile row
// r - r0. Threads thread_id of nthreads share the chunks.
template <int EPI>
__device__ __forceinline__ void epi_store_rows(const GemmParams& p, const __nv_bfloat16* stile, int bm, int bn, int r0,
                                             int r1, int thread_id, int nthreads) {
  typedef __nv_bfloat16 T;
  constexpr int OC = (EPI == kEpiGeglu) ? BN / 2 : BN;  // output columns of the tile
  constexpr int CPR = OC / 8;                          // 16-byte chunks per row
  const int oc0 = (EPI == kEpiGeglu) ? bn / 2 : bn;
  const int ncols = (EPI == kEpiGeglu) ? p.N / 2 : p.N;
#pragma unroll 4
  for (int idx = thread_id; idx < (r1 - r0) * CPR; idx += nthreads) {
    const int rl = idx / CPR, ch = idx - rl * CPR;
    const int m = bm + r0 + rl, n = oc0 + ch * 8;
    if (m >= p.M || n >= ncols) continue;
    uint4 v = *reinterpret_cast<const uint4*>(stile + (size_t)rl * kTileLd + ch * 8);
    if (EPI == kEpiLogits) {
      // bf16-rounded values as float; 8-byte stores (the level's column
      // offset is only even)
      float* o = reinterpret_cast<float*>(p.out) + (size_t)m * p.ldo + p.out_offset + n;
      const __nv_bfloat162* v2 = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (n + 2 * i < ncols) reinterpret_cast<float2*>(o)[i] = __bfloat1622float2(v2[i]);  // N is only even
    } else if (EPI == kEpiDecQKV) {
      const int h = n / 192, rr = n - h * 192, sect = rr >> 6, cc = rr & 63;
      T* dst = sect == 0 ? reinterpret_cast<T*>(p.out) + (size_t)m * p.ldo + h * 64 + cc
                         : reinterpret_cast<T*>(sect == 1 ? p.ck : p.cv) +
                               (((size_t)m * p.H + h) * p.cap + p.pos) * 64 + cc;
      *reinterpret_cast<uint4*>(dst) = v;
    } else if (EPI == kEpiCrossKV) {
      const int two_inner = 2 * p.inner;
      const int layer = n / two_inner, within = n - layer * two_inner;
      const int kv = within / p.inner, rr = within - kv * p.inner;
      const int h = rr >> 6, cc = rr & 63;
      const int b = m / p.S, s = m - b * p.S;
      T* cache = reinterpret_cast<T*>(kv == 0 ? p.ck : p.cv);
      *reinterpret_cast<uint4*>(cache + ((((size_t)layer * p.B + b) * p.H + h) * p.Smax + s) * 64 + cc) = v;
    } else {
      T* o = reinterpret_cast<T*>(p.out) + (size_t)m * p.ldo + n;
      if (EPI == kEpiResid || EPI == kEpiDecResid) {
        const T* rsrc = EPI == kEpiResid ? o : reinterpret_cast<const T*>(p.resid) + (size_t)m * p.ldr + n;
        const uint4 rv = *reinterpret_cast<const uint4*>(rsrc);
        const __nv_bfloat162* a2 = reinterpret_cast<const __nv_bfloat162*>(&rv);
        const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&v);
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 fa = __bfloat1622float2(a2[i]), fb = __bfloat1622float2(b2[i]);
          const __nv_bfloat162 pr = __floats2bfloat162_rn(__fadd_rn(fa.x, fb.x), __fadd_rn(fa.y, fb.y));
          w[i] = *reinterpret_cast<const uint32_t*>(&pr);
        }
        v = make_uint4(w[0], w[1], w[2], w[3]);
      }
      *reinterpret_cast<uint4*>(o) = v;
    }
  }
}

template <int EPI, int KSPLIT>
__global__ void __launch_bounds__(128, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const GemmParams p, int* err) {
  extern __shared__ uint8_t tc_smem_raw[];
  // 1024-byte aligned base for the 128-byte-swizzled tiles
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* done = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  __shared__ int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bm = blockIdx.y * BM, bn = blockIdx.x * BN;
  const int KT_all = (p.K + BK - 1) / BK;
  const int kz = KSPLIT > 1 ? (int)blockIdx.z : 0;
  const int kt0 = kz * KT_all / KSPLIT, kt1 = (kz + 1) * KT_all / KSPLIT;
  const int KT = kt1 - kt0;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
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
      uint8_t* sa = smem + s * STAGE_BYTES;
      mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
      tma_load_2d(sa, &tmA, (kt0 + kt) * BK, bm, &full[s]);
      tma_load_2d(sa + A_BYTES, &tmB, (kt0 + kt) * BK, bn, &full[s]);
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
      const uint32_t sa = smem_u32(smem + s * STAGE_BYTES);
      const uint32_t sb = sa + A_BYTES;
#pragma unroll
      for (int j = 0; j < BK / 16; ++j) {
        // K-major 128B-swizzled tiles: the k-th 16-element slice starts 32 B further
        mma_f16(tmem, smem_desc_sw128(sa + j * 32), smem_desc_sw128(sb + j * 32), kIdesc, (kt | j) != 0);
      }
      mma_commit(&empty[s]);
    }
    mma_commit(done);
  }
  __syncwarp();
  // ---- epilogue: all four warps ----
  // the TMEM loads below are .sync.aligned: decide CTA-uniformly
  const bool ok = __syncthreads_and(mbar_wait_bounded(done, 0, err) ? 1 : 0) && !abort_flag;
  tc_fence_after();
  // Rows [r0, r1) of the tile get the epilogue in this CTA; their bf16 values
  // sit at stile (row r at (r - r0) * kTileLd).
  typedef __nv_bfloat16 T;
  int r0 = 0, r1 = BM;
  T* stile = reinterpret_cast<T*>(smem);
  if constexpr (KSPLIT == 1) {
    if (ok) {
      // Phase 1: TMEM -> registers -> a bf16 tile in the (now idle) pipeline
      // shared memory; thread = tile row. GEGLU pairs (a, g) become one column.
      const int r_local = warp * 32 + lane;
      const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
#pragma unroll 1
      for (int c = 0; c < BN; c += 16) {
        uint32_t r[16];
        tmem_ld16(lane_base + (uint32_t)c, r);
        tmem_wait_ld();
        float f[16];
#pragma unroll
        for (int q = 0; q < 16; ++q) f[q] = __uint_as_float(r[q]);
        tile_row_store<EPI>(stile + (size_t)r_local * kTileLd, c, f);
      }
    }
  } else {
    // Split-K: row r of this CTA's fp32 partial goes to CTA r / RS of the
    // cluster (st.shared::cluster into slot [this rank] of its receive
    // region, which the mainloop never touches, so no CTA waits for another
    // to finish its k-tiles before pushing); after one cluster barrier each
    // CTA sums its RS rows over the slots in rank order with local reads.
    constexpr int RS = BM / KSPLIT;  // rows reduced by this CTA
    float* recv = reinterpret_cast<float*>(smem + SMEM_PIPE + 256);  // after the barrier words
    if (ok) {
      const int r_local = warp * 32 + lane;
      const uint32_t owner = (uint32_t)(r_local / RS);
      float* slot_row = recv + ((size_t)kz * RS + (r_local % RS)) * kPartLd;  // same offset in the owner
      const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
#pragma unroll 1
      for (int c = 0; c < BN; c += 16) {
        uint32_t r[16];
        tmem_ld16(lane_base + (uint32_t)c, r);
        tmem_wait_ld();
#pragma unroll
        for (int q = 0; q < 4; ++q)
          st_cluster_f32x4(slot_row + c + 4 * q, owner, __uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]),
                           __uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3]));
      }
    }
    cluster_sync_all();  // every pushed partial has landed (every CTA arrives, ok or not)
    r0 = kz * RS;
    r1 = r0 + RS;
    stile = reinterpret_cast<T*>(smem);  // this CTA's pipeline buffers are idle now
    if (ok) {
      // thread -> (row, 16-column group): RS rows x 8 groups over 128 threads
      for (int item = tid; item < RS * (BN / 16); item += 128) {
        const int rr = item / (BN / 16), c = (item - rr * (BN / 16)) * 16;
        float f[16];
#pragma unroll
        for (int q = 0; q < 16; ++q) f[q] = recv[(size_t)rr * kPartLd + c + q];
#pragma unroll 1
        for (int z = 1; z < KSPLIT; ++z) {
          const float* src = recv + ((size_t)z * RS + rr) * kPartLd + c;
#pragma unroll
          for (int q = 0; q < 16; ++q) f[q] += src[q];
        }
        tile_row_store<EPI>(stile + (size_t)rr * kTileLd, c, f);
      }
    }
  }
  __syncthreads();
  if (ok) epi_store_rows<EPI>(p, stile, bm, bn, r0, r1, tid, 128);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
}

// 2-D bf16 tensor map over a row-major (rows, cols) matrix with leading
// dimension ld (elements): box 64 columns x 128 rows, 128-byte swizzle,
// zero fill outside the matrix.
bool make_map(CUtensorMap* m, const void* base, int rows, int cols, int ld) {
  auto fn = tcg::encode_tiled_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  const cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)BM};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int EPI, int KSPLIT>
cudaError_t launch_t(const CUtensorMap& a, const CUtensorMap& b, const GemmParams& p, int* err, cudaStream_t s,
                     bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((p.N + BN - 1) / BN, (p.M + BM - 1) / BM, KSPLIT);
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = KSPLIT > 1 ? SMEM_SPLIT : SMEM;
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
  return cudaLaunchKernelEx(&cfg, gemm_tc_kernel<EPI, KSPLIT>, a, b, p, err);
}

template <int EPI>
cudaError_t launch_split(const CUtensorMap& a, const CUtensorMap& b, const GemmParams& p, int ksplit, int* err,
                         cudaStream_t s, bool pdl) {
  switch (ksplit) {
    case 2: return launch_t<EPI, 2>(a, b, p, err, s, pdl);
    case 4: return launch_t<EPI, 4>(a, b, p, err, s, pdl);
    case 8: return launch_t<EPI, 8>(a, b, p, err, s, pdl);
    default: return launch_t<EPI, 1>(a, b, p, err, s, pdl);
  }
}

// Split-K factor: when the output tiles cannot fill the GPU (the decode
// projections of a wide stream: 8-44 tiles), split K over a cluster of up
// to max_ksplit CTAs while the grid stays within one wave and each CTA keeps
// >= 2 k-tiles.
int choose_ksplit(int tiles, int kt, int num_sms, int max_ksplit) {
  int k = 1;
  while (k < 8 && k < max_ksplit && tiles * k * 2 <= num_sms && kt >= 4 * k) k *= 2;
  return k;
}

}  // namespace tc

template <int EPI>
static void set_limits_epi(cudaError_t& e) {
  auto set = [&](const void* f, int bytes) {
    cudaError_t r = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (r != cudaSuccess) e = r;
  };
  set((const void*)tc::gemm_tc_kernel<EPI, 1>, tc::SMEM);
  set((const void*)tc::gemm_tc_kernel<EPI, 2>, tc::SMEM_SPLIT);
  set((const void*)tc::gemm_tc_kernel<EPI, 4>, tc::SMEM_SPLIT);
  set((const void*)tc::gemm_tc_kernel<EPI, 8>, tc::SMEM_SPLIT);
}

cudaError_t gemm_tc_set_smem_limits() {
  cudaError_t e = cudaSuccess;
  set_limits_epi<kEpiStore>(e);
  set_limits_epi<kEpiResid>(e);
  set_limits_epi<kEpiGeglu>(e);
  set_limits_epi<kEpiCrossKV>(e);
  set_limits_epi<kEpiDecResid>(e);
  set_limits_epi<kEpiDecQKV>(e);
  set_limits_epi<kEpiLogits>(e);
  return e;
}

cudaError_t launch_gemm_tc(int epi, const GemmParams& p, int* err, cudaStream_t s, bool pdl) {
  if (p.M <= 0 || p.N <= 0) return cudaSuccess;
  // 16-byte epilogue chunks: 8 output columns (16 GEMM columns for GEGLU)
  if (p.N % (epi == kEpiGeglu ? 16 : epi == kEpiLogits ? 2 : 8) != 0 || p.K % 8 != 0 || p.lda % 8 != 0)
    return cudaErrorInvalidValue;
  if (epi == kEpiLogits) {
    if (p.ldo % 2 || p.out_offset % 2 || (reinterpret_cast<uintptr_t>(p.out) & 7)) return cudaErrorInvalidValue;
  } else if (epi != kEpiCrossKV && (p.ldo % 8 != 0 || (reinterpret_cast<uintptr_t>(p.out) & 15))) {
    return cudaErrorInvalidValue;
  }
  if (epi == kEpiDecResid && (p.ldr % 8 || (reinterpret_cast<uintptr_t>(p.resid) & 15))) return cudaErrorInvalidValue;
  if (epi == kEpiDecQKV && (p.N % 192 || (reinterpret_cast<uintptr_t>(p.ck) & 15) ||
                            (reinterpret_cast<uintptr_t>(p.cv) & 15)))
    return cudaErrorInvalidValue;
  if (epi == kEpiCrossKV && (p.inner % 64 != 0 || (reinterpret_cast<uintptr_t>(p.ck) & 15) ||
                             (reinterpret_cast<uintptr_t>(p.cv) & 15)))
    return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(p.A) & 15) || (reinterpret_cast<uintptr_t>(p.W) & 15)) return cudaErrorInvalidValue;
  CUtensorMap a, b;
  if (!tc::make_map(&a, p.A, p.M, p.K, p.lda) || !tc::make_map(&b, p.W, p.N, p.K, p.K)) return cudaErrorInvalidValue;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int tiles = ((p.N + tc::BN - 1) / tc::BN) * ((p.M + tc::BM - 1) / tc::BM);
  const int ks = tc::choose_ksplit(tiles, (p.K + tc::BK - 1) / tc::BK, sms, p.max_ksplit);
  switch (epi) {
    case kEpiStore: return tc::launch_split<kEpiStore>(a, b, p, ks, err, s, pdl);
    case kEpiResid: return tc::launch_split<kEpiResid>(a, b, p, ks, err, s, pdl);
    case kEpiGeglu: return tc::launch_split<kEpiGeglu>(a, b, p, ks, err, s, pdl);
    case kEpiCrossKV: return tc::launch_split<kEpiCrossKV>(a, b, p, ks, err, s, pdl);
    case kEpiDecResid: return tc::launch_split<kEpiDecResid>(a, b, p, ks, err, s, pdl);
    case kEpiDecQKV: return tc::launch_split<kEpiDecQKV>(a, b, p, ks, err, s, pdl);
    case kEpiLogits: return tc::launch_split<kEpiLogits>(a, b, p, ks, err, s, pdl);
  }
  return cudaErrorInvalidValue;
}

}  // namespace mrtdf
