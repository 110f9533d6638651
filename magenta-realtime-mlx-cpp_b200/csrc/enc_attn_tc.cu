// Encoder self-attention (bf16) on the 5th-generation tensor cores, warp
// specialised.
//
// Reference: the encoder's MultiHeadAttention (depthformer/modules.cpp:243-321,
// scale 1.0, no mask, bidirectional) inside EncoderLayer (modules.cpp:349-358):
// softmax in fp32 over the keys of one (row, head), then P V.
//
// CTA = 128 queries of one (row, head), 320 threads:
//   warps 0-7   softmax: two threads per query row (row = TMEM lane t % 128),
//               each owning 32 of a tile's 64 key columns (the key half);
//   warp 8      TMA producer (lane 0): Q once, then K and V tiles of 64 keys
//               through a 2- or 3-stage ring, 128-byte swizzle, straight from
//               the (B*S, 3*inner) q|k|v rows;
//   warp 9      MMA issuer (lane 0): S = Q K^T (tcgen05.mma M 128, N 64) into
//               one of two 64-column TMEM buffers, then O_h += P_h V_h for the
//               two key halves h (M 128, N 64, V as an MN-major operand) into
//               two more 64-column accumulators.
// One pass over the keys. Each softmax thread keeps its own running maximum
// m over its key half and computes P = exp(s - m), l += P; m is raised only
// when a tile's maximum exceeds it by more than kLazy (then O_h and l are
// scaled by exp(m_old - m_new) once the previous P V has retired), so P stays
// below e^kLazy and rescaling is rare. The end combines the halves exactly:
// O = (a_0 O_0 + a_1 O_1) / (a_0 l_0 + a_1 l_1), a_h = exp(m_h - max(m_0, m_1)),
// i.e. softmax(s) V with fp32 sums. P is split as P_hi + P_lo (both bf16,
// P_lo = bf16(P - P_hi)) into two K-major 128 x 64 tiles (double-buffered) so
// that O += P_hi V + P_lo V keeps ~16 mantissa bits of P. S(j + 1) is issued
// before P(j) V, so the softmax of a tile overlaps the products of its
// neighbours. Keys past S are masked to P = 0 (their K / V rows are other
// rows' data or the TMA's zero fill).
// mbarriers hand every buffer between the roles; every wait is bounded, a
// failed wait stops all roles and reports in the error word, and the MMA
// issuer drains its products before TMEM (256 columns) is released.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>

#include "common.cuh"
#include "device_errors.h"
#include "encoder_kernels.cuh"
#include "tcgen05.cuh"

namespace mrtdf {

namespace {

using namespace tcg;
typedef __nv_bfloat16 bf16;

constexpr int kQ = 128;    // queries per CTA
constexpr int kKt = 64;    // keys per tile
constexpr int kDh = 64;    // head dimension
constexpr int kQBytes = kQ * kDh * 2;     // 16 KB
constexpr int kKVBytes = kKt * kDh * 2;   // 8 KB per K or V tile
constexpr int kPBytes = kQ * kKt * 2;     // 16 KB per P half
// NS K / V ring stages, NPB P buffers: NS 2, NPB 2 (113 KB, one CTA per SM)
// lets a CTA overlap the softmax of one tile with the P V of the previous
// one; NS 3, NPB 1 (97 KB) fits two CTAs per SM, which overlap each other.
template <int NS, int NPB>
struct AttnCfg {
  static constexpr int kOffQ = 0;
  static constexpr int kOffK = kOffQ + kQBytes;
  static constexpr int kOffV = kOffK + NS * kKVBytes;
  static constexpr int kOffPh = kOffV + NS * kKVBytes;
  static constexpr int kOffPl = kOffPh + NPB * kPBytes;
  static constexpr int kOffBar = kOffPl + NPB * kPBytes;
  static constexpr int kSmem = kOffBar + 256 + 1024;  // barriers, + 1024-byte alignment slack
};
constexpr uint32_t kTmemColsA = 256;  // S: 0..63 and 64..127; O_0: 128..191, O_1: 192..255
// A running maximum is raised only when a tile exceeds it by more than this
// (natural-log units): P = exp(s - m) stays below e^8 ~ 2981.
constexpr float kLazy = 8.0f;
// kind::f16, D f32, A / B bf16, M 128, N 64; K-major A and B ...
constexpr uint32_t kIdescS = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(64 >> 3) << 17) |
                             ((uint32_t)(128 >> 4) << 24);
// ... and for P V the B operand (V: keys x dims, dims contiguous) MN-major (bit 16)
constexpr uint32_t kIdescPV = kIdescS | (1u << 16);

__device__ __forceinline__ void umma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                     uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// 16-byte chunk c of 128-byte row r of a 128-byte-swizzled tile
__device__ __forceinline__ uint32_t sw128(int row, int chunk) {
  return (uint32_t)(row * 128 + ((chunk ^ (row & 7)) << 4));
}

struct Bars {
  uint64_t* q_full;
  uint64_t* kv_full;   // [kNS]
  uint64_t* kv_empty;  // [kNS]
  uint64_t* s_full;    // [2]
  uint64_t* s_empty;   // [2]
  uint64_t* p_full;    // [2]
  uint64_t* p_empty;   // [2]
  uint64_t* o_done;
  uint64_t* drain;
};

// kSplit softmax threads per query row, each taking 64 / kSplit key columns
template <int kSplit>
constexpr int threads_of() { return 128 * kSplit + 64; }  // + the TMA and MMA warps

template <int kNS, int kNPB, int kSplit>
__global__ void __launch_bounds__(threads_of<kSplit>(), (kNPB == 1 ? 2 : 1))
    enc_attn_tc_kernel(const __grid_constant__ CUtensorMap tm, const EncAttnParams p) {
  constexpr int kSoft = 128 * kSplit;
  constexpr int kCols = kKt / kSplit;  // key columns per softmax thread
  typedef AttnCfg<kNS, kNPB> C;
  constexpr int kOffQ = C::kOffQ, kOffK = C::kOffK, kOffV = C::kOffV, kOffPh = C::kOffPh, kOffPl = C::kOffPl,
                kOffBar = C::kOffBar;
  extern __shared__ uint8_t raw_smem[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw_smem) + 1023) & ~uintptr_t(1023));
  uint64_t* b0 = reinterpret_cast<uint64_t*>(smem + kOffBar);
  const Bars br{b0, b0 + 1, b0 + 1 + kNS, b0 + 1 + 2 * kNS, b0 + 3 + 2 * kNS, b0 + 5 + 2 * kNS, b0 + 7 + 2 * kNS,
                b0 + 9 + 2 * kNS, b0 + 10 + 2 * kNS};
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(b0 + 11 + 2 * kNS);
  __shared__ int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int q0 = blockIdx.x * kQ;
  const int bh = blockIdx.y, b = bh / p.H, h = bh - b * p.H;
  const int S = p.S;
  const int row0 = b * S;  // first q|k|v row of this sequence
  const int nkt = (S + kKt - 1) / kKt;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemColsA)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 32) {
    mbar_init(br.q_full, 1);
    for (int s = 0; s < kNS; ++s) {
      mbar_init(br.kv_full + s, 1);
      mbar_init(br.kv_empty + s, 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(br.s_full + i, 1);
      mbar_init(br.s_empty + i, kSoft);
      mbar_init(br.p_full + i, kSoft);
      mbar_init(br.p_empty + i, 1);
    }
    mbar_init(br.o_done, 1);
    mbar_init(br.drain, 1);
    fence_mbar_init();
    abort_flag = 0;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  pdl_launch_dependents();
  pdl_wait();

  auto wait = [&](uint64_t* bar, uint32_t parity) -> bool {
    if (*(volatile int*)&abort_flag) return false;
    if (mbar_wait_bounded(bar, parity, p.err)) return true;
    *(volatile int*)&abort_flag = 1;
    return false;
  };

  if (warp == kSoft / 32) {
    // ---- TMA producer ----
    if (lane == 0) {
      const int xq = h * kDh, xk = p.inner + h * kDh, xv = 2 * p.inner + h * kDh;
      mbar_arrive_expect_tx(br.q_full, kQBytes);
      tma_load_2d(smem + kOffQ, &tm, xq, row0 + q0, br.q_full);  // 64-row boxes: two loads
      tma_load_2d(smem + kOffQ + kQBytes / 2, &tm, xq, row0 + q0 + 64, br.q_full);
      int issued = 0;
      for (int u = 0; u < nkt; ++u) {
        const int st = u % kNS;
        if (u >= kNS && !wait(br.kv_empty + st, (uint32_t)(((u / kNS) - 1) & 1))) break;
        mbar_arrive_expect_tx(br.kv_full + st, 2 * kKVBytes);
        tma_load_2d(smem + kOffK + st * kKVBytes, &tm, xk, row0 + u * kKt, br.kv_full + st);
        tma_load_2d(smem + kOffV + st * kKVBytes, &tm, xv, row0 + u * kKt, br.kv_full + st);
        issued = u + 1;
      }
      // no copy may still be landing when the CTA exits: wait (bounded) for
      // the last load of each stage and for Q
      for (int u = (issued > kNS ? issued - kNS : 0); u < issued; ++u)
        mbar_wait_bounded(br.kv_full + u % kNS, (uint32_t)((u / kNS) & 1), p.err);
      mbar_wait_bounded(br.q_full, 0, p.err);
    }
  } else if (warp == kSoft / 32 + 1) {
    // ---- MMA issuer ----
    if (lane == 0) {
      const uint32_t aq = smem_u32(smem + kOffQ);
      bool ok = wait(br.q_full, 0);
      auto issue_s = [&](int u) -> bool {
        const int st = u % kNS, sb = u & 1;
        if (!wait(br.kv_full + st, (uint32_t)((u / kNS) & 1))) return false;
        if (u >= 2 && !wait(br.s_empty + sb, (uint32_t)(((u >> 1) - 1) & 1))) return false;
        tc_fence_after();
        const uint32_t ak = smem_u32(smem + kOffK + st * kKVBytes);
#pragma unroll
        for (int kk = 0; kk < kDh / 16; ++kk)
          umma(tmem + (uint32_t)(sb * 64), smem_desc_sw128(aq + kk * 32), smem_desc_sw128(ak + kk * 32), kIdescS,
               kk != 0);
        mma_commit(br.s_full + sb);
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; ok && j < nkt; ++j) {
        const int st = j % kNS, pb = j % kNPB;
        if (j + 1 < nkt && !(ok = issue_s(j + 1))) break;
        if (!(ok = wait(br.p_full + pb, (uint32_t)((j / kNPB) & 1)))) break;
        tc_fence_after();
        const uint32_t aph = smem_u32(smem + kOffPh + pb * kPBytes), apl = smem_u32(smem + kOffPl + pb * kPBytes);
        const uint32_t av = smem_u32(smem + kOffV + st * kKVBytes);
        // K-major P: the k-th 16-key slice starts 32 bytes further; MN-major
        // V: 16 keys = 16 rows of 128 bytes further (two 8-row swizzle atoms).
        // Slices 0, 1 (keys 0-31) go to O_0, slices 2, 3 to O_1.
#pragma unroll
        for (int kk = 0; kk < kKt / 16; ++kk)
          umma(tmem + 128 + (uint32_t)(kk >> 1) * 64, smem_desc_sw128(aph + kk * 32), smem_desc_sw128(av + kk * 2048),
               kIdescPV, (j != 0 || (kk & 1)) ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < kKt / 16; ++kk)
          umma(tmem + 128 + (uint32_t)(kk >> 1) * 64, smem_desc_sw128(apl + kk * 32), smem_desc_sw128(av + kk * 2048),
               kIdescPV, 1u);
        mma_commit(br.p_empty + pb);
        mma_commit(br.kv_empty + st);
      }
      if (ok) mma_commit(br.o_done);
      // every product issued so far has retired before TMEM is released
      mma_commit(br.drain);
      mbar_wait_bounded(br.drain, 0, p.err);
    }
  } else {
    // ---- softmax: two threads per query row: row = TMEM lane = tid % 128,
    // half = tid / 128 owns key columns 32 half .. + 32 of every S tile and
    // the accumulator O_half ----
    static_assert(kSplit == 2, "one O accumulator per key half");
    __shared__ float xm[kSplit][kQ], xl[kSplit][kQ];
    const int row = tid & (kQ - 1), half = tid >> 7;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const int c0 = half * kCols;
    const uint32_t ocol = 128u + (uint32_t)half * 64u;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; ok && j < nkt; ++j) {
      const int sb = j & 1, pb = j % kNPB;
      ok = wait(br.s_full + sb, (uint32_t)((j >> 1) & 1));
      // the TMEM accesses below are .sync.aligned: decide warp-uniformly
      if (!(ok = __all_sync(0xffffffffu, ok) != 0)) break;
      tc_fence_after();
      uint32_t r[kCols];
      tmem_ld16(tmem + lane_base + (uint32_t)(sb * 64 + c0), r);
      tmem_ld16(tmem + lane_base + (uint32_t)(sb * 64 + c0 + 16), r + 16);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(br.s_empty + sb);
      const int kb = j * kKt + c0;  // key of r[0]
      float mt = -INFINITY;
#pragma unroll
      for (int q = 0; q < kCols; ++q)
        if (kb + q < S) mt = fmaxf(mt, __uint_as_float(r[q]));
      float alpha = 1.f;
      bool resc = false;
      if (mt > m + kLazy) {  // also the first tile with a key (m = -inf)
        if (m != -INFINITY) {
          alpha = __expf(m - mt);
          resc = true;
        }
        m = mt;
        l *= alpha;
      }
      if (__any_sync(0xffffffffu, resc)) {
        // O_half holds products made with the old maximum: once P(j - 1) V
        // has retired (j >= 1: the old maximum came from an earlier tile),
        // scale it in TMEM; the next P V is issued after this thread's
        // p_full arrival below
        ok = wait(br.p_empty + (j - 1) % kNPB, (uint32_t)(((j - 1) / kNPB) & 1));
        if (!(ok = __all_sync(0xffffffffu, ok) != 0)) break;
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 64; c += 16) {
          uint32_t o[16];
          tmem_ld16(tmem + lane_base + ocol + (uint32_t)c, o);
          tmem_wait_ld();
#pragma unroll
          for (int q = 0; q < 16; ++q) o[q] = __float_as_uint(__uint_as_float(o[q]) * alpha);
          tmem_st16(tmem + lane_base + ocol + (uint32_t)c, o);
        }
        tmem_wait_st();
      }
      if (j >= kNPB) {
        ok = wait(br.p_empty + pb, (uint32_t)(((j / kNPB) - 1) & 1));
        if (!(ok = __all_sync(0xffffffffu, ok) != 0)) break;
      }
      uint8_t* ph = smem + kOffPh + pb * kPBytes;
      uint8_t* pl = smem + kOffPl + pb * kPBytes;
#pragma unroll
      for (int c = 0; c < kCols; c += 16) {
        uint32_t hi[8], lo[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int k0 = kb + c + 2 * e;
          const float a0 = k0 < S ? __expf(__uint_as_float(r[c + 2 * e]) - m) : 0.f;
          const float a1 = k0 + 1 < S ? __expf(__uint_as_float(r[c + 2 * e + 1]) - m) : 0.f;
          l += a0;
          l += a1;
          hi[e] = pack_bf16(a0, a1);
          lo[e] = pack_bf16(a0 - __uint_as_float(hi[e] << 16), a1 - __uint_as_float(hi[e] & 0xffff0000u));
        }
        const int ch = (c0 + c) >> 3;  // 16-byte chunk of the 128-byte row
        *reinterpret_cast<uint4*>(ph + sw128(row, ch)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        *reinterpret_cast<uint4*>(ph + sw128(row, ch + 1)) = make_uint4(hi[4], hi[5], hi[6], hi[7]);
        *reinterpret_cast<uint4*>(pl + sw128(row, ch)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        *reinterpret_cast<uint4*>(pl + sw128(row, ch + 1)) = make_uint4(lo[4], lo[5], lo[6], lo[7]);
      }
      tc_fence_before();
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive(br.p_full + pb);
    }
    if (ok) ok = wait(br.o_done, 0);
    // combine the halves (every softmax thread passes here once)
    xm[half][row] = m;
    xl[half][row] = l;
    asm volatile("bar.sync 1, %0;" ::"n"(kSoft) : "memory");
    const float m0 = xm[0][row], m1 = xm[1][row];
    const float mx = fmaxf(m0, m1);  // finite: key 0 is in half 0
    const float w0 = m0 == -INFINITY ? 0.f : __expf(m0 - mx);
    const float w1 = m1 == -INFINITY ? 0.f : __expf(m1 - mx);
    const float inv_l = 1.0f / (w0 * xl[0][row] + w1 * xl[1][row]);
    ok = __all_sync(0xffffffffu, ok) != 0;
    if (ok) {
      tc_fence_after();
      const int qr = q0 + row;
      bf16* out = reinterpret_cast<bf16*>(p.out) + ((size_t)row0 + qr) * p.inner + h * kDh;
#pragma unroll
      for (int c = 0; c < kCols; c += 16) {
        uint32_t x0[16], x1[16];
        tmem_ld16(tmem + lane_base + (uint32_t)(128 + c0 + c), x0);
        tmem_ld16(tmem + lane_base + (uint32_t)(192 + c0 + c), x1);
        tmem_wait_ld();
        uint32_t w[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float v0 = (w0 * __uint_as_float(x0[2 * q]) + w1 * __uint_as_float(x1[2 * q])) * inv_l;
          const float v1 = (w0 * __uint_as_float(x0[2 * q + 1]) + w1 * __uint_as_float(x1[2 * q + 1])) * inv_l;
          w[q] = pack_bf16(v0, v1);
        }
        if (qr < S) {
          reinterpret_cast<uint4*>(out + c0 + c)[0] = make_uint4(w[0], w[1], w[2], w[3]);
          reinterpret_cast<uint4*>(out + c0 + c)[1] = make_uint4(w[4], w[5], w[6], w[7]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemColsA) : "memory");
  }
}

// 2-D bf16 tensor map over the (rows, 3 * inner) q|k|v rows: box 64 columns
// (one head) x 64 rows, 128-byte swizzle, zero fill past the last row.
bool make_qkv_map(CUtensorMap* m, const void* base, int rows, int cols) {
  auto fn = encode_tiled_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  const cuuint32_t box[2] = {64, 64};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

// per-shape variants: one wave (few CTAs) / many waves. Two softmax threads
// per row, one per key half and O accumulator (four per row measured slower
// in a two-pass version, 1.51 vs 1.48 ms at one CFG pair).
constexpr int kSplitFew = 2, kSplitMany = 2;

cudaError_t enc_attn_tc_set_smem_limits() {
  cudaError_t e = cudaFuncSetAttribute(enc_attn_tc_kernel<2, 2, kSplitFew>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       AttnCfg<2, 2>::kSmem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(enc_attn_tc_kernel<3, 1, kSplitMany>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             AttnCfg<3, 1>::kSmem);
  return e;
}

cudaError_t launch_enc_attention_tc(const EncAttnParams& p, cudaStream_t s, bool pdl) {
  if (p.inner % 64 != 0 || p.S <= 0 || !p.err || (reinterpret_cast<uintptr_t>(p.qkv) & 15) ||
      (reinterpret_cast<uintptr_t>(p.out) & 15))
    return cudaErrorInvalidValue;
  CUtensorMap tm;
  if (!make_qkv_map(&tm, p.qkv, p.B * p.S, 3 * p.inner)) return cudaErrorInvalidValue;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const dim3 grid((p.S + kQ - 1) / kQ, p.B * p.H);
  // one wave at one CTA per SM: the in-CTA overlap of NS 2 / NPB 2 wins (one
  // CFG pair: encoder pass 1.54 vs 1.69 ms); many waves: two CTAs per SM
  // (16 / 128 rows: 13.3 / 103.9 ms vs 15.7 / 119.3)
  const bool few = (long long)grid.x * grid.y <= 2LL * sms;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(few ? threads_of<kSplitFew>() : threads_of<kSplitMany>());
  cfg.dynamicSmemBytes = few ? AttnCfg<2, 2>::kSmem : AttnCfg<3, 1>::kSmem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return few ? cudaLaunchKernelEx(&cfg, enc_attn_tc_kernel<2, 2, kSplitFew>, tm, p)
             : cudaLaunchKernelEx(&cfg, enc_attn_tc_kernel<3, 1, kSplitMany>, tm, p);
}

}  // namespace mrtdf
