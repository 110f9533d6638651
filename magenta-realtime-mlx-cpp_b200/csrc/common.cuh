// Device-side building blocks shared by every kernel of the engine:
// bf16 storage helpers, sm_100a PTX wrappers (mbarrier, TMA bulk copy,
// programmatic dependent launch), warp reductions, and the arithmetic that
// must match the CPU oracle bit for bit (Philox4x32-10, the uniform ->
// Gumbel transform, the CFG mix).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "device_errors.h"

namespace mrtdf {

// Longest a device-side wait may take before it gives up and reports
// through the error word: 0.5 s of %globaltimer. A healthy wait takes
// microseconds; the bound keeps a lost completion from holding the GPU.
constexpr unsigned long long kWaitTimeoutNs = 500000000ull;

// ---------------------------------------------------------------------------
// Storage types
// ---------------------------------------------------------------------------
__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// Round a float to the storage type T and back: identity for fp32, RNE to
// bf16 for bf16 (MLX rounds every bf16 op output this way).
template <typename T>
__device__ __forceinline__ float rnd(float v) { return to_f(from_f<T>(v)); }

// Unpack 16 bytes of T into floats: 8 bf16 or 4 fp32.
template <typename T>
struct Vec16;
template <>
struct Vec16<__nv_bfloat16> {
  static constexpr int N = 8;
  __device__ __forceinline__ static void unpack(const uint4& u, float* f) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
};
template <>
struct Vec16<float> {
  static constexpr int N = 4;
  __device__ __forceinline__ static void unpack(const uint4& u, float* f) {
    f[0] = __uint_as_float(u.x);
    f[1] = __uint_as_float(u.y);
    f[2] = __uint_as_float(u.z);
    f[3] = __uint_as_float(u.w);
  }
};

// ---------------------------------------------------------------------------
// Warp helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch (sm_90+). `wait` blocks until every grid this
// one depends on has completed and its memory is visible; `launch_dependents`
// lets the next kernel in the stream start its prologue early.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------------------
// mbarrier + TMA bulk copy (cp.async.bulk, no tensor map: a contiguous byte
// range global -> shared, completion counted in bytes on an mbarrier).
// Both addresses 16-byte aligned, size a multiple of 16.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait: returns false (and sets the kErrMbarTimeout bit of `err`)
// when the phase has not flipped within `timeout_ns` of %globaltimer. The
// timer is read once per 32 polls, so the fast path costs one try_wait.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int* err,
                                                  unsigned long long timeout_ns = kWaitTimeoutNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  for (;;) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > timeout_ns) break;
  }
  if (err) atomicOr(err, kErrMbarTimeout);
  return false;
}

__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------------------
// Bit-exact sampler arithmetic. Every float op below is an explicitly
// rounded intrinsic (no fused multiply-add), so the result equals the CPU
// oracle's -ffp-contract=off build bit for bit.
// ---------------------------------------------------------------------------
// Philox4x32-10 (Salmon et al., SC'11).
__device__ __forceinline__ void philox4x32_10(uint32_t c[4], uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(0xD2511F53u, c[0]), lo0 = 0xD2511F53u * c[0];
    const uint32_t hi1 = __umulhi(0xCD9E8D57u, c[2]), lo1 = 0xCD9E8D57u * c[2];
    const uint32_t n0 = hi1 ^ c[1] ^ k0;
    const uint32_t n2 = hi0 ^ c[3] ^ k1;
    c[0] = n0;
    c[1] = lo1;
    c[2] = n2;
    c[3] = lo0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
}

// Uniform in (0, 1) for vocabulary index `idx` at decode step `step`:
// counter (idx / 4, step, 0, 0), key = seed, word idx % 4,
// value (2 * (x >> 9) + 1) * 2^-24.
__device__ __forceinline__ float philox_uniform(uint64_t seed, uint32_t step, uint32_t idx) {
  uint32_t c[4] = {idx >> 2, step, 0u, 0u};
  philox4x32_10(c, (uint32_t)seed, (uint32_t)(seed >> 32));
  const uint32_t x = c[idx & 3u];
  return __fmul_rn((float)((x >> 9) * 2u + 1u), 1.0f / 16777216.0f);
}

// ln(x) for positive normal x from basic rounded ops: x = m 2^e,
// m in [sqrt(1/2), sqrt(2)), s = (m-1)/(m+1), ln m = 2 atanh(s) by its
// odd power series through s^13, ln x = e ln2_hi + ln m + e ln2_lo.
__device__ __forceinline__ float exact_log(float x) {
  const uint32_t u = __float_as_uint(x);
  int e = (int)((u >> 23) & 0xffu) - 127;
  float m = __uint_as_float((u & 0x007fffffu) | 0x3f800000u);
  if (m > 0x1.6a09e6p+0f) {
    m = __fmul_rn(m, 0.5f);
    e = e + 1;
  }
  const float s = __fdiv_rn(__fsub_rn(m, 1.0f), __fadd_rn(m, 1.0f));
  const float s2 = __fmul_rn(s, s);
  float p = 0x1.3b13b2p-4f;
  p = __fadd_rn(__fmul_rn(p, s2), 0x1.745d18p-4f);
  p = __fadd_rn(__fmul_rn(p, s2), 0x1.c71c72p-4f);
  p = __fadd_rn(__fmul_rn(p, s2), 0x1.24924ap-3f);
  p = __fadd_rn(__fmul_rn(p, s2), 0x1.99999ap-3f);
  p = __fadd_rn(__fmul_rn(p, s2), 0x1.555556p-2f);
  p = __fadd_rn(__fmul_rn(p, s2), 1.0f);
  const float lnm = __fmul_rn(2.0f, __fmul_rn(s, p));
  const float fe = (float)e;
  return __fadd_rn(__fadd_rn(__fmul_rn(fe, 0x1.62e4p-1f), lnm), __fmul_rn(fe, 0x1.7f7d1cp-20f));
}

__device__ __forceinline__ float gumbel_from_uniform(float u) {
  const float a = -exact_log(u);
  return -exact_log(a);
}

// cfg_combine: (1 + w) * cond - w * uncond, products rounded separately.
__device__ __forceinline__ float cfg_mix(float cond, float uncond, float w) {
  const float sc = __fadd_rn(1.0f, w);
  return __fsub_rn(__fmul_rn(sc, cond), __fmul_rn(w, uncond));
}

// Map a float to a uint32 whose unsigned order equals the float order.
__device__ __forceinline__ uint32_t float_order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float float_from_order_key(uint32_t k) {
  const uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(u);
}

// tanh-approximate GELU with the reference's op order and per-op rounding
// to T (gelu_approx, nn_ops.h:66-84; constants cast to the input dtype).
template <typename T>
__device__ __forceinline__ float gelu_approx(float x) {
  const float c0 = rnd<T>(0.7978845608028654f), c1 = rnd<T>(0.044715f);
  const float x2 = rnd<T>(__fmul_rn(x, x));
  const float t1 = rnd<T>(__fmul_rn(c1, x2));
  const float t2 = rnd<T>(__fadd_rn(1.0f, t1));
  const float t3 = rnd<T>(__fmul_rn(x, t2));
  const float inner = rnd<T>(__fmul_rn(c0, t3));
  const float th = rnd<T>(tanhf(inner));
  const float uu = rnd<T>(__fadd_rn(1.0f, th));
  const float v = rnd<T>(__fmul_rn(x, uu));
  return rnd<T>(__fmul_rn(0.5f, v));
}

}  // namespace mrtdf
