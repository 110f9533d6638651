// Fused epilogues shared by the encoder GEMM kernels (mma.sync and
// tcgen05): each call handles two adjacent output columns (n, n + 1), n even.
#pragma once

#include "common.cuh"
#include "encoder_kernels.cuh"

namespace mrtdf {

template <typename T, int EPI>
__device__ __forceinline__ void epi_pair(const GemmParams& p, int m, int n, float v0, float v1) {
  if (m >= p.M || n >= p.N) return;
  T* out = reinterpret_cast<T*>(p.out);
  if (EPI == kEpiStore) {
    out[(size_t)m * p.ldo + n] = from_f<T>(v0);
    out[(size_t)m * p.ldo + n + 1] = from_f<T>(v1);
  } else if (EPI == kEpiResid) {
    T* o = out + (size_t)m * p.ldo + n;
    o[0] = from_f<T>(__fadd_rn(to_f(o[0]), rnd<T>(v0)));
    o[1] = from_f<T>(__fadd_rn(to_f(o[1]), rnd<T>(v1)));
  } else if (EPI == kEpiGeglu) {
    const float a = rnd<T>(v0), g = rnd<T>(v1);
    out[(size_t)m * p.ldo + (n >> 1)] = from_f<T>(__fmul_rn(gelu_approx<T>(a), g));
  } else {  // kEpiCrossKV
    const int two_inner = 2 * p.inner;
    const int layer = n / two_inner, within = n - layer * two_inner;
    const int kv = within / p.inner, rr = within - kv * p.inner;
    const int h = rr >> 6, cc = rr & 63;
    const int b = m / p.S, s = m - b * p.S;
    T* cache = reinterpret_cast<T*>(kv == 0 ? p.ck : p.cv);
    T* dst = cache + ((((size_t)layer * p.B + b) * p.H + h) * p.Smax + s) * 64 + cc;
    dst[0] = from_f<T>(v0);
    dst[1] = from_f<T>(v1);
  }
}

}  // namespace mrtdf
