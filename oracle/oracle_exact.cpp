// TEST INFRASTRUCTURE ONLY - part of the CPU oracle. Nothing in the engine
// links, loads or calls this file; tests/, bench.py's CPU baseline and
// __graft_entry__.smoke() use it as the checker.
//
// The arithmetic whose result must be bit-identical between the oracle and
// the CUDA engine: bf16 rounding, the Philox4x32-10 counter RNG, the
// uniform -> Gumbel transform, the CFG mix and the temperature divide.
// Compiled with -ffp-contract=off so that no multiply-add is fused: every
// float operation here rounds once, exactly as the engine's __fmul_rn /
// __fadd_rn / __fdiv_rn sequence does.
//
// Reference points (rhymeswithlion/magenta-realtime-mlx-cpp):
//   cfg_combine            src/magenta_realtime_mlx/depthformer/decode.cpp:71-85
//   temperature divide     decode.cpp:143 (logits fp32 / T)
//   categorical sampling   decode.cpp:134,147 (mx::random::categorical =
//                          argmax(logits + Gumbel noise); MLX's threefry
//                          stream is not reproducible here, so the draws come
//                          from Philox instead and parity is defined given
//                          identical draws)

#include <cstdint>
#include <cstring>

#include "oracle.h"

namespace oracle {

float bf16_round(float x) {
  uint32_t u;
  std::memcpy(&u, &x, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) {  // NaN: keep it quiet
    u = (u | 0x00400000u) & 0xffff0000u;
  } else {
    const uint32_t lsb = (u >> 16) & 1u;
    u = (u + 0x7fffu + lsb) & 0xffff0000u;  // round to nearest even
  }
  float r;
  std::memcpy(&r, &u, 4);
  return r;
}

// Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as
// easy as 1, 2, 3", SC'11): 10 rounds of the 4x32 Philox S-box with the
// published multipliers and Weyl key increments.
void philox4x32_10(const uint32_t ctr_in[4], const uint32_t key_in[2], uint32_t out[4]) {
  const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u;
  const uint32_t W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
  uint32_t c0 = ctr_in[0], c1 = ctr_in[1], c2 = ctr_in[2], c3 = ctr_in[3];
  uint32_t k0 = key_in[0], k1 = key_in[1];
  for (int r = 0; r < 10; ++r) {
    const uint64_t p0 = (uint64_t)M0 * c0;
    const uint64_t p1 = (uint64_t)M1 * c2;
    const uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
    const uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
    const uint32_t n0 = hi1 ^ c1 ^ k0;
    const uint32_t n1 = lo1;
    const uint32_t n2 = hi0 ^ c3 ^ k1;
    const uint32_t n3 = lo0;
    c0 = n0; c1 = n1; c2 = n2; c3 = n3;
    k0 += W0;
    k1 += W1;
  }
  out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

// Draw for vocabulary index `idx` of decode step `step` (= frame *
// rvq_depth + level) under `seed`: counter (idx / 4, step, 0, 0), key =
// seed split in two words, word idx % 4. Mapped to the open interval (0, 1)
// as (2 * (x >> 9) + 1) * 2^-24, which is exact in float.
float philox_uniform(uint64_t seed, uint32_t step, uint32_t idx) {
  const uint32_t ctr[4] = {idx >> 2, step, 0u, 0u};
  const uint32_t key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
  uint32_t o[4];
  philox4x32_10(ctr, key, o);
  const uint32_t x = o[idx & 3u];
  return (float)((x >> 9) * 2u + 1u) * (1.0f / 16777216.0f);
}

// Natural log of a positive normal float with basic operations only, so the
// result is the same bit pattern on any IEEE-754 machine:
// x = m * 2^e with m in [sqrt(1/2), sqrt(2)), s = (m - 1) / (m + 1),
// ln m = 2 * atanh(s) = 2 * (s + s^3/3 + s^5/5 + ... + s^13/13) (|s| < 0.1716,
// truncation error < 1e-12), ln x = e * ln 2 + ln m.
float exact_log(float x) {
  uint32_t u;
  std::memcpy(&u, &x, 4);
  int e = (int)((u >> 23) & 0xffu) - 127;
  uint32_t mu = (u & 0x007fffffu) | 0x3f800000u;  // m in [1, 2)
  float m;
  std::memcpy(&m, &mu, 4);
  if (m > 0x1.6a09e6p+0f) {  // sqrt(2) rounded to float: move m to [sqrt(1/2), sqrt(2))
    m = m * 0.5f;
    e = e + 1;
  }
  const float s = (m - 1.0f) / (m + 1.0f);
  const float s2 = s * s;
  // Coefficients 1/13 ... 1/3 rounded to float, written as hex literals so
  // every compiler sees the same bits.
  float p = 0x1.3b13b2p-4f;
  p = p * s2 + 0x1.745d18p-4f;
  p = p * s2 + 0x1.c71c72p-4f;
  p = p * s2 + 0x1.24924ap-3f;
  p = p * s2 + 0x1.99999ap-3f;
  p = p * s2 + 0x1.555556p-2f;
  p = p * s2 + 1.0f;
  const float lnm = 2.0f * (s * p);
  const float ln2_hi = 0x1.62e4p-1f;     // upper 17 bits of ln 2: e * ln2_hi is exact
  const float ln2_lo = 0x1.7f7d1cp-20f;  // ln 2 - ln2_hi, rounded to float
  const float fe = (float)e;
  return (fe * ln2_hi + lnm) + fe * ln2_lo;
}

// Gumbel(0, 1) noise from a uniform draw u in (0, 1): -log(-log(u)).
float gumbel_from_uniform(float u) {
  const float a = -exact_log(u);
  return -exact_log(a);
}

// cfg_combine (decode.cpp:71-85): (1 + w) * cond - w * uncond in fp32,
// each product rounded, then the difference.
float cfg_mix(float cond, float uncond, float w) {
  const float sc = 1.0f + w;
  const float a = sc * cond;
  const float b = w * uncond;
  return a - b;
}

float div_temperature(float x, float t) { return x / t; }

float add_noise(float x, float g) { return x + g; }

}  // namespace oracle
