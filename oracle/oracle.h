// TEST INFRASTRUCTURE ONLY - internal header of the CPU oracle (see
// depthformer_oracle.cpp). Nothing in the engine includes this file.
#pragma once

#include <cstdint>

namespace oracle {

// Exact-arithmetic helpers (oracle_exact.cpp, built with -ffp-contract=off).
float bf16_round(float x);
void philox4x32_10(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]);
float philox_uniform(uint64_t seed, uint32_t step, uint32_t idx);
float exact_log(float x);
float gumbel_from_uniform(float u);
float cfg_mix(float cond, float uncond, float w);
float div_temperature(float x, float t);
float add_noise(float x, float g);

}  // namespace oracle
