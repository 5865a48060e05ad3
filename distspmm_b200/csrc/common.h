// common.h — definitions shared by host C++ and device CUDA code.
#pragma once
#include <stdint.h>

#if defined(__CUDACC__)
#define DSP_HD __host__ __device__ __forceinline__
#else
#define DSP_HD inline
#endif

namespace dsp {

// SplitMix64 finaliser (Steele, Lea, Flood, "Fast splittable pseudorandom number
// generators", OOPSLA 2014): a bijective 64-bit mix used as a counter-based generator.
DSP_HD uint64_t mix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

// 64 random bits for the pair (a, b) under `seed`.
DSP_HD uint64_t hash3(uint64_t seed, uint64_t a, uint64_t b) {
  return mix64(mix64(seed ^ mix64(a)) ^ (b * 0xD6E8FEB86659FD93ull));
}

// Uniform [0,1) with 24 bits: k * 2^-24, exact in fp32.
DSP_HD float u01_24(uint64_t bits) { return (float)(bits >> 40) * (1.0f / 16777216.0f); }

// Synthetic dense B element: U(-1,1) = 2u - 1, exact in fp32 (|2k - 2^24| <= 2^24).
DSP_HD float dense_value(uint64_t seed, int64_t row, int64_t col) {
  return 2.0f * u01_24(hash3(seed, (uint64_t)row, (uint64_t)col)) - 1.0f;
}

}  // namespace dsp
