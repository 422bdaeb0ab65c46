// Counter-based random numbers for the synthetic tensor generators.
//
// Every draw is a pure function of (seed, stream, counter), so a tensor is
// defined independently of thread count or implementation: the C++ generator,
// a numpy restatement and a CUDA kernel all produce the same bits.
#pragma once
#include <cmath>
#include <cstdint>

namespace cptc {

// splitmix64 finaliser (Steele, Lea, Flood 2014).
static inline uint64_t mix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

static inline uint64_t rng_u64(uint64_t seed, uint64_t stream, uint64_t ctr) {
  return mix64(mix64(seed * 0xD1B54A32D192ED03ull + stream) ^ ctr);
}

// Uniform double in [0, 1) with 53 random bits.
static inline double rng_unit(uint64_t seed, uint64_t stream, uint64_t ctr) {
  return (double)(rng_u64(seed, stream, ctr) >> 11) * 0x1.0p-53;
}

// Uniform integer in [0, n) by 128-bit multiply-high (Lemire); bias < n/2^64.
static inline uint64_t rng_below(uint64_t seed, uint64_t stream, uint64_t ctr,
                                 uint64_t n) {
  const unsigned __int128 p =
      (unsigned __int128)rng_u64(seed, stream, ctr) * (unsigned __int128)n;
  return (uint64_t)(p >> 64);
}

// Standard normal by the Box-Muller transform on two counter draws.
static inline double rng_normal(uint64_t seed, uint64_t stream, uint64_t ctr) {
  const double u1 = 1.0 - rng_unit(seed, stream, 2 * ctr);  // (0, 1]
  const double u2 = rng_unit(seed, stream, 2 * ctr + 1);
  return std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2);
}

// Poisson(lambda) by inversion of the CDF on one uniform (small lambda only).
static inline uint32_t rng_poisson(uint64_t seed, uint64_t stream, uint64_t ctr,
                                   double lambda) {
  const double u = rng_unit(seed, stream, ctr);
  double p = std::exp(-lambda), cdf = p;
  uint32_t k = 0;
  while (u >= cdf && k < 1000) {
    ++k;
    p *= lambda / (double)k;
    cdf += p;
  }
  return k;
}

}  // namespace cptc
