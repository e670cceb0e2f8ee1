// Counter-based seeded generator for random-init weights and prompts.
// SplitMix64 (Steele, Lea, Flood 2014; constants from Vigna's public-domain
// reference): element i of stream (seed, stream) is the (i+1)-th output of a
// SplitMix64 whose state starts at mix(seed << 32 ^ stream).  Host, device
// and numpy (arc_chain_b200/formats/gen.py) compute identical values, so a
// model generated on the GPU equals the one the CPU oracle generates.
#pragma once
#include <stdint.h>

#if defined(__CUDACC__)
#define RNG_HD __host__ __device__ __forceinline__
#else
#define RNG_HD inline
#endif

namespace arcrng {

constexpr uint64_t GAMMA = 0x9E3779B97F4A7C15ull;

RNG_HD uint64_t fin(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

RNG_HD uint64_t stream_key(uint64_t seed, uint64_t stream) {
  return fin(((seed << 32) ^ stream) + GAMMA);
}

RNG_HD uint64_t at(uint64_t key, uint64_t i) { return fin(key + (i + 1) * GAMMA); }

// int8 weight uniform in [-127, 127]
RNG_HD int8_t weight_i8(uint64_t key, uint64_t i) { return (int8_t)((int)(at(key, i) % 255) - 127); }

}  // namespace arcrng
