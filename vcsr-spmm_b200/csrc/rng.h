// rng.h — counter-based random numbers shared by host and device code, so a
// generator gives the same bits on either side.
//
// vmix64 is the SplitMix64 output function (Steele, Lea & Flood, "Fast
// splittable pseudorandom number generators", OOPSLA 2014): add the golden
// gamma, then two xor-shift-multiply rounds.  A stream key is the mix of
// (seed, stream id); element i of the stream is vmix64(key + i).
#pragma once
#include <cstdint>

#if defined(__CUDACC__)
#define VCSR_HD __host__ __device__ __forceinline__
#else
#define VCSR_HD inline
#endif

namespace vcsr {

VCSR_HD uint64_t vmix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

VCSR_HD uint64_t stream_key(uint64_t seed, uint64_t stream) {
  return vmix64(seed * 0xD1B54A32D192ED03ull ^ vmix64(stream));
}

VCSR_HD uint64_t rnd(uint64_t key, uint64_t i) { return vmix64(key + i); }

// 24-bit uniform in [0, 1): exact in float.
VCSR_HD float u01f(uint64_t x) {
  return (float)(uint32_t)(x >> 40) * (1.0f / 16777216.0f);
}
// 53-bit uniform in [0, 1).
VCSR_HD double u01d(uint64_t x) {
  return (double)(x >> 11) * (1.0 / 9007199254740992.0);
}
// Uniform integer in [0, n) by multiply-shift of the high 32 bits.
VCSR_HD uint32_t below(uint64_t x, uint32_t n) {
  return (uint32_t)(((x >> 32) * (uint64_t)n) >> 32);
}
// lo + (hi - lo) * u, u a 24-bit uniform; exact for lo=-1,hi=1 and lo=0,hi=1.
VCSR_HD float uniform_f(uint64_t x, float lo, float hi) {
  return lo + (hi - lo) * u01f(x);
}

}  // namespace vcsr
