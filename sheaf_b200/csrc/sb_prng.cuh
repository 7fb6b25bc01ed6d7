// Device side of the reference's counter-based PRNG (sheaf/src/core/prng.rs):
// Threefry2x32 with 20 rounds over keys held as four 16-bit f32 limbs.
//   random-split key n: child i = threefry(key, [i, 1])        (prng.rs:81-84)
//   sampling bits of flat element i = threefry(key, [i, 0])    (prng.rs:86-89)
//   uniform = (bits >> 8) * 2^-24                              (prng.rs:91-97)
//   randint = clamp(floor(u * (high - low)) + low, low, high - 1) in f32 (prng.rs:124-134)
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

namespace sb {

__device__ __forceinline__ uint32_t prng_rotl32(uint32_t x, int r) { return (x << r) | (x >> (32 - r)); }

// Threefry2x32-20 (prng.rs:57-79).
__device__ inline void threefry2x32(uint32_t k0, uint32_t k1, uint32_t c0, uint32_t c1, uint32_t& x0, uint32_t& x1) {
  const uint32_t ks[3] = {k0, k1, 0x1BD11BDAu ^ k0 ^ k1};
  const int rot[8] = {13, 15, 26, 6, 17, 29, 16, 24};
  x0 = c0 + ks[0];
  x1 = c1 + ks[1];
#pragma unroll
  for (int r = 0; r < 20; ++r) {
    x0 += x1;
    x1 = x0 ^ prng_rotl32(x1, rot[r & 7]);
    if ((r & 3) == 3) {
      const uint32_t inj = static_cast<uint32_t>((r + 1) / 4);
      x0 += ks[inj % 3];
      x1 += ks[(inj + 1) % 3] + inj;
    }
  }
}

__device__ __forceinline__ void key_decode(const float* limbs, uint32_t& w0, uint32_t& w1) {
  w0 = (static_cast<uint32_t>(limbs[0]) | (static_cast<uint32_t>(limbs[1]) << 16));
  w1 = (static_cast<uint32_t>(limbs[2]) | (static_cast<uint32_t>(limbs[3]) << 16));
}

__device__ __forceinline__ void key_encode(uint32_t w0, uint32_t w1, float* limbs) {
  limbs[0] = static_cast<float>(w0 & 0xFFFFu);
  limbs[1] = static_cast<float>(w0 >> 16);
  limbs[2] = static_cast<float>(w1 & 0xFFFFu);
  limbs[3] = static_cast<float>(w1 >> 16);
}

__device__ __forceinline__ float uniform_from_bits(uint32_t bits) {
  return static_cast<float>(bits >> 8) * (1.0f / 16777216.0f);
}

}  // namespace sb
