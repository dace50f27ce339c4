// Counter-based device draws of the objective's noise (opt-in): Philox4x32-10, the counter-based generator
// of Salmon, Moraes, Dror and Shaw, "Parallel random numbers: as easy as 1, 2, 3" (SC'11), restated from the
// paper: a 128-bit counter (four 32-bit words) is mixed with a 64-bit key by ten rounds of two 32x32->64-bit
// multiplications, the key advancing by the Weyl increments between rounds.
//
// Stream layout of this library: the draw for item i (an event or an anchor) of call number c uses the
// counter (i, stream, c mod 2^32, c / 2^32) and the key (seed mod 2^32, seed / 2^32); stream 0 gives the
// dequantisation jitter u (two uniforms), stream 1 the anchor smoothing noise z (two normals).
//   uniform: (w >> 8) * 2^-24, in [0, 1) with 24 random bits (the fp32 mantissa)
//   normal : Box-Muller on the first two words, r = sqrt(-2 log u1) with u1 = ((w0 >> 8) + 1) * 2^-24 in (0, 1],
//            angle 2 pi u2: (r cos, r sin)
// The reference draws these on the host with torch's CPU generator; the two streams differ, so this path is
// off unless the caller asks for it.
#pragma once
#include "common.cuh"

namespace atlb {

struct Philox4 {
  unsigned x, y, z, w;
};

__host__ __device__ __forceinline__ void mulhilo32(unsigned a, unsigned b, unsigned* hi, unsigned* lo) {
  const unsigned long long p = (unsigned long long)a * (unsigned long long)b;
  *hi = (unsigned)(p >> 32);
  *lo = (unsigned)p;
}

__host__ __device__ __forceinline__ Philox4 philox4x32_10(Philox4 c, unsigned k0, unsigned k1) {
  constexpr unsigned kM0 = 0xD2511F53u, kM1 = 0xCD9E8D57u;  // round multipliers
  constexpr unsigned kW0 = 0x9E3779B9u, kW1 = 0xBB67AE85u;  // key increments (golden ratio, sqrt(3) - 1)
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    unsigned hi0, lo0, hi1, lo1;
    mulhilo32(kM0, c.x, &hi0, &lo0);
    mulhilo32(kM1, c.z, &hi1, &lo1);
    c = Philox4{hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0};
    k0 += kW0;
    k1 += kW1;
  }
  return c;
}

struct RngKey {
  unsigned k0, k1;    // seed words
  unsigned c2, c3;    // call number words
};

inline RngKey make_rng_key(unsigned long long seed, unsigned long long call) {
  return RngKey{(unsigned)seed, (unsigned)(seed >> 32), (unsigned)call, (unsigned)(call >> 32)};
}

// The two uniforms of item i (stream 0).
__device__ __forceinline__ float2 rng_uniform2(const RngKey& K, unsigned long long i) {
  const Philox4 o = philox4x32_10(Philox4{(unsigned)i, (unsigned)(i >> 32) << 1, K.c2, K.c3}, K.k0, K.k1);
  return make_float2((float)(o.x >> 8) * 0x1p-24f, (float)(o.y >> 8) * 0x1p-24f);
}

// The two standard normals of item i (stream 1).
__device__ __forceinline__ float2 rng_normal2(const RngKey& K, unsigned long long i) {
  const Philox4 o = philox4x32_10(Philox4{(unsigned)i, ((unsigned)(i >> 32) << 1) | 1u, K.c2, K.c3}, K.k0, K.k1);
  const float u1 = (float)((o.x >> 8) + 1u) * 0x1p-24f;  // (0, 1]
  const float u2 = (float)(o.y >> 8) * 0x1p-24f;         // [0, 1)
  const float r = sqrtf(-2.f * logf(u1));
  float s, c;
  sincospif(2.f * u2, &s, &c);
  return make_float2(r * c, r * s);
}

}  // namespace atlb
