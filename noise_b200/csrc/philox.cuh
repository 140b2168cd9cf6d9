// Counter-based draws. Every perturbation value in this library is a pure function of
// (seed, step, direction, tensor, vector, element), computed by Philox4x32-10 (Salmon, Moraes,
// Dror, Shaw: "Parallel random numbers: as easy as 1, 2, 3", SC'11) followed by the Box-Muller
// transform. Any kernel can therefore regenerate any draw without storing it, and the host-side
// oracle (oracle/philox.py) reproduces the same integers bit for bit.
//
// Stream layout (one Philox block = 4 x u32 = 4 Gaussians):
//   key     = (seed, step)
//   counter = (element / 4, (tensor << 1) | vector, direction, domain)
//   lane    = element % 4
// `vector` is 0 for the row factor a (length = rows of the parameter) and 1 for the column factor b
// (length = columns); the 1-D mixing scalars use vector 0. Lanes (0,1) and (2,3) of a block are
// Box-Muller pairs: z0 = r cos(2 pi u1), z1 = r sin(2 pi u1) with r = sqrt(-2 ln u0).
#pragma once

#include <stdint.h>

#ifdef __CUDACC__
#define NOISE_HD __host__ __device__ __forceinline__
#else
#define NOISE_HD inline
#endif

namespace noise {

enum : uint32_t {
  kDomainLowRank = 0x4C52u,   // EGGROLL rank-1 factors and mixing-scalar eps
  kDomainDirect = 0x4452u,    // direct (activation-site) draws
};

struct PhiloxKey {
  uint32_t k0, k1;
};

NOISE_HD void philox_mulhilo(uint32_t a, uint32_t b, uint32_t& hi, uint32_t& lo) {
#ifdef __CUDA_ARCH__
  lo = a * b;
  hi = __umulhi(a, b);
#else
  const uint64_t p = (uint64_t)a * (uint64_t)b;
  lo = (uint32_t)p;
  hi = (uint32_t)(p >> 32);
#endif
}

// Philox4x32 with 10 rounds; the key is bumped by the Weyl constants between rounds.
NOISE_HD void philox4x32_10(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3, uint32_t k0, uint32_t k1,
                            uint32_t out[4]) {
  const uint32_t kMul0 = 0xD2511F53u, kMul1 = 0xCD9E8D57u;
  const uint32_t kWeyl0 = 0x9E3779B9u, kWeyl1 = 0xBB67AE85u;
#ifdef __CUDA_ARCH__
#pragma unroll
#endif
  for (int r = 0; r < 10; ++r) {
    uint32_t hi0, lo0, hi1, lo1;
    philox_mulhilo(kMul0, c0, hi0, lo0);
    philox_mulhilo(kMul1, c2, hi1, lo1);
    const uint32_t n0 = hi1 ^ c1 ^ k0;
    const uint32_t n2 = hi0 ^ c3 ^ k1;
    c0 = n0;
    c1 = lo1;
    c2 = n2;
    c3 = lo0;
    k0 += kWeyl0;
    k1 += kWeyl1;
  }
  out[0] = c0;
  out[1] = c1;
  out[2] = c2;
  out[3] = c3;
}

// Uniform in the open interval (0, 1) from the top 24 bits: ((x >> 8) + 0.5) * 2^-24, exact in fp32.
NOISE_HD float u32_to_open_unit(uint32_t x) { return ((float)(x >> 8) + 0.5f) * 5.9604644775390625e-08f; }

#ifdef __CUDACC__
// Box-Muller on one pair. Written with explicit round-to-nearest intrinsics so every kernel that
// inlines it produces the same bits, whatever contraction the surrounding code allows.
__device__ __forceinline__ void box_muller(uint32_t x0, uint32_t x1, float& z0, float& z1) {
  const float u0 = u32_to_open_unit(x0);
  const float u1 = u32_to_open_unit(x1);
  const float r = sqrtf(__fmul_rn(-2.0f, logf(u0)));
  float s, c;
  sincospif(__fmul_rn(2.0f, u1), &s, &c);
  z0 = __fmul_rn(r, c);
  z1 = __fmul_rn(r, s);
}

// Four Gaussians of block `blk` of the (tensor, vector, direction) stream.
__device__ __forceinline__ float4 gauss4(PhiloxKey key, uint32_t blk, uint32_t tensor, uint32_t vec,
                                         uint32_t direction, uint32_t domain = kDomainLowRank) {
  uint32_t x[4];
  philox4x32_10(blk, (tensor << 1) | vec, direction, domain, key.k0, key.k1, x);
  float4 g;
  box_muller(x[0], x[1], g.x, g.y);
  box_muller(x[2], x[3], g.z, g.w);
  return g;
}

// One Gaussian, element `i` of the stream (costs a whole Philox block; use gauss4 for runs).
__device__ __forceinline__ float gauss1(PhiloxKey key, uint32_t i, uint32_t tensor, uint32_t vec,
                                        uint32_t direction, uint32_t domain = kDomainLowRank) {
  const float4 g = gauss4(key, i >> 2, tensor, vec, direction, domain);
  const uint32_t l = i & 3;
  return l == 0 ? g.x : l == 1 ? g.y : l == 2 ? g.z : g.w;
}
#endif

}  // namespace noise
