// Philox4x32-10 counter-based generator (Salmon, Moraes, Dror, Shaw, SC'11)
// and the Gumbel transform of server/engine.py:88-91.
//
// Counter layout (the CPU checker in oracle/philox.py uses the same one):
//   token noise    (b, l, v): ctr = (v >> 2, b*L + l, off_lo, off_hi & 0x7fffffff), word v & 3
//   position noise p = b*L+l: ctr = (p >> 2, 0xffffffff, off_lo, off_hi | 0x80000000), word p & 3
//   key = (seed_lo, seed_hi)
#pragma once
#include <stdint.h>

namespace yapd {

struct Philox4 {
  uint32_t x, y, z, w;
};

__device__ __forceinline__ Philox4 philox4x32_10(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3,
                                                 uint32_t k0, uint32_t k1) {
  const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u;
  const uint32_t W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(M0, c0), lo0 = M0 * c0;
    const uint32_t hi1 = __umulhi(M1, c2), lo1 = M1 * c2;
    const uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
    c0 = n0;
    c1 = lo1;
    c2 = n2;
    c3 = lo0;
    k0 += W0;
    k1 += W1;
  }
  return {c0, c1, c2, c3};
}

__device__ __forceinline__ uint32_t philox_word(const Philox4& r, uint32_t which) {
  return which == 0 ? r.x : which == 1 ? r.y : which == 2 ? r.z : r.w;
}

// Uniform in [0, 1) with 24 random bits, exactly representable in fp32.
__device__ __forceinline__ float uniform_from_word(uint32_t w) {
  return __uint2float_rn(w >> 8) * 5.9604644775390625e-08f;  // 2^-24
}

// -log(max(-log(max(u, 1e-20)), 1e-20))
__device__ __forceinline__ float gumbel_from_uniform(float u) {
  u = fmaxf(u, 1e-20f);
  const float t = fmaxf(-logf(u), 1e-20f);
  return -logf(t);
}

__device__ __forceinline__ float philox_token_gumbel(uint64_t seed, uint64_t offset, uint32_t pos,
                                                     uint32_t v) {
  const Philox4 r = philox4x32_10(v >> 2, pos, (uint32_t)offset,
                                  (uint32_t)(offset >> 32) & 0x7fffffffu, (uint32_t)seed,
                                  (uint32_t)(seed >> 32));
  return gumbel_from_uniform(uniform_from_word(philox_word(r, v & 3u)));
}

__device__ __forceinline__ float philox_position_gumbel(uint64_t seed, uint64_t offset, uint32_t p) {
  const Philox4 r = philox4x32_10(p >> 2, 0xffffffffu, (uint32_t)offset,
                                  ((uint32_t)(offset >> 32) & 0x7fffffffu) | 0x80000000u,
                                  (uint32_t)seed, (uint32_t)(seed >> 32));
  return gumbel_from_uniform(uniform_from_word(philox_word(r, p & 3u)));
}

}  // namespace yapd
