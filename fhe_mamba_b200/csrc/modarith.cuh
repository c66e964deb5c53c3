// Device-side 64-bit modular arithmetic for RNS limbs (moduli q < 2^62).
//
// Constant multipliers use Shoup's precomputed-quotient multiplication: for a
// constant w < q with companion w' = floor(w * 2^64 / q), and any x < 2^64,
//   r = x*w - umulhi(x, w') * q  (mod 2^64)  lies in [0, 2q).
// Butterflies keep residues "lazy" (Harvey's bounds: [0, 4q) forward,
// [0, 2q) inverse) and reduce fully only at the end of a transform.
// Products of two variables (ciphertext tensor products, key inner products)
// use Barrett reduction of the 128-bit product with mu = floor(2^(2n) / q),
// n = bit length of q.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace fhe {

struct Twiddle {  // 16-byte pair so one 128-bit load fetches both words
  uint64_t w;
  uint64_t wp;
};

// Per-modulus constants, one entry per prime of the context (Q then P).
struct Modulus {
  uint64_t q;
  uint64_t mu;       // floor(2^(2n) / q)
  uint32_t n;        // bit length of q
  uint32_t pad;
  uint64_t r64;      // 2^64 mod q
  uint64_t r64p;     // Shoup companion of r64
  uint64_t mu1;      // floor(2^64 / q), Shoup companion of 1
};

__device__ __forceinline__ uint64_t shoup_lazy(uint64_t x, uint64_t w, uint64_t wp, uint64_t q) {
  return x * w - __umul64hi(x, wp) * q;
}

__device__ __forceinline__ uint64_t csub(uint64_t x, uint64_t m) { return x >= m ? x - m : x; }

__device__ __forceinline__ uint64_t shoup_mul(uint64_t x, uint64_t w, uint64_t wp, uint64_t q) {
  return csub(shoup_lazy(x, w, wp, q), q);
}

__device__ __forceinline__ uint64_t add_mod(uint64_t a, uint64_t b, uint64_t q) {
  return csub(a + b, q);
}

__device__ __forceinline__ uint64_t sub_mod(uint64_t a, uint64_t b, uint64_t q) {
  return a >= b ? a - b : a + q - b;
}

__device__ __forceinline__ uint64_t neg_mod(uint64_t a, uint64_t q) { return a ? q - a : 0; }

// Barrett reduction of a 128-bit value x = (hi, lo) < q^2 (or < 2^(2n)).
__device__ __forceinline__ uint64_t barrett_reduce(uint64_t hi, uint64_t lo, const Modulus& m) {
  const uint32_t s = m.n - 1;
  // x1 = x >> (n-1), fits in 64 bits because x < 2^(2n) and n <= 62.
  const uint64_t x1 = (lo >> s) | (hi << (64 - s));
  const uint64_t thi = __umul64hi(x1, m.mu);
  const uint64_t tlo = x1 * m.mu;
  const uint32_t s2 = m.n + 1;
  const uint64_t qhat = (tlo >> s2) | (thi << (64 - s2));
  uint64_t r = lo - qhat * m.q;  // exact: r < 3q < 2^64
  r = csub(r, m.q);
  return csub(r, m.q);
}

// (hi * 2^64 + lo) mod q for any 128-bit value: two Shoup products by
// constants (2^64 mod q and 1) and two conditional subtractions.
__device__ __forceinline__ uint64_t reduce_u128(uint64_t hi, uint64_t lo, const Modulus& m) {
  const uint64_t a = shoup_lazy(hi, m.r64, m.r64p, m.q);
  const uint64_t b = shoup_lazy(lo, 1, m.mu1, m.q);
  return csub(csub(a + b, 2 * m.q), m.q);
}

__device__ __forceinline__ uint64_t mul_mod(uint64_t a, uint64_t b, const Modulus& m) {
  return barrett_reduce(__umul64hi(a, b), a * b, m);
}

}  // namespace fhe
