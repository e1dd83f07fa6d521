// Modular arithmetic on 64-bit words for RNS primes q < 2^61.
//
// Three reductions are used, each where it is cheapest:
//  * Shoup (precomputed quotient) for products with a constant w: one
//    mul.hi plus two mul.lo, result in [0, 2q) for any 64-bit input
//    (Harvey 2014, "Faster arithmetic for number-theoretic transforms").
//  * Barrett on a 128-bit accumulator for data x data products: sums of up
//    to 2^6 products stay below 2^128 and are reduced once.
//  * conditional subtraction for additions kept lazily in [0, 2q) / [0, 4q).
#pragma once
#include <cstdint>

namespace b2f {

struct Mod {
  uint64_t q;     // the prime
  uint64_t m_lo;  // floor(2^128 / q), low word
  uint64_t m_hi;  // floor(2^128 / q), high word
  uint64_t pad;
};

__host__ __device__ __forceinline__ uint64_t mulhi64(uint64_t a, uint64_t b) {
#ifdef __CUDA_ARCH__
  return __umul64hi(a, b);
#else
  return (uint64_t)(((unsigned __int128)a * b) >> 64);
#endif
}

// x * w mod q in [0, 2q); ws = floor(w * 2^64 / q), w < q < 2^63.
__host__ __device__ __forceinline__ uint64_t shoup_lazy(uint64_t x, uint64_t w,
                                                         uint64_t ws,
                                                         uint64_t q) {
  return x * w - mulhi64(x, ws) * q;
}
__host__ __device__ __forceinline__ uint64_t shoup(uint64_t x, uint64_t w,
                                                   uint64_t ws, uint64_t q) {
  uint64_t r = shoup_lazy(x, w, ws, q);
  return r >= q ? r - q : r;
}
__host__ __device__ __forceinline__ uint64_t csub(uint64_t x, uint64_t q) {
  return x >= q ? x - q : x;
}
__host__ __device__ __forceinline__ uint64_t add_mod(uint64_t a, uint64_t b,
                                                     uint64_t q) {
  return csub(a + b, q);
}
__host__ __device__ __forceinline__ uint64_t sub_mod(uint64_t a, uint64_t b,
                                                     uint64_t q) {
  return a >= b ? a - b : a + q - b;
}

// 128-bit accumulator (hi, lo).
struct U128 {
  uint64_t lo, hi;
};
__host__ __device__ __forceinline__ void mac128(U128 &acc, uint64_t a,
                                                uint64_t b) {
  uint64_t lo = a * b, hi = mulhi64(a, b);
  uint64_t s = acc.lo + lo;
  acc.hi += hi + (s < lo);
  acc.lo = s;
}

// (hi*2^64 + lo) mod q.  The quotient estimate floor(s * m / 2^128) with
// m = floor(2^128/q) is exact in its integer parts and undershoots floor(s/q)
// by at most one, so one conditional subtraction finishes the reduction.
__host__ __device__ __forceinline__ uint64_t reduce128(uint64_t hi, uint64_t lo,
                                                       const Mod &M) {
  uint64_t c0 = mulhi64(lo, M.m_lo);
  uint64_t a_lo = hi * M.m_lo, a_hi = mulhi64(hi, M.m_lo);
  uint64_t b_lo = lo * M.m_hi, b_hi = mulhi64(lo, M.m_hi);
  uint64_t s1 = a_lo + b_lo;
  uint64_t carry = s1 < a_lo;
  uint64_t s2 = s1 + c0;
  carry += s2 < s1;
  uint64_t qe = hi * M.m_hi + a_hi + b_hi + carry;
  uint64_t r = lo - qe * M.q;
  return csub(r, M.q);
}
__host__ __device__ __forceinline__ uint64_t mul_mod(uint64_t a, uint64_t b,
                                                     const Mod &M) {
  return reduce128(mulhi64(a, b), a * b, M);
}

}  // namespace b2f
