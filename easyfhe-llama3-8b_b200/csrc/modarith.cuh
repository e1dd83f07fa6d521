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
  uint64_t mu;    // floor(2^(64+k) / q), k = bitlen(q) - 1 (reduce_bk)
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
// acc += a b.  On the GPU the four 32 x 32 partial products go through one
// PTX carry chain, so the low and high halves share them (a separate mul.lo
// and mul.hi repeat partial products; measured 1.4x faster on B200).
__host__ __device__ __forceinline__ void mac128(U128 &acc, uint64_t a,
                                                uint64_t b) {
#ifdef __CUDA_ARCH__
  const uint32_t a0 = (uint32_t)a, a1 = (uint32_t)(a >> 32);
  const uint32_t b0 = (uint32_t)b, b1 = (uint32_t)(b >> 32);
  uint32_t r0, r1, r2, r3;
  asm("{\n\t"
      "mad.lo.cc.u32 %0, %4, %6, %8;\n\t"    // r0 = lo(a0 b0) + acc
      "madc.hi.cc.u32 %1, %4, %6, %9;\n\t"   // r1 = hi(a0 b0) + acc + c
      "madc.lo.cc.u32 %2, %5, %7, %10;\n\t"  // r2 = lo(a1 b1) + acc + c
      "madc.hi.u32 %3, %5, %7, %11;\n\t"     // r3 = hi(a1 b1) + acc + c
      "mad.lo.cc.u32 %1, %4, %7, %1;\n\t"    // + a0 b1 << 32
      "madc.hi.cc.u32 %2, %4, %7, %2;\n\t"
      "addc.u32 %3, %3, 0;\n\t"
      "mad.lo.cc.u32 %1, %5, %6, %1;\n\t"    // + a1 b0 << 32
      "madc.hi.cc.u32 %2, %5, %6, %2;\n\t"
      "addc.u32 %3, %3, 0;\n\t"
      "}"
      : "=&r"(r0), "=&r"(r1), "=&r"(r2), "=&r"(r3)
      : "r"(a0), "r"(a1), "r"(b0), "r"(b1), "r"((uint32_t)acc.lo),
        "r"((uint32_t)(acc.lo >> 32)), "r"((uint32_t)acc.hi),
        "r"((uint32_t)(acc.hi >> 32)));
  acc.lo = ((uint64_t)r1 << 32) | r0;
  acc.hi = ((uint64_t)r3 << 32) | r2;
#else
  uint64_t lo = a * b, hi = mulhi64(a, b);
  uint64_t s = acc.lo + lo;
  acc.hi += hi + (s < lo);
  acc.lo = s;
#endif
}
__host__ __device__ __forceinline__ U128 mul128(uint64_t a, uint64_t b) {
  U128 r = {0, 0};
  mac128(r, a, b);
  return r;
}

// (hi*2^64 + lo) mod q.  The quotient estimate floor(s * m / 2^128) with
// m = floor(2^128/q) is exact in its integer parts and undershoots floor(s/q)
// by at most one, so one conditional subtraction finishes the reduction.
__host__ __device__ __forceinline__ uint64_t reduce128(uint64_t hi, uint64_t lo,
                                                       const Mod &M) {
  const uint64_t c0 = mulhi64(lo, M.m_lo);
  const U128 a = mul128(hi, M.m_lo), b = mul128(lo, M.m_hi);
  const uint64_t s1 = a.lo + b.lo;
  uint64_t carry = s1 < a.lo;
  const uint64_t s2 = s1 + c0;
  carry += s2 < s1;
  const uint64_t qe = hi * M.m_hi + a.hi + b.hi + carry;
  const uint64_t r = lo - qe * M.q;
  return csub(r, M.q);
}
// (hi*2^64 + lo) mod q for a value s below 2^(64+k), k = bitlen(q) - 1 (a
// sum of a few products of residues: terms * (q-1)^2 < 2^(64+k), checked by
// the caller).  Barrett with a one-word quotient estimate:
// qe = floor(floor(s / 2^k) * mu / 2^64), mu = floor(2^(64+k) / q), never
// above floor(s/q) and at most 2 below it, so s - qe q < 3q < 2^64 comes from
// the low words and two conditional subtractions finish it.
__host__ __device__ __forceinline__ uint64_t reduce_bk(uint64_t hi, uint64_t lo,
                                                       const Mod &M) {
#ifdef __CUDA_ARCH__
  const int k = 63 - __clzll((long long)M.q);
#else
  const int k = 63 - __builtin_clzll(M.q);
#endif
  const uint64_t x = (hi << (64 - k)) | (lo >> k);
  const uint64_t r = lo - mulhi64(x, M.mu) * M.q;
  return csub(csub(r, 2 * M.q), M.q);
}
__host__ __device__ __forceinline__ uint64_t mul_mod(uint64_t a, uint64_t b,
                                                     const Mod &M) {
  const U128 p = mul128(a, b);
  return reduce128(p.hi, p.lo, M);
}

}  // namespace b2f
