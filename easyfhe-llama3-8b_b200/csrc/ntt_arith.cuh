// The two butterfly arithmetics of the NTT kernels (and of the butterfly
// rate calibration that serves as their roofline).
#pragma once
#include <cstdint>

#include <cuda_runtime.h>

namespace b2f {

// Integer butterflies: 64-bit words, lazy Shoup products with the twiddle's
// precomputed quotient.
struct IntArith {
  using V = uint64_t;
  using W = ulonglong2;
  uint64_t q, q2;
  __device__ __forceinline__ IntArith(const uint64_t *primes, const double *, int prime)
      : q(primes[prime]), q2(2 * primes[prime]) {}
  static __device__ __forceinline__ W ldtw(const W *tw, int idx) { return __ldg(tw + idx); }
  static __device__ __forceinline__ V from_word(uint64_t v) { return v; }
  static __device__ __forceinline__ uint64_t to_word(V v) { return v; }
  static __device__ __forceinline__ V from_bits(uint64_t v) { return v; }
  static __device__ __forceinline__ uint64_t bits(V v) { return v; }
  static __device__ __forceinline__ W scale(ulonglong2 s) { return s; }
  // y * w mod q in [0, 2q) for any 64-bit y
  __device__ __forceinline__ V mul(V y, W w) const {
    return y * w.x - __umul64hi(y, w.y) * q;
  }
  __device__ __forceinline__ V red2(V a) const { return a >= q2 ? a - q2 : a; }
  __device__ __forceinline__ V red1(V a) const { return a >= q ? a - q : a; }
  __device__ __forceinline__ V add(V a, V b) const { return a + b; }
  // a - b + 2q
  __device__ __forceinline__ V sub2q(V a, V b) const { return a - b + q2; }
};

// Binary64 butterflies for primes below 2^50: residues below 4q < 2^52 are
// exact doubles.  y * w mod q (y < 4q, w < q): h + l = y w exactly (product
// and its FMA error term), qt = rint(h / q) from one FMA against 1/q rounded
// at 2^52, r = (h - qt q) + l exactly; |y w / q - qt| < 1.5, so r lies in
// (-1.5 q, 1.5 q) and r + 2q (r < 0) lands in [0, 2q).  Every operation is
// round-to-nearest without contraction; the results equal the integer ones.
struct FpArith {
  using V = double;
  using W = double;
  static constexpr double kTwo52 = 4503599627370496.0;
  double q, q2, qinv;
  __device__ __forceinline__ FpArith(const uint64_t *primes, const double *qinvs, int prime)
      : q(from_word(primes[prime])), q2(2.0 * from_word(primes[prime])),
        qinv(qinvs[prime]) {}
  static __device__ __forceinline__ W ldtw(const W *tw, int idx) { return __ldg(tw + idx); }
  // exact for v < 2^52: the word as the mantissa of 2^52 + v
  static __device__ __forceinline__ V from_word(uint64_t v) {
    return __dadd_rn(__longlong_as_double((long long)(v | 0x4330000000000000ull)), -kTwo52);
  }
  static __device__ __forceinline__ uint64_t to_word(V v) {
    return (uint64_t)__double_as_longlong(__dadd_rn(v, kTwo52)) & 0x000FFFFFFFFFFFFFull;
  }
  static __device__ __forceinline__ V from_bits(uint64_t v) {
    return __longlong_as_double((long long)v);
  }
  static __device__ __forceinline__ uint64_t bits(V v) {
    return (uint64_t)__double_as_longlong(v);
  }
  static __device__ __forceinline__ W scale(ulonglong2 s) { return from_word(s.x); }
  __device__ __forceinline__ V mul(V y, W w) const {
    const double h = __dmul_rn(y, w);
    const double l = __fma_rn(y, w, -h);
    const double qt = __dadd_rn(__fma_rn(h, qinv, kTwo52), -kTwo52);
    const double r = __dadd_rn(__fma_rn(-qt, q, h), l);
    return r < 0.0 ? __dadd_rn(r, q2) : r;
  }
  __device__ __forceinline__ V red2(V a) const { return a >= q2 ? __dadd_rn(a, -q2) : a; }
  __device__ __forceinline__ V red1(V a) const { return a >= q ? __dadd_rn(a, -q) : a; }
  __device__ __forceinline__ V add(V a, V b) const { return __dadd_rn(a, b); }
  __device__ __forceinline__ V sub2q(V a, V b) const { return __dadd_rn(__dadd_rn(a, -b), q2); }
};

// forward butterfly, values in [0, 4q): (x, y) -> (x + w y, x - w y)
template <class A>
__device__ __forceinline__ void ct_bfly(const A &ar, typename A::V &x, typename A::V &y,
                                        typename A::W w) {
  const typename A::V u = ar.red2(x);
  const typename A::V t = ar.mul(y, w);
  x = ar.add(u, t);
  y = ar.sub2q(u, t);
}

// inverse butterfly, values in [0, 2q): (x, y) -> (x + y, (x - y) w)
template <class A>
__device__ __forceinline__ void gs_bfly(const A &ar, typename A::V &x, typename A::V &y,
                                        typename A::W w) {
  const typename A::V u = ar.red2(ar.add(x, y));
  const typename A::V t = ar.sub2q(x, y);
  x = u;
  y = ar.mul(t, w);
}

}  // namespace b2f
