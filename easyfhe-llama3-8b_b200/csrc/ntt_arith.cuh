// The two butterfly arithmetics of the NTT kernels (and of the butterfly
// rate calibration that serves as their roofline).  Each policy provides the
// forward (Cooley-Tukey) and inverse (Gentleman-Sande) butterflies on its own
// residue representation, conversion from and to fully reduced 64-bit words,
// and the final reduction; the kernels are written against these alone.
#pragma once
#include <cstdint>

#include <cuda_runtime.h>

namespace b2f {

// Integer butterflies: 64-bit words, Harvey's lazy reduction with Shoup
// products (the twiddle's precomputed quotient): forward values in [0, 4q),
// inverse values in [0, 2q).
struct IntArith {
  using V = uint64_t;
  using W = ulonglong2;
  static constexpr bool kFoldScale = false;  // w s would need its Shoup quotient
  uint64_t q, q2;
  __device__ __forceinline__ IntArith(const uint64_t *primes, const double *, int prime)
      : q(primes[prime]), q2(2 * primes[prime]) {}
  static __device__ __forceinline__ W ldtw(const W *tw, int idx) { return __ldg(tw + idx); }
  // four consecutive twiddles from a 64-byte aligned entry: two 32-byte loads
  static __device__ __forceinline__ void ldtw4(const W *tw, W (&w)[4]) {
#pragma unroll
    for (int h = 0; h < 2; ++h)
      asm("ld.global.nc.v4.u64 {%0, %1, %2, %3}, [%4];"
          : "=l"(w[2 * h].x), "=l"(w[2 * h].y), "=l"(w[2 * h + 1].x), "=l"(w[2 * h + 1].y)
          : "l"(tw + 2 * h));
  }
  static __device__ __forceinline__ void ldtw2(const W *tw, W (&w)[2]) {
    asm("ld.global.nc.v4.u64 {%0, %1, %2, %3}, [%4];"
        : "=l"(w[0].x), "=l"(w[0].y), "=l"(w[1].x), "=l"(w[1].y)
        : "l"(tw));
  }
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
  // (x, y) -> (x + w y, x - w y)
  __device__ __forceinline__ void ct(V &x, V &y, W w) const {
    const V u = red2(x), t = mul(y, w);
    x = u + t;
    y = u - t + q2;
  }
  // (x, y) -> (x + y, (x - y) w), split for lanes that own one output each
  __device__ __forceinline__ V gs_sum(V x, V y) const { return red2(x + y); }
  __device__ __forceinline__ V gs_diff(V x, V y, W w) const { return mul(x - y + q2, w); }
  __device__ __forceinline__ void gs(V &x, V &y, W w) const {
    const V u = gs_sum(x, y);
    y = gs_diff(x, y, w);
    x = u;
  }
  // a forward value to [0, q)
  __device__ __forceinline__ V full(V v) const { return red1(red2(v)); }
  // an inverse value times the output scale, in [0, q)
  __device__ __forceinline__ V scale_out(V v, W s) const { return red1(mul(v, s)); }
};

// Binary64 butterflies for primes below 2^50, on signed residues held as
// exact doubles (forward values within 1.5q + q/2^40 in magnitude, inverse
// values within q).  Every operation rounds to nearest without contraction.
//   red(x):    k = rint(x / q) from one FMA against 1/q rounded at 1.5 2^52
//              (integer ulp for |v| < 2^51), r = x - k q exactly: |r| <= q/2.
//   mul(y, w): h + l = y w exactly (product and its FMA error term), k =
//              rint(h / q), r = (h - k q) + l exactly; for |y| <= 2q, w < q,
//              |y w / q - k| <= 1 so |r| <= q.
// Forward: (x, y) -> (red(x) + mul(y, w), red(x) - mul(y, w)) keeps |.| <=
// 1.5q; inverse: (x, y) -> (red(x + y), mul(x - y, w)) keeps |.| <= q.  The
// residues equal the integer path's after the final reduction.
struct FpArith {
  using V = double;
  using W = double;
  static constexpr double kTwo52 = 4503599627370496.0;
  static constexpr double kMagic = 6755399441055744.0;  // 1.5 * 2^52
  static constexpr bool kFoldScale = true;
  double q, qinv;
  __device__ __forceinline__ FpArith(const uint64_t *primes, const double *qinvs, int prime)
      : q(from_word(primes[prime])), qinv(qinvs[prime]) {}
  static __device__ __forceinline__ W ldtw(const W *tw, int idx) { return __ldg(tw + idx); }
  // four (two) consecutive twiddles from a 32-byte (16-byte) aligned entry
  static __device__ __forceinline__ void ldtw4(const W *tw, W (&w)[4]) {
    asm("ld.global.nc.v4.f64 {%0, %1, %2, %3}, [%4];"
        : "=d"(w[0]), "=d"(w[1]), "=d"(w[2]), "=d"(w[3])
        : "l"(tw));
  }
  static __device__ __forceinline__ void ldtw2(const W *tw, W (&w)[2]) {
    const double2 v = __ldg(reinterpret_cast<const double2 *>(tw));
    w[0] = v.x;
    w[1] = v.y;
  }
  // exact for 0 <= v < 2^52: the word as the mantissa of 2^52 + v
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
  __device__ __forceinline__ V red(V x) const {
    const double k = __dadd_rn(__fma_rn(x, qinv, kMagic), -kMagic);
    return __fma_rn(-k, q, x);
  }
  __device__ __forceinline__ V mul(V y, W w) const {
    const double h = __dmul_rn(y, w);
    const double l = __fma_rn(y, w, -h);
    const double k = __dadd_rn(__fma_rn(h, qinv, kMagic), -kMagic);
    return __dadd_rn(__fma_rn(-k, q, h), l);
  }
  __device__ __forceinline__ void ct(V &x, V &y, W w) const {
    const V u = red(x), t = mul(y, w);
    x = __dadd_rn(u, t);
    y = __dadd_rn(u, -t);
  }
  __device__ __forceinline__ V gs_sum(V x, V y) const { return red(__dadd_rn(x, y)); }
  __device__ __forceinline__ V gs_diff(V x, V y, W w) const {
    return mul(__dadd_rn(x, -y), w);
  }
  __device__ __forceinline__ void gs(V &x, V &y, W w) const {
    const V u = gs_sum(x, y);
    y = gs_diff(x, y, w);
    x = u;
  }
  __device__ __forceinline__ V full(V v) const {
    const V r = red(v);
    return r < 0.0 ? __dadd_rn(r, q) : r;
  }
  __device__ __forceinline__ V scale_out(V v, W s) const { return full(mul(v, s)); }
  // w s mod q in [0, q), and the last inverse butterfly with the output scale
  // folded in: ((x + y) s, (x - y) ws), fully reduced (|x +- y| <= 2q)
  __device__ __forceinline__ W fold(W w, W s) const { return full(mul(w, s)); }
  __device__ __forceinline__ void gs_scaled(V &x, V &y, W s, W ws) const {
    const V u = full(mul(__dadd_rn(x, y), s));
    y = full(mul(__dadd_rn(x, -y), ws));
    x = u;
  }
};

template <class A>
__device__ __forceinline__ void ct_bfly(const A &ar, typename A::V &x, typename A::V &y,
                                        typename A::W w) {
  ar.ct(x, y, w);
}

template <class A>
__device__ __forceinline__ void gs_bfly(const A &ar, typename A::V &x, typename A::V &y,
                                        typename A::W w) {
  ar.gs(x, y, w);
}

}  // namespace b2f
