// Per-item key switching descriptors shared by the key-switch kernels and the
// NTT whose epilogue finishes a ModDown, and the evaluation-slot permutation
// of an automorphism.
#pragma once
#include <cstdint>

#include "b2f_internal.h"

namespace b2f {

// Per-item key pointers and galois elements of one launch, passed by value.
// With shared != 0 every item uses entry 0 (a batch sharing one key); hoisted
// rotations of one ciphertext use one entry per rotation.
constexpr int kMaxItems = 64;
// In per-item mode item i is rotation i % per of ciphertext i / per (the
// ciphertext indexes c1, ext and c0; out_ct_stride and pos[] place the result).
struct ItemKeys {
  const uint64_t *key[kMaxItems];
  uint32_t g[kMaxItems];
  int16_t pos[kMaxItems];  // output slot of rotation r within its ciphertext
  int shared;
  int per = 1;             // rotations per ciphertext (per-item mode)
  long long out_ct_stride; // words between ciphertexts' outputs (per-item mode)
  __host__ __device__ int at(int i) const { return shared ? 0 : i % per; }
  __host__ __device__ int ct(int i) const { return shared ? i : i / per; }
  __host__ __device__ long long out(int i, long long stride) const {
    return shared ? (long long)i * stride
                  : ct(i) * out_ct_stride + (long long)pos[i % per] * stride;
  }
};

__device__ __forceinline__ uint32_t brv16(uint32_t x) { return __brev(x) >> 16; }

// source evaluation index of output k under X -> X^g (g odd, < 2N)
__device__ __forceinline__ uint32_t auto_src(uint32_t k, uint32_t g) {
  uint32_t e = 2 * brv16(k) + 1;
  uint32_t e2 = (e * g) & (2 * kN - 1);  // modulo 2^17: the low word suffices
  return brv16((e2 - 1) >> 1);
}

// inverse of an odd g modulo 2N (Newton iteration on the 2-adic inverse)
__host__ __device__ __forceinline__ uint32_t galois_inverse(uint32_t g) {
  uint32_t x = g;  // correct to 3 bits
#pragma unroll
  for (int i = 0; i < 4; ++i) x *= 2u - g * x;  // 6, 12, 24, 48 bits
  return x & (2u * kN - 1u);
}

}  // namespace b2f
