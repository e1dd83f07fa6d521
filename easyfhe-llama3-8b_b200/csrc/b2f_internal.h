// Internal declarations shared by the libb200fhe translation units.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/b200fhe.h"
#include "modarith.cuh"

namespace b2f {

constexpr int kLogN = 16;
constexpr int kN = 1 << kLogN;

void set_error(const char *fmt, ...);
int cuda_status(cudaError_t e, const char *what);

#define B2F_CHECK_ARG(cond, ...)          \
  do {                                    \
    if (!(cond)) {                        \
      ::b2f::set_error(__VA_ARGS__);      \
      return B2F_ERR_ARG;                 \
    }                                     \
  } while (0)
#define B2F_CUDA(call)                                        \
  do {                                                        \
    cudaError_t _e = (call);                                  \
    if (_e != cudaSuccess) return ::b2f::cuda_status(_e, #call); \
  } while (0)
#define B2F_LAUNCHED(what)                                        \
  do {                                                            \
    cudaError_t _e = cudaGetLastError();                          \
    if (_e != cudaSuccess) return ::b2f::cuda_status(_e, what);   \
  } while (0)

// One NTT job: the limb at in_off of an input item is transformed modulo
// prime `prime` into the limb at out_off of the output item (in place when
// the two coincide), scaled (inverse only) by the Shoup pair scale[scale_idx].
struct LimbJob {
  uint32_t in_off;   // input limb offset from the item base, units of N
  uint32_t out_off;  // output limb offset from the item base, units of N
  uint16_t prime;
  uint16_t scale_idx;
  uint32_t pad;
};

// Constants of the hybrid key switch at one level (l Q-limbs).
struct LevelTables {
  int l = 0, beta = 0;
  // per Q limb i < l: N^-1 * [Qhat_{j(i),i}^-1] mod q_i (Shoup pair)
  ulonglong2 *modup_scale = nullptr;
  // [beta][l+K][alpha]: [Qhat_{j,i}] mod p_t (Shoup pair w.r.t. p_t)
  ulonglong2 *modup_conv = nullptr;
  // rescale: for i < l-1, [q_{l-1}^-1] mod q_i and [q_{l-1}] mod q_i
  ulonglong2 *rescale_inv = nullptr;
  uint64_t *rescale_qlast = nullptr;
};

}  // namespace b2f

struct b2f_context {
  int device = 0;
  int log_n = b2f::kLogN;
  int n = b2f::kN;
  int L = 0, K = 0, dnum = 0, alpha = 0, digits = 0;
  std::vector<uint64_t> primes;  // q_0..q_{L-1}, p_0..p_{K-1}
  std::vector<uint64_t> psi;     // minimal primitive 2N-th roots
  // device tables
  uint64_t *d_primes = nullptr;       // L+K
  b2f::Mod *d_mod = nullptr;          // L+K Barrett constants
  ulonglong2 *d_tw_fwd = nullptr;     // (L+K) x N  (psi^bitrev(k), Shoup)
  ulonglong2 *d_tw_inv = nullptr;     // (L+K) x N
  ulonglong2 *d_ninv = nullptr;       // L+K: N^-1
  ulonglong2 *d_i_factor = nullptr;   // L+K: psi^(N/2) (multiply by i)
  ulonglong2 *d_moddown_scale = nullptr;  // K: N^-1 * [Phat_k^-1] mod p_k
  ulonglong2 *d_moddown_conv = nullptr;   // L x K: [Phat_k] mod q_i
  ulonglong2 *d_moddown_pinv = nullptr;   // L: [P^-1] mod q_i
  uint64_t *d_pmod = nullptr;             // L: [P] mod q_i
  std::vector<b2f::LevelTables> levels;   // index l = 1..L
  // FFT tables for encode/decode (FP64)
  double2 *d_ksi = nullptr;     // M+1 roots exp(2 pi i k / M)
  uint32_t *d_rot_group = nullptr;  // N/2 entries 5^j mod M
  // cached NTT job tables
  std::mutex mu;
  std::map<std::vector<int>, b2f::LimbJob *> jobs;
  std::vector<void *> owned;
};

namespace b2f {
const LimbJob *job_table(b2f_context *ctx, const std::vector<int> &key,
                         const std::vector<LimbJob> &jobs);
// items x jobs_per_item limb transforms; item i reads in + i*in_stride and
// writes out + i*out_stride (strides in words).  scales == NULL: N^-1.
int launch_ntt(b2f_context *ctx, const uint64_t *in, long long in_stride,
               uint64_t *out, long long out_stride, const LimbJob *jobs,
               int jobs_per_item, int items, int inverse,
               const ulonglong2 *scales, cudaStream_t s);
// jobs for num_polys polys of (q_limbs Q + p_limbs P) limbs, contiguous
int ntt_polys(b2f_context *ctx, uint64_t *data, int num_polys, int q_limbs,
              int p_limbs, int inverse, cudaStream_t s);
inline int prime_of(const b2f_context *ctx, int q_limbs, int limb) {
  return limb < q_limbs ? limb : ctx->L + (limb - q_limbs);
}
}  // namespace b2f
