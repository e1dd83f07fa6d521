// Internal declarations shared by the libb200fhe translation units.
#pragma once
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include <nvtx3/nvToolsExt.h>

#include "../../include/b200fhe.h"
#include "modarith.cuh"

namespace b2f {

// Counts one kernel launch (relaxed atomic; read by b2f_launch_count).
void note_launch();

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
// NVTX range over one entry point (header-only NVTX v3: a no-op unless a
// profiler is attached), so profiles group kernels by the operation that
// launched them.
struct NvtxRange {
  explicit NvtxRange(const char *name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange &) = delete;
  NvtxRange &operator=(const NvtxRange &) = delete;
};
#define B2F_RANGE(name) ::b2f::NvtxRange b2f_range_guard_(name)

// Every kernel launch of the library is followed by B2F_LAUNCHED (or, where
// the launch site cleans up before returning, by note_launch and its own
// error check): the launch is counted (b2f_launch_count) and a launch error
// becomes the entry point's status.
#define B2F_LAUNCHED(what)                                        \
  do {                                                            \
    ::b2f::note_launch();                                         \
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
// Constants to reduce a value below 2^80 modulo p (2^33 < p < 2^62):
// mu = floor(2^64 / p) (fits 32 bits), r = 2^64 mod p, rs its Shoup quotient.
struct Red79 {
  uint64_t p, r, rs, mu;
};

struct LevelTables {
  int l = 0, beta = 0;
  // per Q limb i < l: N^-1 * [Qhat_{j(i),i}^-1] mod q_i (Shoup pair)
  ulonglong2 *modup_scale = nullptr;
  // ModUp conversion constants [Qhat_{j,i}] mod p_t as byte-split tensor-core
  // operands: per digit j a
  // u8 matrix of conv_rows(l+K-width_j) x conv_kpad(alpha) (conv_bytes)
  uint8_t *modup_bytes = nullptr;
  size_t modup_bytes_stride = 0;  // bytes per digit
  // rescale: for i < l-1, [q_{l-1}^-1] mod q_i and [q_{l-1}] mod q_i
  ulonglong2 *rescale_inv = nullptr;
  uint64_t *rescale_qlast = nullptr;
  // relinearisation fused with its rescale (l >= 2, K >= 1): the removed
  // limbs R = {q_{l-1}} u P (r = 0 is q_{l-1}, r = 1 + k is p_k), M = P q_{l-1}
  //   mdr_scale[r]: N^-1 [(M/r)^-1] mod r (Shoup pair w.r.t. r)
  //   mdr_rinv[r]:  1 / r in binary64
  //   mdr_bytes:    conv_bytes of the conversion of K+2 words (the K+1 removed
  //                 residues, then the rounding word v) to q_0..q_{l-2}, with
  //                 constants [M/r] mod q_i and -[M] mod q_i for v
  ulonglong2 *mdr_scale = nullptr;
  double *mdr_rinv = nullptr;
  uint8_t *mdr_bytes = nullptr;
};

// Byte-split operands of a base conversion out_t = sum_{i<w} x_i c_{t,i} mod
// p_t (t < T) for the u8 tensor-core path: x_i = sum_a x_{i,a} 2^(8a), and
// row (group G, tile m, r) of the constant matrix, r < 16, holds for target
// t = 8G + (r & 7) and output byte b = 2m + (r >> 3) the bytes b of
// c_{t,i} 2^(8a) mod p_t at column k = 8i + a.  Then
// sum_b 2^(8b) sum_k A[row(t,b)][k] x_bytes[k] = sum_i c_{t,i} x_i (mod p_t),
// and the four 16-row tiles of a group give one thread every byte position
// of its outputs.
inline int conv_wpad(int w) { return w <= 4 ? 4 : (w <= 8 ? 8 : 16); }
inline int conv_kpad(int w) { return 8 * conv_wpad(w); }
inline int conv_groups(int T) { return (T + 7) / 8; }
inline size_t conv_rows(int T) { return (size_t)conv_groups(T) * 64; }
// c(t, i) gives c_{t,i} (t < T, i < w) and p(t) the target prime; rows are
// kp >= conv_kpad(w) bytes (zero beyond 8 w)
template <class C, class Pm>
void conv_bytes(uint8_t *A, int T, int w, int kp, C c, Pm p) {
  for (size_t r = 0; r < conv_rows(T); ++r) {
    const int G = (int)(r / 64), m = (int)(r % 64) / 16, rr = (int)(r % 16);
    const int t = 8 * G + (rr & 7), b = 2 * m + (rr >> 3);
    for (int k = 0; k < kp; ++k) {
      const int i = k / 8, a = k % 8;
      uint8_t v = 0;
      if (t < T && i < w) {
        const uint64_t pt = p(t);
        const uint64_t shifted =
            (uint64_t)(((unsigned __int128)(c(t, i) % pt) << (8 * a)) % pt);
        v = (uint8_t)(shifted >> (8 * b));
      }
      A[r * kp + k] = v;
    }
  }
}

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
  b2f::Red79 *d_red79 = nullptr;      // L+K constants of reduce79
  ulonglong2 *d_tw_fwd = nullptr;     // (L+K) x N  (psi^bitrev(k), Shoup)
  ulonglong2 *d_tw_inv = nullptr;     // (L+K) x N
  // binary64 arithmetic (NTT butterflies, key inner product) when every
  // prime is below 2^50: the same twiddles as doubles, and 1/q per prime
  bool fp64_ok = false, fp64 = false;
  // BSGS multiply-accumulate: 0 = tensor cores wherever exact (mac_mma.cu),
  // 1 = CUDA cores only (b2f_set_mac_path)
  int mac_path = 0;
  // fast base conversions of the key switch (b2f_set_conv_path): 0 = the
  // faster kernel, measured on B200 (ModDown of 16+ ciphertexts on tcgen05,
  // the rest on mma.sync), 1 = mma.sync always, 2 = tcgen05 (conv_umma.cu)
  int conv_path = 0;
  // the BSGS giant chain (b2f_set_giant_chain): 0 = kept in Q_l u P with one
  // ModDown per chain, 1 = a full rotation (ModDown of both polys) per giant
  int giant_chain = 0;
  double *d_twd_fwd = nullptr, *d_twd_inv = nullptr, *d_qinv = nullptr;
  double *d_md_conv_f64 = nullptr;  // L x K: [Phat_k] mod q_i as doubles
  ulonglong2 *d_ninv = nullptr;       // L+K: N^-1
  ulonglong2 *d_i_factor = nullptr;   // L+K: psi^(N/2) (multiply by i)
  ulonglong2 *d_moddown_scale = nullptr;  // K: N^-1 * [Phat_k^-1] mod p_k
  uint8_t *d_moddown_bytes = nullptr;     // [Phat_k] mod q_i, byte split (conv_bytes)
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
// Tensor-core BSGS multiply-accumulate (mac_mma.cu): eligibility for one call
// and the launch of one chunk of G <= 8 giants starting at giant g0.
bool mac_mma_eligible(const b2f_context *ctx, int baby_count, int l, int ql, int cts);
int launch_mac_mma(b2f_context *ctx, const uint64_t *babies, int baby_count,
                   const uint64_t *pts, int g0, int G, int l, uint64_t *out,
                   int out_giants, int cts, int giant_major, int ql, cudaStream_t s);

// tcgen05 base conversions (conv_umma.cu); -1 when the shape is not taken
int launch_modup_conv_umma(b2f_context *ctx, const uint64_t *xt, uint64_t *ext, int l,
                           int cts, cudaStream_t s);
// polys: 2, or 1 for the first poly of each ciphertext at the pointers given
// (pass both pointers offset by one poly to convert the second polys only)
int launch_moddown_conv_umma(b2f_context *ctx, const uint64_t *acc, uint64_t *conv, int l,
                             int cts, cudaStream_t s, int polys = 2);

// BSGS giant chain in Q_l u P (keyswitch.cu): giant j of ciphertext c at
// sums + j gs + c cs (2 x l limbs, or 2 x (l+K) with ext) -> out
// [cts][2][l][N] = Horner over the giants with the one giant key; G >= 2
size_t giant_chain_workspace(const b2f_context *ctx, int cts, int l);
int giant_chain_ext(b2f_context *ctx, const uint64_t *sums, int ext, long long gs,
                    long long cs, int cts, int G, int l, uint64_t galois, const uint64_t *key,
                    uint64_t *out, void *ws, size_t ws_bytes, cudaStream_t s);

const LimbJob *job_table(b2f_context *ctx, const std::vector<int> &key,
                         const std::vector<LimbJob> &jobs);
// items x jobs_per_item limb transforms; item i reads in + i*in_stride and
// writes out + i*out_stride (strides in words).  scales == NULL: N^-1.
int launch_ntt(b2f_context *ctx, const uint64_t *in, long long in_stride,
               uint64_t *out, long long out_stride, const LimbJob *jobs,
               int jobs_per_item, int items, int inverse,
               const ulonglong2 *scales, cudaStream_t s);
struct ItemKeys;
// The last step of a ModDown: NTT of conv [item][2][q_limbs][N] (the P part
// converted to Q) whose epilogue writes, for item it and poly b,
//   out + keys.out(it, out_stride) + (b q_limbs + i) N, at slot dst(j):
//   ((acc_b[i][j] - NTT(conv)_b[i][j]) [P^-1]_{q_i} (* qinv_i)) + add_b[i][j]
// acc [item][2][lk][N]; add_b (optional) of ciphertext keys.ct(it) at
// add_stride; dst the slot permutation of X -> X^(g^-1), g = keys.g[at(it)].
// With z (binary64 contexts, K <= 4) the transform computes its own input,
// the conversion sum_k z_k [Phat_k]_{q_i} of the scaled P limbs l .. l+K-1 of
// z [item][2][lk][N] (conv is then not read).
// A post-operation folded into that epilogue (the Paterson-Stockmeyer step
// of homo_mul_relin_rescale_postop): the result times 2 (dbl), add_b
// subtracted instead of added (add_neg), and cadd[i] added to poly 0.
// second_only: only the second poly of each item (b = 1; conv's and acc's
// layouts unchanged), written as one poly at out + keys.out(it, out_stride) +
// i N; the conversion must come from conv (no z).
struct EpiPostOp {
  int dbl = 0;
  int add_neg = 0;
  int has_cadd = 0;
  uint64_t cadd[64] = {};  // [q_limbs] residues, by value in the kernel parameters
};
int ntt_moddown(b2f_context *ctx, uint64_t *conv, int items, int q_limbs, int lk,
                const uint64_t *acc, const uint64_t *add0, const uint64_t *add1,
                long long add_stride, uint64_t *out, long long out_stride,
                const ulonglong2 *qinv, const ItemKeys &keys, cudaStream_t s,
                const uint64_t *z = nullptr, const EpiPostOp *post = nullptr,
                bool second_only = false);
// Rescale of num_polys polys [poly][l][N] (NTT form) to out [poly][l-1][N]:
// last [poly][N] holds each poly's last limb in coefficient form; one forward
// NTT launch lifts it to every q_i in its input stage and finishes
// (c_i - NTT(lift)) q_{l-1}^-1 in its epilogue.
int ntt_rescale(b2f_context *ctx, const uint64_t *last, const uint64_t *in, uint64_t *out,
                int num_polys, int l, cudaStream_t s);
// The same with its job table given: l-1 rows LimbJob{0, i, i, i} in device
// memory (ntt_rescale takes them from the context's cache).
int ntt_rescale_jobs(b2f_context *ctx, const uint64_t *last, const uint64_t *in,
                     uint64_t *out, int num_polys, int l, const LimbJob *jobs,
                     cudaStream_t s);
// jobs for num_polys polys of (q_limbs Q + p_limbs P) limbs, contiguous
int ntt_polys(b2f_context *ctx, uint64_t *data, int num_polys, int q_limbs,
              int p_limbs, int inverse, cudaStream_t s);
inline int prime_of(const b2f_context *ctx, int q_limbs, int limb) {
  return limb < q_limbs ? limb : ctx->L + (limb - q_limbs);
}
}  // namespace b2f
