// Hybrid key switching (Han-Ki 2020) for HRotate, hoisted rotations and
// relinearisation, in the evaluation (NTT) form.
//
// For c1 at l limbs, digits D_j = [j*alpha, min((j+1)*alpha, l)), j < beta:
//   1. xt   = iNTT(c1) * [Qhat_{j,i}^-1]_{q_i}           (scale folded in iNTT)
//   2. ext_j[t] = sum_{i in D_j} xt_i * [Qhat_{j,i}]_{p_t}, t outside D_j
//      (fast base conversion), then NTT;  ext_j[t] = c1[t] for t in D_j
//   3. acc_b[t] = sum_j ext_j[t] * key[j][b][t]         (b = 0, 1)
//   4. ModDown: z_k = iNTT(acc_b[P_k]) * [Phat_k^-1]_{p_k};
//      conv_i = NTT(sum_k z_k [Phat_k]_{q_i});
//      d_b[i] = (acc_b[i] - conv_i) * [P^-1]_{q_i}
//   5. HRotate: out = (pi_g(c0 + d0), pi_g(d1)).  Step 4's last NTT finishes
//      the ModDown in its epilogue (ntt_moddown): the combine, the addition
//      of c0 and the automorphism (a scatter by g^-1) happen as the
//      transform stores, so conv never returns to HBM.  Relinearisation adds
//      (d0, d1) of the degree-2 ciphertext instead and uses g = 1.
// Every key limb (digit, poly, prime) is read by one grid row that covers all
// ciphertexts of the batch, so a batch sharing a key streams it once.
#include "b2f_internal.h"
#include "ksitems.cuh"
#include "ntt_arith.cuh"

namespace b2f {
namespace {

constexpr int TPB = 256;

// ---------------------------------------------------------------------
// Base conversion on the u8 tensor cores (mma.sync m16n8k32, s32
// accumulate).  The input words are their own byte matrix: coefficient n's
// limbs x_0..x_{w-1} stored as consecutive 64-bit words are the bytes
// x_{i,a} at k = 8 i + a of column n.  The constant matrix (conv_bytes)
// puts, for each group of 8 targets, output byte 2m in rows 0-7 and byte
// 2m+1 in rows 8-15 of tile m, so after the four tiles the thread holding
// row g has all eight byte sums of target 8G+g for its two columns:
// V = sum_b C_b 2^(8b) < 2^79, reduced once (Barrett).  Exact: the residue
// equals sum_i x_i c_{t,i} mod p_t.
// ---------------------------------------------------------------------
constexpr int CNB = 256;  // coefficients (= threads) per conversion block

__device__ __forceinline__ void mma_u8(int (&c)[4], uint32_t a0, uint32_t a1,
                                       uint32_t a2, uint32_t a3, uint32_t b0,
                                       uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

inline size_t conv_mma_smem(int kp, int T) {
  const int stride = kp / 4 + 4;  // words; = 4 mod 8 keeps fragment loads conflict free
  return ((size_t)CNB + conv_rows(T)) * stride * 4;
}

// a * b mod 2^64 and floor(a * b / 2^64) for a 32-bit b
__device__ __forceinline__ uint64_t mul_lo_32(uint64_t a, uint32_t b) {
  return (uint64_t)(uint32_t)a * b + (((uint64_t)(uint32_t)(a >> 32) * b) << 32);
}
__device__ __forceinline__ uint64_t mul_hi_32(uint64_t a, uint32_t b) {
  return ((uint64_t)(uint32_t)(a >> 32) * b + (((uint64_t)(uint32_t)a * b) >> 32)) >> 32;
}

// (hi 2^64 + lo) mod p for hi < 2^16: lo by Barrett with the 32-bit
// mu = floor(2^64/p) (quotient short by at most one, remainder < 2p), hi by
// a Shoup product with 2^64 mod p (< 2p); both lazily, then two
// conditional subtractions.
__device__ __forceinline__ uint64_t reduce79(uint64_t hi, uint64_t lo, const Red79 &R) {
  const uint64_t p = R.p;
  const uint64_t qe = mul_hi_32(lo, (uint32_t)R.mu);
  uint64_t r0 = lo - mul_lo_32(p, (uint32_t)qe);
  const uint32_t h = (uint32_t)hi;
  const uint64_t y1 = mul_lo_32(R.r, h) - mul_lo_32(p, (uint32_t)mul_hi_32(R.rs, h));
  uint64_t v = r0 + y1;  // < 4p
  v = v >= 2 * p ? v - 2 * p : v;
  return v >= p ? v - p : v;
}

// out(t): limb pointer of target t < T; red(t): its reduce79 constants.
// x: limb 0 of the w input limbs; the block converts coefficients
// [n0, n0 + CNB).  KW = 32-bit words per operand row (kp / 4).  With ROUND,
// input word w is v = floor(sum_{i<w} x_i * rinv[i] + 1/2), evaluated in
// binary64 with each product and sum rounded to nearest in i order (A holds
// the constants of w + 1 words).
template <int KW, bool ROUND = false, class Out, class Rd>
__device__ __forceinline__ void conv_mma_block(const uint64_t *__restrict__ x,
                                               int w,
                                               const uint8_t *__restrict__ A,
                                               int T, Out out, Rd red, int n0,
                                               const double *__restrict__ rinv = nullptr) {
  constexpr int ST = KW + 4;
  extern __shared__ __align__(16) uint32_t csm[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, tq = lane & 3;
  const int groups = (T + 7) / 8;
  uint32_t *Xs = csm;
  uint32_t *As = csm + CNB * ST;
  const uint4 *Ag = reinterpret_cast<const uint4 *>(A);
  const int quads = groups * 64 * (KW / 4);  // 16-byte pieces of A
  for (int idx = tid; idx < quads; idx += CNB) {
    const uint4 v = __ldg(Ag + idx);
    uint32_t *d = As + (idx / (KW / 4)) * ST + (idx % (KW / 4)) * 4;
    d[0] = v.x;
    d[1] = v.y;
    d[2] = v.z;
    d[3] = v.w;
  }
  uint64_t xv[KW / 2];
#pragma unroll
  for (int i = 0; i < KW / 2; ++i) xv[i] = i < w ? x[(size_t)i * kN + n0 + tid] : 0;
  if (ROUND) {
    double f = 0.0;
#pragma unroll
    for (int i = 0; i < KW / 2; ++i)
      if (i < w) f = __dadd_rn(f, __dmul_rn(__ull2double_rn(xv[i]), __ldg(rinv + i)));
    const uint64_t v = __double2ull_rz(__dadd_rn(f, 0.5));
#pragma unroll
    for (int i = 0; i < KW / 2; ++i)
      if (i == w) xv[i] = v;
  }
#pragma unroll
  for (int i = 0; i < KW / 2; ++i) {
    Xs[tid * ST + 2 * i] = (uint32_t)xv[i];
    Xs[tid * ST + 2 * i + 1] = (uint32_t)(xv[i] >> 32);
  }
  __syncthreads();
  // the warp's four n-tiles (B fragments read from shared memory per group)
  const uint32_t *ag = As + g * ST + tq;
  for (int G = 0; G < groups; ++G, ag += 64 * ST) {
    // A fragments of the group's four tiles, reused by the four n-tiles
    uint32_t af[4][KW / 8][4];
#pragma unroll
    for (int m = 0; m < 4; ++m)
#pragma unroll
      for (int kk = 0; kk < KW / 8; ++kk) {
        const uint32_t *ar = ag + m * 16 * ST + 8 * kk;
        af[m][kk][0] = ar[0];
        af[m][kk][1] = ar[8 * ST];
        af[m][kk][2] = ar[4];
        af[m][kk][3] = ar[8 * ST + 4];
      }
    const int t = 8 * G + g;
    const bool live = t < T;
    Red79 R{};
    uint64_t *obase = nullptr;
    if (live) {
      R = red(t);
      obase = out(t) + n0 + 2 * tq;
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      uint32_t bf[KW / 4];
      {
        const uint32_t *xr = Xs + ((warp * 4 + u) * 8 + g) * ST + tq;
#pragma unroll
        for (int kk = 0; kk < KW / 8; ++kk) {
          bf[2 * kk] = xr[8 * kk];
          bf[2 * kk + 1] = xr[8 * kk + 4];
        }
      }
      int acc[4][4];
#pragma unroll
      for (int m = 0; m < 4; ++m) acc[m][0] = acc[m][1] = acc[m][2] = acc[m][3] = 0;
#pragma unroll
      for (int kk = 0; kk < KW / 8; ++kk)
#pragma unroll
        for (int m = 0; m < 4; ++m)
          mma_u8(acc[m], af[m][kk][0], af[m][kk][1], af[m][kk][2], af[m][kk][3],
                 bf[2 * kk], bf[2 * kk + 1]);
      if (live) {
        uint64_t *o = obase + (warp * 4 + u) * 8;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          // byte sums 0-3 and 4-7 (each < 2^22): u32 x constant + u64 terms,
          // one wide multiply-add each
          uint64_t lo4 = (uint32_t)acc[0][c], hi4 = (uint32_t)acc[2][c];
          lo4 += (uint64_t)(uint32_t)acc[0][2 + c] * 256u;
          hi4 += (uint64_t)(uint32_t)acc[2][2 + c] * 256u;
          lo4 += (uint64_t)(uint32_t)acc[1][c] * 65536u;
          hi4 += (uint64_t)(uint32_t)acc[3][c] * 65536u;
          lo4 += (uint64_t)(uint32_t)acc[1][2 + c] * 16777216u;
          hi4 += (uint64_t)(uint32_t)acc[3][2 + c] * 16777216u;
          const uint64_t lo = lo4 + (hi4 << 32);
          const uint64_t hi = (hi4 >> 32) + (lo < lo4);
          o[c] = reduce79(hi, lo, R);
        }
      }
    }
  }
}

// ModUp step 2 on tensor cores.  grid (N/CNB, beta, cts)
template <int KW>
__global__ void __launch_bounds__(CNB) modup_conv_mma_kernel(
    const uint64_t *__restrict__ xt, uint64_t *__restrict__ ext,
    const uint8_t *__restrict__ bytes, size_t bytes_stride,
    const Red79 *__restrict__ reds, int l, int K, int L, int alpha) {
  const int j = blockIdx.y, ct = blockIdx.z, beta = gridDim.y, lk = l + K;
  const int lo = j * alpha, hi = min(lo + alpha, l), w = hi - lo;
  uint64_t *dst = ext + ((size_t)ct * beta + j) * lk * kN;
  conv_mma_block<KW>(
      xt + ((size_t)ct * l + lo) * kN, w, bytes + j * bytes_stride, lk - w,
      [=](int tau) { return dst + (size_t)(tau < lo ? tau : tau + w) * kN; },
      [=](int tau) {
        const int t = tau < lo ? tau : tau + w;
        return reds[t < l ? t : L + (t - l)];
      },
      blockIdx.x * CNB);
}

// ModDown step 4b on tensor cores.  grid (N/CNB, 2, cts)
template <int KW>
__global__ void __launch_bounds__(CNB) moddown_conv_mma_kernel(
    const uint64_t *__restrict__ acc, uint64_t *__restrict__ conv_out,
    const uint8_t *__restrict__ bytes, const Red79 *__restrict__ reds, int l,
    int K) {
  const int b = blockIdx.y, ct = blockIdx.z, lk = l + K;
  uint64_t *o = conv_out + (((size_t)ct * 2 + b) * l) * kN;
  conv_mma_block<KW>(
      acc + (((size_t)ct * 2 + b) * lk + l) * kN, K, bytes, l,
      [=](int t) { return o + (size_t)t * kN; }, [=](int t) { return reds[t]; },
      blockIdx.x * CNB);
}

// Fused relinearise + rescale, step 4: the K+1 removed limbs (coefficient
// form, times N^-1 (M/r)^-1, limbs l-1 .. l+K-1 of acc) and their rounding
// word to each q_i, i < l-1.  grid (N/CNB, 2, cts); conv [ct][2][l-1][N]
template <int KW>
__global__ void __launch_bounds__(CNB) moddown_rescale_conv_mma_kernel(
    const uint64_t *__restrict__ acc, uint64_t *__restrict__ conv_out,
    const uint8_t *__restrict__ bytes, const double *__restrict__ rinv,
    const Red79 *__restrict__ reds, int l, int K) {
  const int b = blockIdx.y, ct = blockIdx.z, lk = l + K;
  uint64_t *o = conv_out + (((size_t)ct * 2 + b) * (l - 1)) * kN;
  conv_mma_block<KW, true>(
      acc + (((size_t)ct * 2 + b) * lk + l - 1) * kN, K + 1, bytes, l - 1,
      [=](int t) { return o + (size_t)t * kN; }, [=](int t) { return reds[t]; },
      blockIdx.x * CNB, rinv);
}

template <class Kern>
int set_smem(Kern k, size_t bytes) {
  if (bytes > 48 * 1024)
    B2F_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)bytes));
  return B2F_OK;
}

int launch_modup_conv(b2f_context *ctx, const uint64_t *xt, uint64_t *ext, int l,
                      int cts, cudaStream_t s) {
  if (ctx->conv_path == 2) {
    const int rc = launch_modup_conv_umma(ctx, xt, ext, l, cts, s);
    if (rc >= 0) return rc;
  }
  const LevelTables &T = ctx->levels[l];
  const int K = ctx->K, lk = l + K, kp = conv_kpad(ctx->alpha);
  const size_t sm = conv_mma_smem(kp, lk);
  const dim3 grid(kN / CNB, T.beta, cts);
  int rc;
#define B2F_MODUP(KWV)                                                        \
  if ((rc = set_smem(modup_conv_mma_kernel<KWV>, sm))) return rc;             \
  modup_conv_mma_kernel<KWV><<<grid, CNB, sm, s>>>(                           \
      xt, ext, T.modup_bytes, T.modup_bytes_stride, ctx->d_red79, l, K, ctx->L, \
      ctx->alpha);
  if (kp == 32) {
    B2F_MODUP(8)
  } else if (kp == 64) {
    B2F_MODUP(16)
  } else {
    B2F_MODUP(32)
  }
#undef B2F_MODUP
  B2F_LAUNCHED("modup_conv_mma_kernel");
  return B2F_OK;
}

// polys 1: the first poly of each ciphertext only (offset both pointers by
// one poly for the second)
int launch_moddown_conv(b2f_context *ctx, const uint64_t *acc, uint64_t *conv,
                        int l, int cts, cudaStream_t s, int polys = 2) {
  // tcgen05 by default only from 32 polys (16 ciphertexts): per ModDown
  // conversion at l = 13 it takes 149 against 152.5 us there, but 83.5 / 79.5
  // us at 8 ciphertexts, 52.4 / 41.9 at 4 and 23.7 / 15.1 at 1 (64 coefficient
  // tiles a launch cannot fill the GPU)
  if (ctx->conv_path == 2 || (ctx->conv_path == 0 && cts * polys >= 32)) {
    const int rc = launch_moddown_conv_umma(ctx, acc, conv, l, cts, s, polys);
    if (rc >= 0) return rc;
  }
  const int K = ctx->K, kp = conv_kpad(K);
  const size_t sm = conv_mma_smem(kp, l);
  const dim3 grid(kN / CNB, polys, cts);
  int rc;
#define B2F_MODDOWN(KWV)                                                \
  if ((rc = set_smem(moddown_conv_mma_kernel<KWV>, sm))) return rc;     \
  moddown_conv_mma_kernel<KWV><<<grid, CNB, sm, s>>>(acc, conv, ctx->d_moddown_bytes, \
                                                     ctx->d_red79, l, K);
  if (kp == 32) {
    B2F_MODDOWN(8)
  } else if (kp == 64) {
    B2F_MODDOWN(16)
  } else {
    B2F_MODDOWN(32)
  }
#undef B2F_MODDOWN
  B2F_LAUNCHED("moddown_conv_mma_kernel");
  return B2F_OK;
}

int launch_moddown_rescale_conv(b2f_context *ctx, const uint64_t *acc,
                                uint64_t *conv, int l, int cts, cudaStream_t s) {
  const LevelTables &T = ctx->levels[l];
  const int K = ctx->K, kp = conv_kpad(K + 2);
  const size_t sm = conv_mma_smem(kp, l - 1);
  const dim3 grid(kN / CNB, 2, cts);
  int rc;
#define B2F_MDR(KWV)                                                              \
  if ((rc = set_smem(moddown_rescale_conv_mma_kernel<KWV>, sm))) return rc;       \
  moddown_rescale_conv_mma_kernel<KWV><<<grid, CNB, sm, s>>>(                     \
      acc, conv, T.mdr_bytes, T.mdr_rinv, ctx->d_red79, l, K);
  if (kp == 32) {
    B2F_MDR(8)
  } else if (kp == 64) {
    B2F_MDR(16)
  } else {
    B2F_MDR(32)
  }
#undef B2F_MDR
  B2F_LAUNCHED("moddown_rescale_conv_mma_kernel");
  return B2F_OK;
}

// Step 3: key inner product.  grid (N/TPB, items, l+K): the slowest grid
// axis is the target limb, so a key limb shared by a batch, or an ext limb
// shared by the hoisted rotations of one ciphertext (ext_stride = 0, c1_stride
// = 0), is reused across the items in L2.  BK: the sums (beta products, one
// more with pre0) stay below 2^(64+k) for every prime of the launch, so the
// one-word Barrett reduce_bk replaces the 128-bit one (the kernel is
// issue-bound; the reduction was half its instructions).
// CHAIN: a rotation left in Q_l u P finishes here, the automorphism folded
// into the store: the sums at evaluation n get x_0[n] (the first poly of the
// ciphertext of item it, ct = items.ct(it), over Q_l u P, or with x_q P times
// a Q_l poly on the Q limbs: one more product term before the reduction) and,
// after the reduction, s_b[k] (optional: the next giant's sum of a giant
// chain step, as giant_step_kernel adds it), and go to out +
// items.out(it, 2 (l+K) N) at k = pi_g^-1(n), g = items.g[items.at(it)]; acc
// is never written and the automorphism costs no pass of its own.
struct ChainStep {
  const uint64_t *x = nullptr;  // [ct][2][l+K][N], or (x_q) [ct][2][l][N], at x_cs
  long long x_cs = 0;
  int x_q = 0;
  const uint64_t *s = nullptr;  // null, or [ct][2][l+K or (s_q) l][N] at s_cs
  long long s_cs = 0;
  int s_q = 0;
  uint64_t *out = nullptr;      // [..][2][l+K][N] at items.out
};
template <bool BK, bool CHAIN = false>
__global__ void __launch_bounds__(TPB) key_inner_product_kernel(
    const uint64_t *__restrict__ c1, long long c1_stride,
    const uint64_t *__restrict__ ext, long long ext_stride, const ItemKeys items,
    uint64_t *__restrict__ acc, const Mod *__restrict__ mods, int l, int K,
    int L, int alpha, int beta, const uint64_t *__restrict__ pre0 = nullptr,
    const uint64_t *__restrict__ pre1 = nullptr, long long pre_stride = 0,
    const uint64_t *__restrict__ pmod = nullptr, const ChainStep chain = ChainStep{}) {
  const int n = blockIdx.x * TPB + threadIdx.x;
  const int it = blockIdx.y, t = blockIdx.z, ct = items.ct(it);
  const int lk = l + K, np = L + K;
  const int gp = t < l ? t : L + (t - l);
  const Mod M = mods[gp];
  const uint64_t *__restrict__ key = items.key[items.at(it)];
  U128 s0 = {0, 0}, s1 = {0, 0};
  // digits in groups of four: all loads of a group are issued before its
  // multiplies, so each thread keeps 12 memory requests in flight
  auto digit = [&](int j) -> const uint64_t * {
    const int lo = j * alpha, hi = min(lo + alpha, l);
    return (t >= lo && t < hi) ? c1 + ct * c1_stride + (size_t)t * kN + n
                               : ext + ct * ext_stride + ((size_t)j * lk + t) * kN + n;
  };
  const size_t kstep = (size_t)2 * np * kN;
  const uint64_t *kb = key + (size_t)gp * kN + n;
  for (int j = 0; j < beta; j += 4) {
    uint64_t e[4], k0[4], k1[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (j + u < beta) {
        e[u] = *digit(j + u);
        k0[u] = __ldg(kb + (j + u) * kstep);
        k1[u] = __ldg(kb + (j + u) * kstep + (size_t)np * kN);
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (j + u < beta) {
        mac128(s0, e[u], k0[u]);
        mac128(s1, e[u], k1[u]);
      }
    }
  }
  if (pre0 != nullptr && t < l) {  // + P (pre0, pre1) on the Q limbs
    const uint64_t pm = pmod[t];
    const size_t at = ct * pre_stride + (size_t)t * kN + n;
    mac128(s0, pre0[at], pm);
    mac128(s1, pre1[at], pm);
  }
  if constexpr (CHAIN) {
    const uint64_t *x0 = chain.x + ct * chain.x_cs + (size_t)t * kN + n;
    if (!chain.x_q)
      mac128(s0, *x0, 1);
    else if (t < l)  // a Q_l poly has no limb t >= l
      mac128(s0, *x0, pmod[t]);
    uint64_t w0 = BK ? reduce_bk(s0.hi, s0.lo, M) : reduce128(s0.hi, s0.lo, M);
    uint64_t w1 = BK ? reduce_bk(s1.hi, s1.lo, M) : reduce128(s1.hi, s1.lo, M);
    const uint32_t k = auto_src((uint32_t)n, galois_inverse(items.g[items.at(it)]));
    if (chain.s) {
      const uint64_t *sb = chain.s + ct * chain.s_cs + (size_t)t * kN + k;
      const size_t sp = (size_t)(chain.s_q ? l : lk) * kN;  // poly stride of s
      if (!chain.s_q) {
        w0 = add_mod(w0, sb[0], M.q);
        w1 = add_mod(w1, sb[sp], M.q);
      } else if (t < l) {
        w0 = add_mod(w0, mul_mod(pmod[t], sb[0], M), M.q);
        w1 = add_mod(w1, mul_mod(pmod[t], sb[sp], M), M.q);
      }
    }
    uint64_t *o = chain.out + items.out(it, 2LL * lk * kN) + (size_t)t * kN + k;
    o[0] = w0;
    o[(size_t)lk * kN] = w1;
    return;
  }
  uint64_t *o = acc + ((size_t)it * 2 * lk + t) * kN + n;
  if (BK) {
    o[0] = reduce_bk(s0.hi, s0.lo, M);
    o[(size_t)lk * kN] = reduce_bk(s1.hi, s1.lo, M);
  } else {
    o[0] = reduce128(s0.hi, s0.lo, M);
    o[(size_t)lk * kN] = reduce128(s1.hi, s1.lo, M);
  }
}

bool sums_fit_reduce_bk(const b2f_context *ctx, int l, int terms);

// The key inner product of rotations left in Q_l u P with the automorphism
// and the additions of CHAIN above folded in (integer contexts).
int launch_key_inner_product_chain(b2f_context *ctx, int cts, const uint64_t *c1,
                                   long long c1_stride, const uint64_t *ext,
                                   long long ext_stride, const ItemKeys &items, int l,
                                   const ChainStep &chain, cudaStream_t s) {
  const int K = ctx->K, beta = ctx->levels[l].beta;
  const dim3 grid(kN / TPB, cts, l + K);
  if (sums_fit_reduce_bk(ctx, l, beta + 1))
    key_inner_product_kernel<true, true><<<grid, TPB, 0, s>>>(
        c1, c1_stride, ext, ext_stride, items, nullptr, ctx->d_mod, l, K, ctx->L, ctx->alpha,
        beta, nullptr, nullptr, 0, ctx->d_pmod, chain);
  else
    key_inner_product_kernel<false, true><<<grid, TPB, 0, s>>>(
        c1, c1_stride, ext, ext_stride, items, nullptr, ctx->d_mod, l, K, ctx->L, ctx->alpha,
        beta, nullptr, nullptr, 0, ctx->d_pmod, chain);
  B2F_LAUNCHED("key_inner_product_kernel");
  return B2F_OK;
}

// terms * (q - 1)^2 < 2^(64+k) for every prime of Q_l u P: sums of `terms`
// products of residues may take reduce_bk
bool sums_fit_reduce_bk(const b2f_context *ctx, int l, int terms) {
  using u128 = unsigned __int128;
  for (int t = 0; t < l + ctx->K; ++t) {
    const uint64_t q = ctx->primes[t < l ? t : ctx->L + t - l];
    const int k = 63 - __builtin_clzll(q);
    if (k < 1 || k > 62 || (u128)(q - 1) * (q - 1) * (u128)terms >= (u128)1 << (64 + k))
      return false;
  }
  return true;
}

// Step 3 in binary64 (every prime below 2^50): each product is an exact
// signed residue of magnitude <= q (FpArith::mul), sums of up to three stay
// exact integers below 2^53 and are brought back within q/2 by one rounding
// reduction per group; the result equals the integer kernel's.  grid
// (N/(2 TPB), items, l+K): a thread owns coefficients n and n + N/2.
__global__ void __launch_bounds__(TPB) key_inner_product_f64_kernel(
    const uint64_t *__restrict__ c1, long long c1_stride,
    const uint64_t *__restrict__ ext, long long ext_stride, const ItemKeys items,
    uint64_t *__restrict__ acc, const uint64_t *__restrict__ primes,
    const double *__restrict__ qinvs, int l, int K, int L, int alpha, int beta,
    const uint64_t *__restrict__ pre0, const uint64_t *__restrict__ pre1,
    long long pre_stride, const uint64_t *__restrict__ pmod) {
  using F = FpArith;
  constexpr int H = kN / 2;  // each thread: coefficients n and n + N/2
  const int n = blockIdx.x * TPB + threadIdx.x;
  const int it = blockIdx.y, t = blockIdx.z, ct = items.ct(it);
  const int lk = l + K, np = L + K;
  const int gp = t < l ? t : L + (t - l);
  const F ar(primes, qinvs, gp);
  const uint64_t *__restrict__ key = items.key[items.at(it)];
  double s0[2] = {0.0, 0.0}, s1[2] = {0.0, 0.0};
  auto digit = [&](int j) -> const uint64_t * {
    const int lo = j * alpha, hi = min(lo + alpha, l);
    return (t >= lo && t < hi) ? c1 + ct * c1_stride + (size_t)t * kN + n
                               : ext + ct * ext_stride + ((size_t)j * lk + t) * kN + n;
  };
  const size_t kstep = (size_t)2 * np * kN;
  const uint64_t *kb = key + (size_t)gp * kN + n;
  // digits in groups of three: all 18 loads of a group are in flight before
  // its multiplies
  for (int j = 0; j < beta; j += 3) {
    uint64_t e[3][2], k0[3][2], k1[3][2];
#pragma unroll
    for (int u = 0; u < 3; ++u) {
      if (j + u < beta) {
        const uint64_t *d = digit(j + u);
        const uint64_t *k = kb + (j + u) * kstep;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          e[u][h] = d[h * H];
          k0[u][h] = __ldg(k + h * H);
          k1[u][h] = __ldg(k + (size_t)np * kN + h * H);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < 3; ++u) {
      if (j + u < beta) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const double ed = F::from_word(e[u][h]);
          s0[h] = __dadd_rn(s0[h], ar.mul(ed, F::from_word(k0[u][h])));
          s1[h] = __dadd_rn(s1[h], ar.mul(ed, F::from_word(k1[u][h])));
        }
      }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      s0[h] = ar.red(s0[h]);
      s1[h] = ar.red(s1[h]);
    }
  }
  uint64_t *o = acc + ((size_t)it * 2 * lk + t) * kN + n;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    if (pre0 != nullptr && t < l) {  // + P (pre0, pre1) on the Q limbs
      const double pm = F::from_word(pmod[t]);
      const size_t at = ct * pre_stride + (size_t)t * kN + n + h * H;
      s0[h] = __dadd_rn(s0[h], ar.mul(F::from_word(pre0[at]), pm));
      s1[h] = __dadd_rn(s1[h], ar.mul(F::from_word(pre1[at]), pm));
    }
    o[h * H] = F::to_word(ar.full(s0[h]));
    o[(size_t)lk * kN + h * H] = F::to_word(ar.full(s1[h]));
  }
}

// Step 3 in binary64, software-pipelined: a block walks IPR tiles of 2 TPB
// consecutive coefficients of one (item, target limb); each thread copies its
// next tile's digit and key words (16-byte pieces: coefficients n, n+1) into
// its own slots of a double-buffered shared array with cp.async while it
// computes the current tile, so loads stay in flight through the arithmetic.
// Slots are private to their thread: cp.async.wait_group alone orders them.
// grid (N / (2 TPB IPR), items, l+K); dynamic shared memory 2 x 3 beta x TPB
// x 16 bytes (beta <= 4).  Same arithmetic as key_inner_product_f64_kernel.
constexpr int IPR = 8;  // tiles per block

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
  const uint32_t d = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(d), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait1() {
  asm volatile("cp.async.wait_group 1;\n" ::: "memory");
}

__global__ void __launch_bounds__(TPB, 2) key_inner_product_f64_pipe_kernel(
    const uint64_t *__restrict__ c1, long long c1_stride,
    const uint64_t *__restrict__ ext, long long ext_stride, const ItemKeys items,
    uint64_t *__restrict__ acc, const uint64_t *__restrict__ primes,
    const double *__restrict__ qinvs, int l, int K, int L, int alpha, int beta) {
  using F = FpArith;
  extern __shared__ __align__(16) ulonglong2 ipsm[];  // [stage][3 beta][TPB]
  const int tid = threadIdx.x;
  const int it = blockIdx.y, t = blockIdx.z, ct = items.ct(it);
  const int lk = l + K, np = L + K, A = 3 * beta;
  const int gp = t < l ? t : L + (t - l);
  const F ar(primes, qinvs, gp);
  const uint64_t *__restrict__ key = items.key[items.at(it)];
  const size_t kstep = (size_t)2 * np * kN;
  const uint64_t *kb = key + (size_t)gp * kN;
  const int nb = blockIdx.x * (2 * TPB * IPR);
  auto issue = [&](int r) {
    const int n = nb + 2 * (tid + TPB * r);
    ulonglong2 *slot = ipsm + (size_t)(r & 1) * A * TPB + tid;
    for (int j = 0; j < beta; ++j) {
      const int lo = j * alpha, hi = min(lo + alpha, l);
      const uint64_t *d = (t >= lo && t < hi)
                              ? c1 + ct * c1_stride + (size_t)t * kN
                              : ext + ct * ext_stride + ((size_t)j * lk + t) * kN;
      const uint64_t *k = kb + j * kstep;
      cp_async16(slot + (3 * j) * TPB, d + n);
      cp_async16(slot + (3 * j + 1) * TPB, k + n);
      cp_async16(slot + (3 * j + 2) * TPB, k + (size_t)np * kN + n);
    }
    cp_async_commit();
  };
  issue(0);
  for (int r = 0; r < IPR; ++r) {
    if (r + 1 < IPR)
      issue(r + 1);
    else
      cp_async_commit();  // an empty group keeps "all but the newest" meaning tile r
    cp_async_wait1();
    const ulonglong2 *slot = ipsm + (size_t)(r & 1) * A * TPB + tid;
    double s0[2] = {0.0, 0.0}, s1[2] = {0.0, 0.0};
    for (int j = 0; j < beta; ++j) {
      const ulonglong2 e = slot[(3 * j) * TPB], k0 = slot[(3 * j + 1) * TPB],
                       k1 = slot[(3 * j + 2) * TPB];
      const double e0 = F::from_word(e.x), e1 = F::from_word(e.y);
      s0[0] = __dadd_rn(s0[0], ar.mul(e0, F::from_word(k0.x)));
      s0[1] = __dadd_rn(s0[1], ar.mul(e1, F::from_word(k0.y)));
      s1[0] = __dadd_rn(s1[0], ar.mul(e0, F::from_word(k1.x)));
      s1[1] = __dadd_rn(s1[1], ar.mul(e1, F::from_word(k1.y)));
      if (j % 3 == 2) {  // sums of up to three products stay below 2^53
        s0[0] = ar.red(s0[0]);
        s0[1] = ar.red(s0[1]);
        s1[0] = ar.red(s1[0]);
        s1[1] = ar.red(s1[1]);
      }
    }
    const int n = nb + 2 * (tid + TPB * r);
    uint64_t *o = acc + ((size_t)it * 2 * lk + t) * kN + n;
    *reinterpret_cast<ulonglong2 *>(o) =
        make_ulonglong2(F::to_word(ar.full(s0[0])), F::to_word(ar.full(s0[1])));
    *reinterpret_cast<ulonglong2 *>(o + (size_t)lk * kN) =
        make_ulonglong2(F::to_word(ar.full(s1[0])), F::to_word(ar.full(s1[1])));
  }
}

// Step 3 launcher: grid (N/TPB, items, l+K) in the context's arithmetic.
int launch_key_inner_product(b2f_context *ctx, int items_n, const uint64_t *c1,
                             long long c1_stride, const uint64_t *ext,
                             long long ext_stride, const ItemKeys &items,
                             uint64_t *acc, int l, cudaStream_t s,
                             const uint64_t *pre0 = nullptr,
                             const uint64_t *pre1 = nullptr,
                             long long pre_stride = 0) {
  const int K = ctx->K, beta = ctx->levels[l].beta;
  const dim3 grid(kN / TPB, items_n, l + K);
  if (ctx->fp64 && pre0 == nullptr && beta <= 4) {
    const size_t sm = (size_t)2 * 3 * beta * TPB * sizeof(ulonglong2);
    int rc;
    if ((rc = set_smem(key_inner_product_f64_pipe_kernel, sm))) return rc;
    key_inner_product_f64_pipe_kernel<<<dim3(kN / (2 * TPB * IPR), items_n, l + K), TPB, sm,
                                        s>>>(c1, c1_stride, ext, ext_stride, items, acc,
                                             ctx->d_primes, ctx->d_qinv, l, K, ctx->L,
                                             ctx->alpha, beta);
  } else if (ctx->fp64)
    key_inner_product_f64_kernel<<<dim3(kN / TPB / 2, items_n, l + K), TPB, 0, s>>>(
        c1, c1_stride, ext, ext_stride, items, acc, ctx->d_primes, ctx->d_qinv, l, K,
        ctx->L, ctx->alpha, beta, pre0, pre1, pre_stride, ctx->d_pmod);
  else if (sums_fit_reduce_bk(ctx, l, beta + (pre0 != nullptr)))
    key_inner_product_kernel<true><<<grid, TPB, 0, s>>>(
        c1, c1_stride, ext, ext_stride, items, acc, ctx->d_mod, l, K, ctx->L,
        ctx->alpha, beta, pre0, pre1, pre_stride, ctx->d_pmod);
  else
    key_inner_product_kernel<false><<<grid, TPB, 0, s>>>(
        c1, c1_stride, ext, ext_stride, items, acc, ctx->d_mod, l, K, ctx->L,
        ctx->alpha, beta, pre0, pre1, pre_stride, ctx->d_pmod);
  B2F_LAUNCHED("key_inner_product_kernel");
  return B2F_OK;
}




__global__ void __launch_bounds__(TPB) automorphism_kernel(
    const uint64_t *__restrict__ in, uint64_t *__restrict__ out, uint32_t g) {
  const int k = blockIdx.x * TPB + threadIdx.x;
  const size_t limb = blockIdx.y;
  out[limb * kN + k] = in[limb * kN + auto_src(k, g)];
}

// Extended-basis rotation output (double hoisting): for every limb t of
// Q_l u P, out0[t][k] = (t < l ? [P]_{q_t} c0[t] : 0)[src] + acc0[t][src],
// out1[t][k] = acc1[t][src], src = pi_g(k); an item without a key (g = 1)
// has no acc and its output is (P c0, P c1).  grid (N/TPB, l+K, 2 items);
// item r reads acc slot slot[r] (-1: none).
struct ExtItems {
  uint32_t g[kMaxItems];
  int16_t slot[kMaxItems];
};
__global__ void __launch_bounds__(TPB) ext_combine_kernel(
    const uint64_t *__restrict__ acc, const uint64_t *__restrict__ ct,
    uint64_t *__restrict__ out, const Mod *__restrict__ mods,
    const uint64_t *__restrict__ pmod, int l, int K, int L, const ExtItems items,
    int identity_only = 0) {
  const int k = blockIdx.x * TPB + threadIdx.x;
  const int t = blockIdx.y, b = blockIdx.z & 1, r = blockIdx.z >> 1;
  const int lk = l + K;
  const uint32_t g = items.g[r];
  const int slot = items.slot[r];
  if (identity_only && slot >= 0) return;  // written by the key inner product
  const uint32_t src = g == 1 ? (uint32_t)k : auto_src(k, g);
  const Mod M = mods[t < l ? t : L + (t - l)];
  const uint64_t *a = slot >= 0 ? acc + (size_t)slot * 2 * lk * kN : nullptr;
  uint64_t v = 0;
  if (t < l && (a == nullptr || b == 0))
    v = mul_mod(pmod[t], ct[((size_t)b * l + t) * kN + src], M);
  if (a) v = add_mod(v, a[((size_t)b * lk + t) * kN + src], M.q);
  out[(((size_t)r * 2 + b) * lk + t) * kN + k] = v;
}

// One step of the BSGS giant chain kept in Q_l u P (Horner over the giants,
// one ModDown at the end): for ciphertext c, limb t < l+K and poly b,
//   out_b[t][k] = x_b[t][src] + acc_b[t][src] + s_b[t][k],  src = pi_g(k),
// x_1 = 0 (the key switch replaced the second poly); x_0 the previous state's
// first poly over Q_l u P ([c][2][l+K][N]) or, x_q, P times the first poly of
// a Q_l ciphertext (zero on the P limbs); s the next giant's sum over
// Q_l u P or, s_q, P times a Q_l ciphertext.  x and s at their ciphertext
// strides (words).  grid (N/TPB, l+K, 2 C).
__global__ void __launch_bounds__(TPB) giant_step_kernel(
    const uint64_t *__restrict__ x, int x_q, long long x_cs, const uint64_t *__restrict__ acc,
    const uint64_t *__restrict__ sg, int s_q, long long s_cs, uint64_t *__restrict__ out,
    const Mod *__restrict__ mods, const uint64_t *__restrict__ pmod, int l, int K, int L,
    uint32_t g) {
  const int k = blockIdx.x * TPB + threadIdx.x;
  const int t = blockIdx.y, b = blockIdx.z & 1, c = blockIdx.z >> 1;
  const int lk = l + K;
  const uint32_t src = auto_src(k, g);
  const Mod M = mods[t < l ? t : L + (t - l)];
  uint64_t v = acc[(((size_t)c * 2 + b) * lk + t) * kN + src];
  if (b == 0) {
    const uint64_t *x0 = x + c * x_cs + (size_t)t * kN + src;
    if (!x_q)
      v = add_mod(v, *x0, M.q);
    else if (t < l)
      v = add_mod(v, mul_mod(pmod[t], *x0, M), M.q);
  }
  const uint64_t *sb = sg + c * s_cs + ((size_t)b * (s_q ? l : lk) + t) * kN + k;
  if (!s_q)
    v = add_mod(v, *sb, M.q);
  else if (t < l)
    v = add_mod(v, mul_mod(pmod[t], *sb, M), M.q);
  out[(((size_t)c * 2 + b) * lk + t) * kN + k] = v;
}

// ---------------------------------------------------------------------
// host orchestration
// ---------------------------------------------------------------------
struct Scratch {
  b2f_context *ctx;
  cudaStream_t s;
  void *owned = nullptr;
  char *base = nullptr;
  size_t used = 0, cap = 0;
  int init(void *ws, size_t ws_bytes, size_t need) {
    if (ws) {
      // buffers are carved at 256-byte granularity and read and written with
      // vector accesses of up to 32 bytes
      if ((uintptr_t)ws & 255) {
        set_error("workspace must be 256-byte aligned (%p)", ws);
        return B2F_ERR_ARG;
      }
      if (ws_bytes < need) {
        set_error("workspace too small: %zu bytes given, %zu needed", ws_bytes,
                  need);
        return B2F_ERR_ARG;
      }
      base = static_cast<char *>(ws);
      cap = ws_bytes;
      return B2F_OK;
    }
    B2F_CUDA(cudaMallocAsync(&owned, need ? need : 16, s));
    base = static_cast<char *>(owned);
    cap = need;
    return B2F_OK;
  }
  uint64_t *take(size_t words) {
    size_t bytes = (words * 8 + 255) & ~size_t(255);
    char *p = base + used;
    used += bytes;
    return reinterpret_cast<uint64_t *>(p);
  }
  ~Scratch() {
    if (owned) cudaFreeAsync(owned, s);
  }
};

inline size_t rnd(size_t words) { return (words * 8 + 255) & ~size_t(255); }

size_t modup_bytes(const b2f_context *ctx, int cts, int l) {
  const int beta = (l + ctx->alpha - 1) / ctx->alpha;
  return rnd((size_t)cts * l * kN) + rnd((size_t)cts * beta * (l + ctx->K) * kN);
}
size_t moddown_bytes(const b2f_context *ctx, int cts, int l) {
  return rnd((size_t)cts * 2 * (l + ctx->K) * kN) + rnd((size_t)cts * 2 * l * kN);
}

// ModUp of c1 (cts ciphertext-strided) into ext; xt is scratch.
int modup(b2f_context *ctx, const uint64_t *c1, long long c1_stride, int cts,
          int l, uint64_t *xt, uint64_t *ext, cudaStream_t s) {
  const LevelTables &T = ctx->levels[l];
  const int K = ctx->K, lk = l + K, beta = T.beta, alpha = ctx->alpha;
  // 1. iNTT with the per-digit Qhat^-1 scale: c1 -> xt
  std::vector<LimbJob> jobs(l);
  for (int i = 0; i < l; ++i)
    jobs[i] = LimbJob{(uint32_t)i, (uint32_t)i, (uint16_t)i, (uint16_t)i, 0};
  const LimbJob *d = job_table(ctx, {1, l}, jobs);
  if (!d) return B2F_ERR_NOMEM;
  int rc = launch_ntt(ctx, c1, c1_stride, xt, (long long)l * kN, d, l, cts, 1,
                      T.modup_scale, s);
  if (rc) return rc;
  // 2. base conversion
  if ((rc = launch_modup_conv(ctx, xt, ext, l, cts, s))) return rc;
  // 3. NTT of the converted limbs
  std::vector<LimbJob> fj;
  for (int j = 0; j < beta; ++j) {
    int lo = j * alpha, hi = std::min(lo + alpha, l);
    for (int t = 0; t < lk; ++t) {
      if (t >= lo && t < hi) continue;
      uint32_t off = (uint32_t)(j * lk + t);
      fj.push_back(LimbJob{off, off, (uint16_t)prime_of(ctx, l, t), 0, 0});
    }
  }
  d = job_table(ctx, {2, l}, fj);
  if (!d) return B2F_ERR_NOMEM;
  const long long es = (long long)beta * lk * kN;
  return launch_ntt(ctx, ext, es, ext, es, d, (int)fj.size(), cts, 0, nullptr,
                    s);
}

// Inner product with one key and ModDown; writes out (cts x 2 x l limbs).
int ip_moddown(b2f_context *ctx, const uint64_t *c1, long long c1_stride,
               const uint64_t *ext, long long ext_stride, int cts, int l,
               const ItemKeys &items, const uint64_t *add0, const uint64_t *add1,
               long long add_stride, uint64_t *out, long long out_stride,
               uint64_t *acc, uint64_t *conv, cudaStream_t s) {
  const LevelTables &T = ctx->levels[l];
  const int K = ctx->K, lk = l + K;
  int rc = launch_key_inner_product(ctx, cts, c1, c1_stride, ext, ext_stride, items,
                                    acc, l, s);
  if (rc) return rc;
  // iNTT of the P limbs of both polys, scaled by N^-1 Phat_k^-1
  std::vector<LimbJob> pj;
  for (int b = 0; b < 2; ++b)
    for (int k = 0; k < K; ++k) {
      uint32_t off = (uint32_t)(b * lk + l + k);
      pj.push_back(LimbJob{off, off, (uint16_t)(ctx->L + k), (uint16_t)k, 0});
    }
  const LimbJob *d = job_table(ctx, {3, l}, pj);
  if (!d) return B2F_ERR_NOMEM;
  const long long as = 2LL * lk * kN;
  rc = launch_ntt(ctx, acc, as, acc, as, d, 2 * K, cts, 1,
                      ctx->d_moddown_scale, s);
  if (rc) return rc;
  if (ctx->fp64 && ctx->d_md_conv_f64)  // the conversion inside the transform
    return ntt_moddown(ctx, conv, cts, l, lk, acc, add0, add1, add_stride, out,
                       out_stride, nullptr, items, s, acc);
  if ((rc = launch_moddown_conv(ctx, acc, conv, l, cts, s))) return rc;
  return ntt_moddown(ctx, conv, cts, l, lk, acc, add0, add1, add_stride, out, out_stride,
                     nullptr, items, s);
}

int check_level(const b2f_context *ctx, int l, const char *fn) {
  if (!ctx) {
    set_error("%s: null context", fn);
    return B2F_ERR_ARG;
  }
  if (l < 1 || l > ctx->L) {
    set_error("%s: level limbs %d outside [1, %d]", fn, l, ctx->L);
    return B2F_ERR_ARG;
  }
  if (ctx->K < 1 || ctx->K > 16) {
    set_error("%s: key switching needs 1..16 special primes (K=%d)", fn,
              ctx->K);
    return B2F_ERR_UNSUPPORTED;
  }
  if (ctx->alpha > 16) {
    set_error("%s: digits wider than 16 limbs are not supported (alpha=%d)",
              fn, ctx->alpha);
    return B2F_ERR_UNSUPPORTED;
  }
  return B2F_OK;
}

bool valid_galois(uint64_t g) { return (g & 1) && g < 2ull * kN; }

}  // namespace

size_t rotate_workspace(const b2f_context *ctx, int cts, int l) {
  return modup_bytes(ctx, cts, l) + moddown_bytes(ctx, cts, l);
}

size_t giant_chain_workspace(const b2f_context *ctx, int cts, int l) {
  const size_t lk = l + ctx->K, beta = ctx->levels[l].beta, c = cts;
  return 3 * rnd(c * 2 * lk * kN) + 2 * rnd(c * l * kN) + rnd(c * beta * lk * kN) +
         rnd(c * 2 * l * kN);
}

// Horner over the giants with the one giant key (acc = sum_{G-1}; acc =
// rot(acc) + sum_j), the chain kept in Q_l u P: a rotation's key switch leaves
// P times its result there (no ModDown), the next rotation ModDowns only the
// state's second poly (the one it key-switches) and carries the first poly's
// automorphism over in Q_l u P, and the next giant's sum joins (P times a Q_l
// sum on the Q limbs, or an extended sum as it is).  One ModDown of both
// polys ends the chain: per giant step a ModDown of one poly (K inverse, l
// forward limb transforms) instead of two, and extended sums need no ModDown
// of their own.  Giant j of ciphertext c: sums + j gs + c cs (words), 2 x l
// limbs, or 2 x (l+K) with ext; out [cts][2][l][N]; G >= 2.
int giant_chain_ext(b2f_context *ctx, const uint64_t *sums, int ext, long long gs,
                    long long cs, int cts, int G, int l, uint64_t galois, const uint64_t *key,
                    uint64_t *out, void *ws, size_t ws_bytes, cudaStream_t s) {
  int rc = check_level(ctx, l, "b2f_giant_chain");
  if (rc) return rc;
  B2F_CHECK_ARG(valid_galois(galois), "b2f_giant_chain: giant galois element %llu is not "
                "an odd residue below 2N", (unsigned long long)galois);
  B2F_CHECK_ARG(G >= 2 && cts >= 1, "b2f_giant_chain: chain of %d giants, %d ciphertexts",
                G, cts);
  Scratch sc{ctx, s};
  if ((rc = sc.init(ws, ws_bytes, giant_chain_workspace(ctx, cts, l)))) return rc;
  const int K = ctx->K, lk = l + K, beta = ctx->levels[l].beta;
  uint64_t *state[2] = {sc.take((size_t)cts * 2 * lk * kN),
                        sc.take((size_t)cts * 2 * lk * kN)};
  uint64_t *acc = sc.take((size_t)cts * 2 * lk * kN);
  uint64_t *c1p = sc.take((size_t)cts * l * kN);
  uint64_t *xt = sc.take((size_t)cts * l * kN);
  uint64_t *extd = sc.take((size_t)cts * beta * lk * kN);
  uint64_t *conv = sc.take((size_t)cts * 2 * l * kN);
  const long long as = 2LL * lk * kN;
  ItemKeys it{};
  it.key[0] = key;
  it.g[0] = (uint32_t)galois;
  it.shared = 1;
  const ItemKeys plain{{}, {1u}, {}, 1};
  // inverse transforms of the P limbs of the second poly (in place), and of
  // both polys for the last ModDown
  std::vector<LimbJob> p1, p2;
  for (int b = 0; b < 2; ++b)
    for (int k = 0; k < K; ++k) {
      const uint32_t off = (uint32_t)(b * lk + l + k);
      const LimbJob j{off, off, (uint16_t)(ctx->L + k), (uint16_t)k, 0};
      if (b) p1.push_back(j);
      p2.push_back(j);
    }
  const LimbJob *d1 = job_table(ctx, {13, l}, p1);
  const LimbJob *d2 = job_table(ctx, {3, l}, p2);
  if (!d1 || !d2) return B2F_ERR_NOMEM;

  uint64_t *x = nullptr;  // the state in Q_l u P, [cts][2][l+K][N]
  const uint64_t *top = sums + (G - 1) * gs;
  if (ext) {  // the last giant's extended sum is the first state (its own copy:
              // the second poly's P limbs are transformed in place)
    x = state[1];
    B2F_CUDA(cudaMemcpy2DAsync(x, as * 8, top, cs * 8, as * 8, cts,
                               cudaMemcpyDeviceToDevice, s));
  }
  for (int j = G - 2, cur = 0; j >= 0; --j, cur ^= 1) {
    const uint64_t *c1 = top + (size_t)l * kN;
    long long c1s = cs;
    if (x) {  // ModDown of the state's second poly: c1p = (x_1 - C(x_1[P])) P^-1
      if ((rc = launch_ntt(ctx, x, as, x, as, d1, K, cts, 1, ctx->d_moddown_scale, s)))
        return rc;
      if ((rc = launch_moddown_conv(ctx, x + (size_t)lk * kN, conv + (size_t)l * kN, l, cts,
                                    s, 1)))
        return rc;
      if ((rc = ntt_moddown(ctx, conv, cts, l, lk, x, nullptr, nullptr, 0, c1p,
                            (long long)l * kN, nullptr, plain, s, nullptr, nullptr, true)))
        return rc;
      c1 = c1p;
      c1s = (long long)l * kN;
    }
    if ((rc = modup(ctx, c1, c1s, cts, l, xt, extd, s))) return rc;
    uint64_t *next = state[cur];
    if (next == x) next = state[cur ^ 1];
    if (!ctx->fp64) {  // the step inside the key inner product
      ChainStep cs_{};
      cs_.x = x ? x : top;
      cs_.x_cs = x ? as : cs;
      cs_.x_q = x ? 0 : 1;
      cs_.s = sums + j * gs;
      cs_.s_cs = cs;
      cs_.s_q = ext ? 0 : 1;
      cs_.out = next;
      if ((rc = launch_key_inner_product_chain(ctx, cts, c1, c1s, extd,
                                               (long long)beta * lk * kN, it, l, cs_, s)))
        return rc;
    } else {
      if ((rc = launch_key_inner_product(ctx, cts, c1, c1s, extd, (long long)beta * lk * kN,
                                         it, acc, l, s)))
        return rc;
      giant_step_kernel<<<dim3(kN / TPB, lk, 2 * cts), TPB, 0, s>>>(
          x ? x : top, x ? 0 : 1, x ? as : cs, acc, sums + j * gs, ext ? 0 : 1, cs, next,
          ctx->d_mod, ctx->d_pmod, l, K, ctx->L, (uint32_t)galois);
      B2F_LAUNCHED("giant_step_kernel");
    }
    x = next;
  }
  // the one ModDown of both polys
  if ((rc = launch_ntt(ctx, x, as, x, as, d2, 2 * K, cts, 1, ctx->d_moddown_scale, s)))
    return rc;
  if (ctx->fp64 && ctx->d_md_conv_f64)
    return ntt_moddown(ctx, conv, cts, l, lk, x, nullptr, nullptr, 0, out, 2LL * l * kN,
                       nullptr, plain, s, x);
  if ((rc = launch_moddown_conv(ctx, x, conv, l, cts, s))) return rc;
  return ntt_moddown(ctx, conv, cts, l, lk, x, nullptr, nullptr, 0, out, 2LL * l * kN, nullptr,
                     plain, s);
}

}  // namespace b2f

using namespace b2f;

extern "C" {

size_t b2f_rotate_workspace(const b2f_context *ctx, int num_cts, int l) {
  if (!ctx || l < 1 || l > ctx->L || num_cts < 0) return 0;
  return rotate_workspace(ctx, num_cts, l);
}

int b2f_rotate(b2f_context *ctx, const uint64_t *ct_in, uint64_t *ct_out,
               int num_cts, int l, uint64_t galois, const uint64_t *key,
               void *ws, size_t ws_bytes, void *stream) {
  B2F_RANGE("b2f_rotate");
  int rc = check_level(ctx, l, "b2f_rotate");
  if (rc) return rc;
  B2F_CHECK_ARG(ct_in && ct_out && key && num_cts >= 0,
                "b2f_rotate: null argument");
  B2F_CHECK_ARG(valid_galois(galois), "b2f_rotate: galois element %llu is not "
                "an odd residue below 2N", (unsigned long long)galois);
  B2F_CHECK_ARG(ct_in != ct_out, "b2f_rotate: in-place rotation is not supported");
  if (num_cts == 0) return B2F_OK;
  cudaStream_t s = (cudaStream_t)stream;
  Scratch sc{ctx, s};
  if ((rc = sc.init(ws, ws_bytes, rotate_workspace(ctx, num_cts, l)))) return rc;
  const int beta = ctx->levels[l].beta, lk = l + ctx->K;
  uint64_t *xt = sc.take((size_t)num_cts * l * kN);
  uint64_t *ext = sc.take((size_t)num_cts * beta * lk * kN);
  uint64_t *acc = sc.take((size_t)num_cts * 2 * lk * kN);
  uint64_t *conv = sc.take((size_t)num_cts * 2 * l * kN);
  const long long cs = 2LL * l * kN;
  if ((rc = modup(ctx, ct_in + (size_t)l * kN, cs, num_cts, l, xt, ext, s)))
    return rc;
  ItemKeys it{};
  it.key[0] = key;
  it.g[0] = (uint32_t)galois;
  it.shared = 1;
  return ip_moddown(ctx, ct_in + (size_t)l * kN, cs, ext,
                    (long long)beta * lk * kN, num_cts, l, it, ct_in, nullptr,
                    cs, ct_out, cs, acc, conv, s);
}

size_t b2f_relinearize_workspace(const b2f_context *ctx, int num_cts, int l) {
  if (!ctx || l < 1 || l > ctx->L || num_cts < 0) return 0;
  return rotate_workspace(ctx, num_cts, l);
}

int b2f_relinearize(b2f_context *ctx, const uint64_t *ct3_in, uint64_t *ct_out,
                    int num_cts, int l, const uint64_t *relin_key, void *ws,
                    size_t ws_bytes, void *stream) {
  B2F_RANGE("b2f_relinearize");
  int rc = check_level(ctx, l, "b2f_relinearize");
  if (rc) return rc;
  B2F_CHECK_ARG(ct3_in && ct_out && relin_key && num_cts >= 0,
                "b2f_relinearize: null argument");
  if (num_cts == 0) return B2F_OK;
  cudaStream_t s = (cudaStream_t)stream;
  Scratch sc{ctx, s};
  if ((rc = sc.init(ws, ws_bytes, rotate_workspace(ctx, num_cts, l)))) return rc;
  const int beta = ctx->levels[l].beta, lk = l + ctx->K;
  uint64_t *xt = sc.take((size_t)num_cts * l * kN);
  uint64_t *ext = sc.take((size_t)num_cts * beta * lk * kN);
  uint64_t *acc = sc.take((size_t)num_cts * 2 * lk * kN);
  uint64_t *conv = sc.take((size_t)num_cts * 2 * l * kN);
  const long long s3 = 3LL * l * kN;
  const uint64_t *d2 = ct3_in + 2 * (size_t)l * kN;
  if ((rc = modup(ctx, d2, s3, num_cts, l, xt, ext, s))) return rc;
  ItemKeys it{};
  it.key[0] = relin_key;
  it.g[0] = 1u;
  it.shared = 1;
  return ip_moddown(ctx, d2, s3, ext, (long long)beta * lk * kN, num_cts, l, it,
                    ct3_in, ct3_in + (size_t)l * kN, s3, ct_out, 2LL * l * kN,
                    acc, conv, s);
}

size_t b2f_relinearize_rescale_workspace(const b2f_context *ctx, int num_cts,
                                         int l) {
  if (!ctx || l < 2 || l > ctx->L || num_cts < 0) return 0;
  return rotate_workspace(ctx, num_cts, l);
}

// Relinearisation and the rescale after it as one exact rounding division by
// M = P q_{l-1}: Y_b = P d_b + IP_b(ModUp(d2), key) over Q_l u P, then
// out_b = round(Y_b / M) over Q_{l-1}, with the removed limbs R = {q_{l-1}}
// u P converted by the rounded (centred) fast base conversion.  Saves the
// forward NTT of the l ModDown outputs and the rescale's own transforms.
static int relinearize_rescale_impl(b2f_context *ctx, const uint64_t *ct3_in,
                                    uint64_t *ct_out, int num_cts, int l,
                                    const uint64_t *relin_key, void *ws, size_t ws_bytes,
                                    void *stream, const uint64_t *sub, int sub_limbs,
                                    const EpiPostOp *post);

int b2f_relinearize_rescale(b2f_context *ctx, const uint64_t *ct3_in,
                            uint64_t *ct_out, int num_cts, int l,
                            const uint64_t *relin_key, void *ws, size_t ws_bytes,
                            void *stream) {
  B2F_RANGE("b2f_relinearize_rescale");
  return relinearize_rescale_impl(ctx, ct3_in, ct_out, num_cts, l, relin_key, ws, ws_bytes,
                                  stream, nullptr, 0, nullptr);
}

int b2f_relinearize_rescale_postop(b2f_context *ctx, const uint64_t *ct3_in,
                                   uint64_t *ct_out, int num_cts, int l,
                                   const uint64_t *relin_key, int apply_double,
                                   const uint64_t *sub, int sub_limbs,
                                   const uint64_t *scalar_residues, void *ws,
                                   size_t ws_bytes, void *stream) {
  B2F_RANGE("b2f_relinearize_rescale_postop");
  B2F_CHECK_ARG(!sub || (sub_limbs >= l - 1 && sub_limbs <= ctx->L),
                "b2f_relinearize_rescale_postop: the subtrahend has %d limbs, the result "
                "%d", sub_limbs, l - 1);
  B2F_CHECK_ARG(!sub || (sub != ct_out && sub != ct3_in),
                "b2f_relinearize_rescale_postop: the subtrahend overlaps an argument");
  B2F_CHECK_ARG(l - 1 <= 64, "b2f_relinearize_rescale_postop: at most 65 limbs");
  EpiPostOp post;
  post.dbl = apply_double ? 1 : 0;
  post.add_neg = sub ? 1 : 0;
  if (scalar_residues) {  // host residues: into the kernel parameters
    post.has_cadd = 1;
    for (int i = 0; i < l - 1; ++i) post.cadd[i] = scalar_residues[i] % ctx->primes[i];
  }
  return relinearize_rescale_impl(ctx, ct3_in, ct_out, num_cts, l, relin_key, ws, ws_bytes,
                                  stream, sub, sub_limbs, &post);
}

static int relinearize_rescale_impl(b2f_context *ctx, const uint64_t *ct3_in,
                                    uint64_t *ct_out, int num_cts, int l,
                                    const uint64_t *relin_key, void *ws, size_t ws_bytes,
                                    void *stream, const uint64_t *sub, int sub_limbs,
                                    const EpiPostOp *post) {
  int rc = check_level(ctx, l, "b2f_relinearize_rescale");
  if (rc) return rc;
  B2F_CHECK_ARG(l >= 2, "b2f_relinearize_rescale: needs at least 2 limbs, got %d", l);
  B2F_CHECK_ARG(ct3_in && ct_out && relin_key && num_cts >= 0,
                "b2f_relinearize_rescale: null argument");
  B2F_CHECK_ARG(ct3_in != ct_out,
                "b2f_relinearize_rescale: in-place operation is not supported");
  if (num_cts == 0) return B2F_OK;
  cudaStream_t s = (cudaStream_t)stream;
  Scratch sc{ctx, s};
  if ((rc = sc.init(ws, ws_bytes, rotate_workspace(ctx, num_cts, l)))) return rc;
  const LevelTables &T = ctx->levels[l];
  const int K = ctx->K, L = ctx->L, beta = T.beta, lk = l + K;
  uint64_t *xt = sc.take((size_t)num_cts * l * kN);
  uint64_t *ext = sc.take((size_t)num_cts * beta * lk * kN);
  uint64_t *acc = sc.take((size_t)num_cts * 2 * lk * kN);
  uint64_t *conv = sc.take((size_t)num_cts * 2 * l * kN);
  const long long s3 = 3LL * l * kN;
  const uint64_t *d2 = ct3_in + 2 * (size_t)l * kN;
  if ((rc = modup(ctx, d2, s3, num_cts, l, xt, ext, s))) return rc;
  ItemKeys it{};
  it.key[0] = relin_key;
  it.g[0] = 1u;
  it.shared = 1;
  if ((rc = launch_key_inner_product(ctx, num_cts, d2, s3, ext, (long long)beta * lk * kN,
                                     it, acc, l, s, ct3_in, ct3_in + (size_t)l * kN, s3)))
    return rc;
  // iNTT of the removed limbs of both polys, scaled by N^-1 (M/r)^-1
  std::vector<LimbJob> rj;
  for (int b = 0; b < 2; ++b)
    for (int r = 0; r <= K; ++r) {
      const uint32_t off = (uint32_t)(b * lk + l - 1 + r);
      rj.push_back(LimbJob{off, off, (uint16_t)(r ? L + r - 1 : l - 1), (uint16_t)r, 0});
    }
  const LimbJob *d = job_table(ctx, {7, l}, rj);
  if (!d) return B2F_ERR_NOMEM;
  const long long as = 2LL * lk * kN;
  if ((rc = launch_ntt(ctx, acc, as, acc, as, d, 2 * (K + 1), num_cts, 1,
                       T.mdr_scale, s)))
    return rc;
  if ((rc = launch_moddown_rescale_conv(ctx, acc, conv, l, num_cts, s))) return rc;
  // the subtrahend of the post-operation enters as the epilogue's add input
  // (its first l-1 limbs, each ciphertext 2 sub_limbs limbs apart)
  const uint64_t *s0 = sub, *s1 = sub ? sub + (size_t)sub_limbs * kN : nullptr;
  return ntt_moddown(ctx, conv, num_cts, l - 1, lk, acc, s0, s1,
                     sub ? 2LL * sub_limbs * kN : 0, ct_out, 2LL * (l - 1) * kN,
                     T.rescale_inv, it, s, nullptr, post);
}

size_t b2f_modup_batch_workspace(const b2f_context *ctx, int num_cts, int l) {
  if (!ctx || l < 1 || l > ctx->L || num_cts < 0) return 0;
  return rnd((size_t)std::max(num_cts, 1) * l * kN);
}

int b2f_modup_batch(b2f_context *ctx, const uint64_t *ct, int num_cts, int l,
                    uint64_t *ext, void *ws, size_t ws_bytes, void *stream) {
  B2F_RANGE("b2f_modup_batch");
  int rc = check_level(ctx, l, "b2f_modup");
  if (rc) return rc;
  B2F_CHECK_ARG(ct && ext && num_cts >= 0, "b2f_modup: null argument");
  if (!num_cts) return B2F_OK;
  cudaStream_t s = (cudaStream_t)stream;
  Scratch sc{ctx, s};
  if ((rc = sc.init(ws, ws_bytes, b2f_modup_batch_workspace(ctx, num_cts, l))))
    return rc;
  uint64_t *xt = sc.take((size_t)num_cts * l * kN);
  return modup(ctx, ct + (size_t)l * kN, 2LL * l * kN, num_cts, l, xt, ext, s);
}

size_t b2f_modup_workspace(const b2f_context *ctx, int l) {
  return b2f_modup_batch_workspace(ctx, 1, l);
}

int b2f_modup(b2f_context *ctx, const uint64_t *ct, int l, uint64_t *ext,
              void *ws, size_t ws_bytes, void *stream) {
  return b2f_modup_batch(ctx, ct, 1, l, ext, ws, ws_bytes, stream);
}

size_t b2f_rotate_hoisted_batch_workspace(const b2f_context *ctx, int num_cts,
                                          int count, int l) {
  if (!ctx || l < 1 || l > ctx->L || count < 0 || num_cts < 0) return 0;
  const long long items = std::max(1LL, (long long)num_cts * std::max(count, 1));
  return moddown_bytes(ctx, (int)std::min<long long>(items, kMaxItems), l);
}

size_t b2f_rotate_hoisted_workspace(const b2f_context *ctx, int count, int l) {
  return b2f_rotate_hoisted_batch_workspace(ctx, 1, count, l);
}

int b2f_rotate_hoisted_batch(b2f_context *ctx, const uint64_t *ct, int num_cts,
                             int l, const uint64_t *ext, int count,
                             const uint64_t *galois, const uint64_t *const *keys,
                             uint64_t *out, void *ws, size_t ws_bytes,
                             void *stream) {
  B2F_RANGE("b2f_rotate_hoisted_batch");
  int rc = check_level(ctx, l, "b2f_rotate_hoisted");
  if (rc) return rc;
  B2F_CHECK_ARG(ct && out && count >= 0 && num_cts >= 0 &&
                    (count == 0 || (galois && keys)),
                "b2f_rotate_hoisted: null argument");
  bool need_ext = false;
  for (int r = 0; r < count; ++r) {
    B2F_CHECK_ARG(valid_galois(galois[r]),
                  "b2f_rotate_hoisted: bad galois element %llu",
                  (unsigned long long)galois[r]);
    if (galois[r] != 1) {
      B2F_CHECK_ARG(keys[r], "b2f_rotate_hoisted: key %d is null", r);
      need_ext = true;
    }
  }
  B2F_CHECK_ARG(!need_ext || ext, "b2f_rotate_hoisted: ModUp digits are null");
  if (!num_cts || !count) return B2F_OK;
  cudaStream_t s = (cudaStream_t)stream;
  Scratch sc{ctx, s};
  if ((rc = sc.init(ws, ws_bytes,
                    b2f_rotate_hoisted_batch_workspace(ctx, num_cts, count, l))))
    return rc;
  const int lk = l + ctx->K;
  const long long items_max =
      std::min<long long>((long long)num_cts * count, kMaxItems);
  uint64_t *acc = sc.take((size_t)items_max * 2 * lk * kN);
  uint64_t *conv = sc.take((size_t)items_max * 2 * l * kN);
  const long long cs = 2LL * l * kN;                 // one ciphertext
  const long long ocs = (long long)count * cs;       // one ciphertext's outputs
  const long long es = (long long)ctx->levels[l].beta * lk * kN;
  // identity items are copies; the keyed rotations go through the key switch
  // in launch groups of up to kMaxItems (rotations x ciphertexts)
  std::vector<int> keyed;
  for (int r = 0; r < count; ++r) {
    if (galois[r] == 1) {
      for (int c = 0; c < num_cts; ++c)
        B2F_CUDA(cudaMemcpyAsync(out + c * ocs + (size_t)r * cs, ct + c * cs,
                                 cs * 8, cudaMemcpyDeviceToDevice, s));
    } else {
      keyed.push_back(r);
    }
  }
  // A launch group takes up to 16 ciphertexts and as many rotations as fit
  // in kMaxItems items (ciphertext-major: the items of one ciphertext share
  // its digits, and the same rotation of the group's ciphertexts follows
  // within kMaxItems items, while its key limbs are still in L2): each
  // rotation key streams from HBM once per group of ciphertexts, not once per
  // ciphertext (at l = 13, 16 ciphertexts x 63 rotations: 2.6 GB of key
  // limbs instead of 42 GB).
  const int cgroup = std::min(num_cts, 16);
  const int rblock = std::max(1, kMaxItems / std::max(cgroup, 1));
  for (size_t p = 0; p < keyed.size(); p += rblock) {
    const int R = (int)std::min<size_t>(rblock, keyed.size() - p);
    ItemKeys it{};
    it.shared = 0;
    it.per = R;
    it.out_ct_stride = ocs;
    for (int i = 0; i < R; ++i) {
      it.key[i] = keys[keyed[p + i]];
      it.g[i] = (uint32_t)galois[keyed[p + i]];
      it.pos[i] = (int16_t)(keyed[p + i] - keyed[p]);
    }
    const int group = std::max(1, kMaxItems / R);  // ciphertexts per launch group
    for (int c0 = 0; c0 < num_cts; c0 += group) {
      const int nc = std::min(group, num_cts - c0);
      rc = ip_moddown(ctx, ct + c0 * cs + (size_t)l * kN, cs, ext + c0 * es, es,
                      nc * R, l, it, ct + c0 * cs, nullptr, cs,
                      out + c0 * ocs + (size_t)keyed[p] * cs, cs, acc, conv, s);
      if (rc) return rc;
    }
  }
  return B2F_OK;
}

int b2f_rotate_hoisted(b2f_context *ctx, const uint64_t *ct, int l,
                       const uint64_t *ext, int count, const uint64_t *galois,
                       const uint64_t *const *keys, uint64_t *out, void *ws,
                       size_t ws_bytes, void *stream) {
  return b2f_rotate_hoisted_batch(ctx, ct, 1, l, ext, count, galois, keys, out,
                                  ws, ws_bytes, stream);
}

size_t b2f_rotate_hoisted_ext_workspace(const b2f_context *ctx, int count, int l) {
  if (!ctx || l < 1 || l > ctx->L || count < 0) return 0;
  return rnd((size_t)std::max(1, std::min(count, kMaxItems)) * 2 * (l + ctx->K) * kN);
}

int b2f_rotate_hoisted_ext(b2f_context *ctx, const uint64_t *ct, int l,
                           const uint64_t *ext, int count, const uint64_t *galois,
                           const uint64_t *const *keys, uint64_t *out, void *ws,
                           size_t ws_bytes, void *stream) {
  B2F_RANGE("b2f_rotate_hoisted_ext");
  int rc = check_level(ctx, l, "b2f_rotate_hoisted_ext");
  if (rc) return rc;
  B2F_CHECK_ARG(ct && out && count >= 0 && (count == 0 || galois),
                "b2f_rotate_hoisted_ext: null argument");
  bool need_ext = false;
  for (int r = 0; r < count; ++r) {
    B2F_CHECK_ARG(valid_galois(galois[r]),
                  "b2f_rotate_hoisted_ext: bad galois element %llu",
                  (unsigned long long)galois[r]);
    if (galois[r] != 1) {
      B2F_CHECK_ARG(keys && keys[r], "b2f_rotate_hoisted_ext: key %d is null", r);
      need_ext = true;
    }
  }
  B2F_CHECK_ARG(!need_ext || ext, "b2f_rotate_hoisted_ext: ModUp digits are null");
  cudaStream_t s = (cudaStream_t)stream;
  Scratch sc{ctx, s};
  if ((rc = sc.init(ws, ws_bytes, b2f_rotate_hoisted_ext_workspace(ctx, count, l))))
    return rc;
  const int K = ctx->K, lk = l + K;
  const int chunk = std::max(1, std::min(count, kMaxItems));
  uint64_t *acc = sc.take((size_t)chunk * 2 * lk * kN);
  const LevelTables &T = ctx->levels[l];
  for (int p = 0; p < count; p += kMaxItems) {
    const int n = std::min(kMaxItems, count - p);
    ItemKeys it{};
    ExtItems ex{};
    int keyed = 0;
    for (int i = 0; i < n; ++i) {
      ex.g[i] = (uint32_t)galois[p + i];
      ex.slot[i] = -1;
      if (galois[p + i] != 1) {
        it.key[keyed] = keys[p + i];
        it.g[keyed] = (uint32_t)galois[p + i];
        it.pos[keyed] = (int16_t)i;
        ex.slot[i] = (int16_t)keyed++;
      }
    }
    uint64_t *outp = out + (size_t)p * 2 * lk * kN;
    const bool fold = !ctx->fp64;  // the automorphism and P c0 in the key IP's store
    if (keyed) {
      it.shared = 0;
      it.per = keyed;  // one ciphertext: item i is keyed rotation i
      it.out_ct_stride = 0;
      if (fold) {
        ChainStep cs_{};
        cs_.x = ct;  // P c0 on the Q limbs
        cs_.x_q = 1;
        cs_.out = outp;
        if ((rc = launch_key_inner_product_chain(ctx, keyed, ct + (size_t)l * kN, 0, ext, 0,
                                                 it, l, cs_, s)))
          return rc;
      } else if ((rc = launch_key_inner_product(ctx, keyed, ct + (size_t)l * kN, 0, ext, 0,
                                                it, acc, l, s))) {
        return rc;
      }
    }
    if (!fold || keyed < n) {
      ext_combine_kernel<<<dim3(kN / TPB, lk, 2 * n), TPB, 0, s>>>(
          acc, ct, outp, ctx->d_mod, ctx->d_pmod, l, K, ctx->L, ex, fold ? 1 : 0);
      B2F_LAUNCHED("ext_combine_kernel");
    }
  }
  return B2F_OK;
}

size_t b2f_moddown_ext_workspace(const b2f_context *ctx, int num_cts, int l) {
  if (!ctx || l < 1 || l > ctx->L || num_cts < 0) return 0;
  return moddown_bytes(ctx, num_cts, l);
}

int b2f_moddown_ext(b2f_context *ctx, const uint64_t *in, int num_cts, int l,
                    uint64_t *out, void *ws, size_t ws_bytes, void *stream) {
  B2F_RANGE("b2f_moddown_ext");
  int rc = check_level(ctx, l, "b2f_moddown_ext");
  if (rc) return rc;
  B2F_CHECK_ARG(in && out && num_cts >= 0, "b2f_moddown_ext: null argument");
  if (!num_cts) return B2F_OK;
  cudaStream_t s = (cudaStream_t)stream;
  Scratch sc{ctx, s};
  if ((rc = sc.init(ws, ws_bytes, moddown_bytes(ctx, num_cts, l)))) return rc;
  const int K = ctx->K, lk = l + K;
  uint64_t *pcoef = sc.take((size_t)num_cts * 2 * lk * kN);  // P limbs only
  uint64_t *conv = sc.take((size_t)num_cts * 2 * l * kN);
  std::vector<LimbJob> pj;
  for (int b = 0; b < 2; ++b)
    for (int k = 0; k < K; ++k) {
      uint32_t off = (uint32_t)(b * lk + l + k);
      pj.push_back(LimbJob{off, off, (uint16_t)(ctx->L + k), (uint16_t)k, 0});
    }
  const LimbJob *d = job_table(ctx, {3, l}, pj);
  if (!d) return B2F_ERR_NOMEM;
  const long long as = 2LL * lk * kN;
  if ((rc = launch_ntt(ctx, in, as, pcoef, as, d, 2 * K, num_cts, 1,
                       ctx->d_moddown_scale, s)))
    return rc;
  if (ctx->fp64 && ctx->d_md_conv_f64)
    return ntt_moddown(ctx, conv, num_cts, l, lk, in, nullptr, nullptr, 0, out,
                       2LL * l * kN, nullptr, ItemKeys{{}, {1u}, {}, 1}, s, pcoef);
  if ((rc = launch_moddown_conv(ctx, pcoef, conv, l, num_cts, s))) return rc;
  return ntt_moddown(ctx, conv, num_cts, l, lk, in, nullptr, nullptr, 0, out, 2LL * l * kN,
                     nullptr, ItemKeys{{}, {1u}, {}, 1}, s);
}

size_t b2f_giant_chain_workspace(const b2f_context *ctx, int num_cts, int l) {
  if (!ctx || l < 1 || l > ctx->L || num_cts < 0) return 0;
  return giant_chain_workspace(ctx, std::max(num_cts, 1), l);
}

int b2f_giant_chain(b2f_context *ctx, const uint64_t *sums, int extended, int num_cts,
                    int giant_count, int l, uint64_t giant_galois, const uint64_t *giant_key,
                    uint64_t *out, void *ws, size_t ws_bytes, void *stream) {
  B2F_RANGE("b2f_giant_chain");
  int rc = check_level(ctx, l, "b2f_giant_chain");
  if (rc) return rc;
  B2F_CHECK_ARG(sums && out && num_cts >= 0 && giant_count >= 1 &&
                    (extended == 0 || extended == 1),
                "b2f_giant_chain: bad argument");
  B2F_CHECK_ARG(giant_count == 1 || giant_key,
                "b2f_giant_chain: giant_count > 1 needs the giant rotation key");
  if (!num_cts) return B2F_OK;
  cudaStream_t s = (cudaStream_t)stream;
  const long long limbs = extended ? l + ctx->K : l, gs = 2 * limbs * kN;
  if (giant_count == 1) {
    if (extended) return b2f_moddown_ext(ctx, sums, num_cts, l, out, ws, ws_bytes, stream);
    B2F_CUDA(cudaMemcpyAsync(out, sums, (size_t)num_cts * gs * 8, cudaMemcpyDeviceToDevice, s));
    return B2F_OK;
  }
  return giant_chain_ext(ctx, sums, extended, gs, gs * giant_count, num_cts, giant_count, l,
                         giant_galois, giant_key, out, ws, ws_bytes, s);
}

int b2f_automorphism(b2f_context *ctx, const uint64_t *in, uint64_t *out,
                     int num_polys, int limbs, uint64_t galois, void *stream) {
  B2F_CHECK_ARG(ctx && in && out && num_polys >= 0 && limbs >= 0,
                "b2f_automorphism: bad argument");
  B2F_CHECK_ARG(valid_galois(galois), "b2f_automorphism: bad galois element");
  B2F_CHECK_ARG(in != out, "b2f_automorphism: in-place is not supported");
  if (!num_polys || !limbs) return B2F_OK;
  automorphism_kernel<<<dim3(kN / TPB, num_polys * limbs), TPB, 0,
                        (cudaStream_t)stream>>>(in, out, (uint32_t)galois);
  B2F_LAUNCHED("automorphism_kernel");
  return B2F_OK;
}

}  // extern "C"
