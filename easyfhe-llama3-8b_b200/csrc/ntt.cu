// Batched negacyclic NTT / inverse NTT for N = 2^16 on sm_100a.
//
// One thread-block cluster of 16 CTAs owns one limb (2^16 words = 512 KiB):
// the limb is read from HBM once and written once, and everything in between
// stays on chip.  Seen as a 16 x 4096 matrix (element g = 4096 r + c), the
// forward transform (Cooley-Tukey, natural order in, bit-reversed out):
//   1. each thread takes one column c (the 16 rows at stride 4096, straight
//      from HBM) and runs stages 0-3 on it as a radix-16 step in registers;
//   2. row r of every column goes to CTA r through distributed shared memory,
//      so CTA r then holds the contiguous block [4096 r, 4096 (r+1));
//   3. stages 4-15 run in three radix-16 register passes over the block:
//      stride 256 (CTA-wide), stride 16 (each half-warp owns a 256-word
//      segment, so only warp synchronisation is needed) and stride 1 (a
//      thread's 16 consecutive words, entirely in registers);
//   4. each thread writes its 16 consecutive outputs with 16-byte stores.
// 256 threads x 16 words per CTA and 64 registers give four CTAs per SM.
// The inverse (Gentleman-Sande, bit-reversed in, natural out) runs the same
// steps backwards and folds N^-1 (times an optional per-limb constant) into
// the final stage.  The butterfly arithmetic is a policy (ntt_arith.cuh):
// 64-bit integer Shoup products with Harvey's lazy reduction, or, when every
// prime is below 2^50, exact binary64 products on signed residues, which this
// GPU issues at a higher rate.  Outputs are fully reduced either way.
// Shared memory holds the block padded by one word per 16 (pad(e) = e + e/16),
// which keeps all three pass patterns and both cluster exchanges free of bank
// conflicts; the passes address it and the twiddle tables as per-pass bases
// plus immediate offsets.  Cluster barriers are split-phase, their latency
// hidden behind loads and butterflies.
// The forward transform that finishes a ModDown (or a rescale) in its
// epilogue keeps 8-CTA clusters of 512 threads: with its extra input and
// epilogue traffic that shape measured faster (namespace md below).
#include <cooperative_groups.h>

#include <atomic>

#include "b2f_internal.h"
#include "ksitems.cuh"
#include "ntt_arith.cuh"

namespace cg = cooperative_groups;

namespace b2f {
namespace {

constexpr int CL = 16;                      // CTAs per cluster = per limb
constexpr int BLK = kN / CL;                // 4096 words per CTA
constexpr int NT = 256;                     // threads per CTA, 16 words each
constexpr int SMEM_BYTES = (BLK + BLK / 16) * 8;  // 34816

// one pad word per 16 keeps every access pattern free of bank conflicts
__device__ __forceinline__ int pad(int e) { return e + (e >> 4); }

// 32-byte accesses (one full sector per lane; the launch checks the 32-byte
// alignment of the limbs): a thread's 16 consecutive words in four requests,
// neither sector half requested twice
__device__ __forceinline__ void ld32(const uint64_t *p, uint64_t (&w)[4]) {
  asm volatile("ld.global.v4.u64 {%0, %1, %2, %3}, [%4];"
               : "=l"(w[0]), "=l"(w[1]), "=l"(w[2]), "=l"(w[3])
               : "l"(p));
}
__device__ __forceinline__ void st32(uint64_t *p, uint64_t a, uint64_t b, uint64_t c,
                                     uint64_t d) {
  asm volatile("st.global.v4.u64 [%0], {%1, %2, %3, %4};" ::"l"(p), "l"(a), "l"(b), "l"(c),
               "l"(d)
               : "memory");
}

struct NttParams {
  const uint64_t *in;
  uint64_t *out;
  const LimbJob *jobs;
  long long in_stride, out_stride;
  const void *tw;            // [prime][N]: ulonglong2 (integer) or double
  const uint64_t *primes;
  const double *qinv;        // binary64 arithmetic only
  const ulonglong2 *scales;  // inverse only
  int jobs_per_item;
  int items;
};

// Twiddles: stage s of element j uses entry 2^s + j / 2^(16-s) of the
// prime's table (psi powers in bit-reversed order).

// Four CT stages s0..s0+3 on 16 registers with element index
// j(k) = base + k * stride; at local stage t the pairs are (k, k + d),
// d = 8 >> t, and each block of 2d registers shares one twiddle.  For the
// four steps' (base, stride) the stage-s index splits without carry:
// (base + blk stride) >> (16 - s) = (base >> (16 - s)) + (blk stride >> (16 - s)),
// so each twiddle is a per-stage base plus a constant offset.
template <class A>
__device__ __forceinline__ void ct_pass(const A &ar, typename A::V (&x)[16],
                                        const typename A::W *tw, int s0, int base,
                                        int stride) {
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    const int d = 8 >> t, sh = kLogN - (s0 + t);
    const typename A::W *tws = tw + (1 << (s0 + t)) + (base >> sh);
#pragma unroll
    for (int blk = 0; blk < 16; blk += 2 * d) {
      const typename A::W w = A::ldtw(tws, (blk * stride) >> sh);
#pragma unroll
      for (int k = blk; k < blk + d; ++k) ct_bfly(ar, x[k], x[k + d], w);
    }
  }
}

// GS stages s0+3 down to s0+TMIN (the inverse order)
template <class A, int TMIN>
__device__ __forceinline__ void gs_pass(const A &ar, typename A::V (&x)[16],
                                        const typename A::W *tw, int s0, int base,
                                        int stride) {
#pragma unroll
  for (int t = 3; t >= TMIN; --t) {
    const int d = 8 >> t, sh = kLogN - (s0 + t);
    const typename A::W *tws = tw + (1 << (s0 + t)) + (base >> sh);
#pragma unroll
    for (int blk = 0; blk < 16; blk += 2 * d) {
      const typename A::W w = A::ldtw(tws, (blk * stride) >> sh);
#pragma unroll
      for (int k = blk; k < blk + d; ++k) gs_bfly(ar, x[k], x[k + d], w);
    }
  }
}

// The stride-1 pass (stages s0..s0+3 on a thread's 16 consecutive elements
// from base, a multiple of 16): stage s0 + t uses 2^t consecutive table
// entries starting at 2^(s0+t) + base / 2^(16-s0-t), which are loaded four
// (or two) at a time with vector loads, each lane taking whole sectors
// instead of one word of each of several sectors per instruction.
template <class A, bool INV>
__device__ __forceinline__ void pass1(const A &ar, typename A::V (&x)[16],
                                      const typename A::W *tw, int s0, int base) {
  using W = typename A::W;
  auto bfly = [&](int k, int d, W w) {
    if constexpr (INV)
      gs_bfly(ar, x[k], x[k + d], w);
    else
      ct_bfly(ar, x[k], x[k + d], w);
  };
  auto stage = [&](int t) {
    const int d = 8 >> t, sh = kLogN - (s0 + t);
    const W *tws = tw + (1 << (s0 + t)) + (base >> sh);
    if (t == 0) {
      const W w = A::ldtw(tws, 0);
#pragma unroll
      for (int k = 0; k < 8; ++k) bfly(k, 8, w);
    } else if (t == 1) {
      W w[2];
      A::ldtw2(tws, w);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        bfly(k, 4, w[0]);
        bfly(8 + k, 4, w[1]);
      }
    } else {
      // 4 or 8 twiddles, four at a time: block b of 2d registers uses w[b]
#pragma unroll
      for (int q = 0; q < (1 << t); q += 4) {
        W w[4];
        A::ldtw4(tws + q, w);
#pragma unroll
        for (int b = 0; b < 4; ++b)
#pragma unroll
          for (int k = 0; k < d; ++k) bfly((q + b) * 2 * d + k, d, w[b]);
      }
    }
  };
  if constexpr (INV) {
#pragma unroll
    for (int t = 3; t >= 0; --t) stage(t);
  } else {
#pragma unroll
    for (int t = 0; t < 4; ++t) stage(t);
  }
}

// Register passes over a CTA's block (element e of the block, 16 per thread):
//   A: e = tid + 256 k                    (pad: +272 k)
//   B: e = 256 (tid/16) + tid%16 + 16 k   (pad: +17 k; a half-warp's segment)
//   C: e = 16 tid + k                     (pad: +k; the same segment)

template <class A>
__global__ void __cluster_dims__(CL, 1, 1) __launch_bounds__(NT, 4)
    ntt_fwd_kernel(NttParams P) {
  using V = typename A::V;
  using W = typename A::W;
  extern __shared__ __align__(16) uint64_t buf[];
  V *vb = reinterpret_cast<V *>(buf);
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int tid = threadIdx.x;
  // job-major order: consecutive clusters transform the same limb job (one
  // prime) of consecutive items, so clusters running together share one
  // twiddle table in L2
  const long long job_id = blockIdx.x / CL;
  const long long item = job_id % P.items;
  const LimbJob job = P.jobs[job_id / P.items];
  const uint64_t *a = P.in + item * P.in_stride + (long long)job.in_off * kN;
  uint64_t *o = P.out + item * P.out_stride + (long long)job.out_off * kN;
  const A ar(P.primes, P.qinv, job.prime);
  const W *tw = static_cast<const W *>(P.tw) + (size_t)job.prime * kN;
  const int jb = rank * BLK;
  // split-phase cluster barrier: arriving now and waiting just before the
  // first remote shared-memory write certifies that every CTA of the cluster
  // is resident, with the barrier's latency hidden behind the loads and
  // stages 0-3 (nothing needs publishing yet, so the arrive is relaxed)
  asm volatile("barrier.cluster.arrive.relaxed.aligned;\n" ::: "memory");
  // stages 0-3 on column col (rows r at stride 4096), straight from HBM
  const int col = rank * 256 + tid;
  V x[16];
#pragma unroll
  for (int r = 0; r < 16; ++r) x[r] = A::from_word(a[r * BLK + col]);
  ct_pass(ar, x, tw, 0, col, BLK);
  asm volatile("barrier.cluster.wait.aligned;\n" ::: "memory");
  // row r of this column goes to CTA r, position col of its block
#pragma unroll
  for (int r = 0; r < 16; ++r) cluster.map_shared_rank(vb, r)[pad(col)] = x[r];
  cluster.sync();
  {
    V *p = vb + pad(tid);
#pragma unroll
    for (int k = 0; k < 16; ++k) x[k] = p[272 * k];
    ct_pass(ar, x, tw, 4, jb + tid, 256);
#pragma unroll
    for (int k = 0; k < 16; ++k) p[272 * k] = x[k];
  }
  __syncthreads();
  {
    const int e0 = 256 * (tid >> 4) + (tid & 15);
    V *p = vb + pad(e0);
#pragma unroll
    for (int k = 0; k < 16; ++k) x[k] = p[17 * k];
    ct_pass(ar, x, tw, 8, jb + e0, 16);
#pragma unroll
    for (int k = 0; k < 16; ++k) p[17 * k] = x[k];
  }
  __syncwarp();
  {
    const V *p = vb + pad(16 * tid);
#pragma unroll
    for (int k = 0; k < 16; ++k) x[k] = p[k];
  }
  pass1<A, false>(ar, x, tw, 12, jb + 16 * tid);
  // x[k] is element 16 tid + k of the block: 32-byte stores
  o += jb + 16 * tid;
#pragma unroll
  for (int m = 0; m < 4; ++m)
    st32(o + 4 * m, A::to_word(ar.full(x[4 * m])), A::to_word(ar.full(x[4 * m + 1])),
         A::to_word(ar.full(x[4 * m + 2])), A::to_word(ar.full(x[4 * m + 3])));
}

template <class A>
__global__ void __cluster_dims__(CL, 1, 1) __launch_bounds__(NT, 4)
    ntt_inv_kernel(NttParams P) {
  using V = typename A::V;
  using W = typename A::W;
  extern __shared__ __align__(16) uint64_t buf[];
  V *vb = reinterpret_cast<V *>(buf);
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int tid = threadIdx.x;
  // job-major order, as the forward
  const long long job_id = blockIdx.x / CL;
  const long long item = job_id % P.items;
  const LimbJob job = P.jobs[job_id / P.items];
  const uint64_t *a = P.in + item * P.in_stride + (long long)job.in_off * kN;
  uint64_t *o = P.out + item * P.out_stride + (long long)job.out_off * kN;
  const A ar(P.primes, P.qinv, job.prime);
  const W *tw = static_cast<const W *>(P.tw) + (size_t)job.prime * kN;
  const int jb = rank * BLK;
  V x[16];
  // stages 15-12 on the thread's 16 consecutive words, straight from HBM
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    uint64_t w[4];
    ld32(a + jb + 16 * tid + 4 * m, w);
#pragma unroll
    for (int u = 0; u < 4; ++u) x[4 * m + u] = A::from_word(w[u]);
  }
  pass1<A, true>(ar, x, tw, 12, jb + 16 * tid);
  {
    V *p = vb + pad(16 * tid);
#pragma unroll
    for (int k = 0; k < 16; ++k) p[k] = x[k];
  }
  __syncwarp();
  {
    const int e0 = 256 * (tid >> 4) + (tid & 15);
    V *p = vb + pad(e0);
#pragma unroll
    for (int k = 0; k < 16; ++k) x[k] = p[17 * k];
    gs_pass<A, 0>(ar, x, tw, 8, jb + e0, 16);
#pragma unroll
    for (int k = 0; k < 16; ++k) p[17 * k] = x[k];
  }
  __syncthreads();
  {
    const V *p = vb + pad(tid);
#pragma unroll
    for (int k = 0; k < 16; ++k) x[k] = p[272 * k];
  }
  // split-phase: this thread's reads of its block are done (release); the
  // wait after stages 7-4 means every CTA has finished reading its block
  asm volatile("barrier.cluster.arrive.aligned;\n" ::: "memory");
  gs_pass<A, 0>(ar, x, tw, 4, jb + tid, 256);
  asm volatile("barrier.cluster.wait.aligned;\n" ::: "memory");
  // element tid + 256 k of row `rank` is column tid + 256 k: CTA k keeps it
  // at [row rank][column tid]
#pragma unroll
  for (int k = 0; k < 16; ++k) cluster.map_shared_rank(vb, k)[pad(rank * 256 + tid)] = x[k];
  cluster.sync();
  const int col = rank * 256 + tid;
#pragma unroll
  for (int r = 0; r < 16; ++r) x[r] = vb[pad(r * 256 + tid)];
  gs_pass<A, 1>(ar, x, tw, 0, col, BLK);  // stages 3-1
  {
    const W w = A::ldtw(tw, 1);
    const W sc = A::scale(P.scales[job.scale_idx]);
    if constexpr (A::kFoldScale) {
      // stage 0 with the output scale folded in: ((x + y) s, (x - y) w s)
      const W wsc = ar.fold(w, sc);
#pragma unroll
      for (int k = 0; k < 8; ++k) ar.gs_scaled(x[k], x[k + 8], sc, wsc);
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) gs_bfly(ar, x[k], x[k + 8], w);
#pragma unroll
      for (int k = 0; k < 16; ++k) x[k] = ar.scale_out(x[k], sc);
    }
  }
#pragma unroll
  for (int r = 0; r < 16; ++r) o[r * BLK + col] = A::to_word(x[r]);
}

// The forward transform as the last step of a ModDown (the NTT of the P part
// converted to Q), its epilogue finishing the ModDown: for item it (poly
// p = 2 it + b, limb i) and every evaluation j of the limb,
//   out_b[i][dst(j)] = (acc_b[i][j] - v[j]) * [P^-1]_{q_i} (* qinv_i) + add_b[i][j]
// with dst = the slot permutation of X -> X^(g^-1) (the inverse of the
// gather out[k] = w[src_g(k)]).  Each warp walks its own 512 evaluations in
// lane-interleaved pairs (coalesced reads of acc and add); a pair j, j + 1
// (j even) lands on one aligned pair of words, since bit-reversing j + 1 adds
// 2^16 to the exponent 2 brv(j) + 1, which an odd g keeps at 2^16 modulo 2^17,
// so the source indices differ in bit 0 only: one 16-byte store per pair,
// and the 32 stores of a warp land in one aligned 64-word block.  The
// converted limbs never reach HBM.
struct ModDownOut {
  const uint64_t *acc;          // [item][2][lk][N]
  const uint64_t *add0, *add1;  // [ct][..][N] at add_stride, or null
  long long add_stride;
  uint64_t *out;                // items.out(it, out_stride) + (b l_out + i) N
  long long out_stride;
  const ulonglong2 *pinv;       // [P^-1] mod q_i
  const ulonglong2 *qinv;       // a second factor mod q_i, or null
  const uint64_t *primes;
  ItemKeys items;
  int lk, l_out;
  // binary64 only, zK > 0: the transform's input is the ModDown conversion
  // itself, sum_k z_k [Phat_k]_{q_i} with z the K scaled P limbs of item it,
  // poly b (limbs l_out .. l_out + zK - 1 of z [item][2][lk][N]); zconv
  // [i][zK] the constants as doubles.  Replaces the conversion kernel and its
  // round trip through HBM when K is small.
  const uint64_t *z;
  const double *zconv;
  int zK;
  // rescale (lift != 0): the input is the centred lift of the last limb's
  // coefficients zlast [item][N] (below q_last) modulo q_i, and the epilogue
  // with pinv = [q_last^-1]_{q_i} and acc = the input ciphertext gives the
  // rescaled limb: (c_i - NTT(lift)) q_last^-1
  int lift;
  const uint64_t *zlast;
  const uint64_t *qlast_mod;  // [q_last]_{q_i}
  uint64_t q_last;
  const Mod *mods;
  // post-operation (EpiPostOp): x2, subtract add_b, add cadd[i] to poly 0
  int dbl, add_neg, has_cadd;
  uint64_t cadd[64];
  // 1: the transform's items are the second polys of acc's items only (item
  // it = transform item, b = 1), written as single polys: out(it) + i N
  int one_poly = 0;
};

// The forward transform that finishes a ModDown runs on clusters of 8 CTAs
// of 512 threads (8192 words per CTA, two CTAs per SM), which measured
// faster than 16-CTA clusters for this kernel's larger input and epilogue
// traffic.  Stages 0-2 run on two columns of 8 rows per thread before the
// cluster exchange, stages 3-15 in three register passes, the last stage
// across lane pairs tid, tid^1.
namespace md {

constexpr int CL = 8;                       // CTAs per cluster = per limb
constexpr int BLK = kN / CL;                // 8192 words per CTA
constexpr int NT = 512;                     // threads per CTA, 16 words each
constexpr int SEG = 512;                    // words owned by one warp in B/C
constexpr int SMEM_BYTES = (BLK + 2 * (BLK / 32)) * 8;  // 69632

// two pad words per 32 keep every pass free of shared-memory bank conflicts
__device__ __forceinline__ int pad(int l) { return l + ((l >> 5) << 1); }

// pad(l + STRIDE k) = pad(l) + pad_step<STRIDE>() k for k < 16: exact when
// STRIDE is a multiple of 32 (each step adds STRIDE / 32 blocks), or when
// l's offset in its 32-word block plus 15 STRIDE stays inside the block (pass
// C: STRIDE 2, l mod 32 <= 1).  The accesses then use immediate offsets.
template <int STRIDE>
__device__ constexpr int pad_step() {
  return STRIDE % 32 == 0 ? STRIDE + STRIDE / 16 : STRIDE;
}
template <int STRIDE, class V>
__device__ __forceinline__ void load16(V (&x)[16], const V *buf, int l) {
  const V *p = buf + pad(l);
#pragma unroll
  for (int k = 0; k < 16; ++k) x[k] = p[pad_step<STRIDE>() * k];
}
template <int STRIDE, class V>
__device__ __forceinline__ void store16(const V (&x)[16], V *buf, int l) {
  V *p = buf + pad(l);
#pragma unroll
  for (int k = 0; k < 16; ++k) p[pad_step<STRIDE>() * k] = x[k];
}

// Passes over a CTA's block (element l = base + stride k):
//   A: stages 3-6,   base tid,                        stride 512 (CTA-wide)
//   B: stages 7-10,  base (tid/32)*512 + tid%32,      stride 32
//   C: stages 11-14, base (tid/2)*32 + tid%2,         stride 2, then stage 15
//      across lanes tid, tid^1.
// Warp w touches only words [512 w, 512 w + 512) in B and C, so the B <-> C
// exchange and the output staging need only warp synchronisation.

template <class A>
__global__ void __cluster_dims__(CL, 1, 1) __launch_bounds__(NT, 2)
    ntt_moddown_kernel(NttParams P, ModDownOut epi) {
  using V = typename A::V;
  using W = typename A::W;
  extern __shared__ __align__(16) uint64_t buf[];
  V *vb = reinterpret_cast<V *>(buf);
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // when every limb of an item reads the same input (the K scaled P words of
  // the in-transform conversion, or the last limb of a rescale), item-major
  // order: the clusters of one item run together and that input stays in L2
  // (job-major, it is evicted between an item's limbs); otherwise job-major,
  // so clusters running together share one twiddle table
  const long long job_id = blockIdx.x / CL;
  const bool item_major = epi.zK > 0 || epi.lift;
  const long long item = item_major ? job_id / P.jobs_per_item : job_id % P.items;
  const LimbJob job = P.jobs[item_major ? job_id % P.jobs_per_item : job_id / P.items];
  const uint64_t *a = P.in + item * P.in_stride + (long long)job.in_off * kN;
  const A ar(P.primes, P.qinv, job.prime);
  const W *tw = static_cast<const W *>(P.tw) + (size_t)job.prime * kN;

  {
    // the epilogue's inputs for this CTA's block: into L2 while the
    // transform runs (bulk prefetch, 64 KiB per array)
    if (tid == 0) {
      const int it = epi.one_poly ? (int)item : (int)(item >> 1);
      const int b = epi.one_poly ? 1 : (int)(item & 1), i = (int)job.out_off;
      const uint64_t *accl =
          epi.acc + (((size_t)it * 2 + b) * epi.lk + i) * kN + (size_t)rank * BLK;
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(accl), "r"(BLK * 8)
                   : "memory");
      const uint64_t *addl = b ? epi.add1 : epi.add0;
      if (addl) {
        addl += epi.items.ct(it) * epi.add_stride + (size_t)i * kN + (size_t)rank * BLK;
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(addl), "r"(BLK * 8)
                     : "memory");
      }
    }
  }
  // split-phase cluster barrier: arriving now and waiting just before the
  // first remote shared-memory write certifies that every CTA of the cluster
  // is resident, with the barrier's latency hidden behind the loads and
  // stages 0-2 (nothing needs publishing yet, so the arrive is relaxed)
  asm volatile("barrier.cluster.arrive.relaxed.aligned;\n" ::: "memory");
  V x[16];
  // stages 0-2 on columns c0, c0+1 (rows k at stride 8192), straight from HBM
  const int c0 = rank * 1024 + 2 * tid;
  bool converted = false;
  {
    if (epi.lift) {
      const int i = (int)job.out_off;
      const uint64_t *zb = epi.zlast + item * kN + c0;
      const uint64_t half = (epi.q_last - 1) / 2;
      if constexpr (A::kFoldScale) {  // binary64: signed lift, then |x| <= q_i/2
        const double ql = A::from_word(epi.q_last);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const ulonglong2 v = *reinterpret_cast<const ulonglong2 *>(zb + k * BLK);
          x[k] = ar.red(v.x > half ? __dadd_rn(A::from_word(v.x), -ql) : A::from_word(v.x));
          x[8 + k] =
              ar.red(v.y > half ? __dadd_rn(A::from_word(v.y), -ql) : A::from_word(v.y));
        }
      } else {  // integer: z mod q_i, minus q_last for the upper half
        const Mod M = epi.mods[i];
        const uint64_t qm = epi.qlast_mod[i];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const ulonglong2 v = *reinterpret_cast<const ulonglong2 *>(zb + k * BLK);
          uint64_t r0 = reduce128(0, v.x, M), r1 = reduce128(0, v.y, M);
          if (v.x > half) r0 = sub_mod(r0, qm, M.q);
          if (v.y > half) r1 = sub_mod(r1, qm, M.q);
          x[k] = A::from_word(r0);
          x[8 + k] = A::from_word(r1);
        }
      }
      converted = true;
    }
  }
  if constexpr (A::kFoldScale) {
    if (!converted && epi.zK > 0) {
      // x = sum_k z_k c_{i,k}: K exact products (|.| <= q each, sum below
      // 2^52 for K <= 4), reduced to |x| <= q/2 before the first stage
      const int it = epi.one_poly ? (int)item : (int)(item >> 1);
      const int b = epi.one_poly ? 1 : (int)(item & 1), i = (int)job.out_off;
      const uint64_t *zb = epi.z + (((size_t)it * 2 + b) * epi.lk + epi.l_out) * kN + c0;
#pragma unroll
      for (int k = 0; k < 16; ++k) x[k] = 0.0;
      for (int kk = 0; kk < epi.zK; ++kk) {
        const double c = __ldg(epi.zconv + (size_t)i * epi.zK + kk);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const ulonglong2 v =
              *reinterpret_cast<const ulonglong2 *>(zb + (size_t)kk * kN + k * BLK);
          x[k] = __dadd_rn(x[k], ar.mul(A::from_word(v.x), c));
          x[8 + k] = __dadd_rn(x[8 + k], ar.mul(A::from_word(v.y), c));
        }
      }
#pragma unroll
      for (int k = 0; k < 16; ++k) x[k] = ar.red(x[k]);
      converted = true;
    }
  }
  if (!converted) {
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const ulonglong2 v = *reinterpret_cast<const ulonglong2 *>(a + c0 + k * BLK);
      x[k] = A::from_word(v.x);
      x[8 + k] = A::from_word(v.y);
    }
  }
  {
    // stage by stage over both columns, one twiddle live at a time
    {
      const W w = A::ldtw(tw, 1);
#pragma unroll
      for (int h = 0; h < 16; h += 8)
#pragma unroll
        for (int k = 0; k < 4; ++k) ct_bfly(ar, x[h + k], x[h + k + 4], w);
    }
#pragma unroll
    for (int m = 0; m < 2; ++m) {
      const W w = A::ldtw(tw, 2 + m);
#pragma unroll
      for (int h = 0; h < 16; h += 8) {
        ct_bfly(ar, x[h + 4 * m], x[h + 4 * m + 2], w);
        ct_bfly(ar, x[h + 4 * m + 1], x[h + 4 * m + 3], w);
      }
    }
#pragma unroll
    for (int k = 0; k < 8; k += 2) {
      const W w = A::ldtw(tw, 4 + k / 2);
#pragma unroll
      for (int h = 0; h < 16; h += 8) ct_bfly(ar, x[h + k], x[h + k + 1], w);
    }
  }
  asm volatile("barrier.cluster.wait.aligned;\n" ::: "memory");
  // row k of every column belongs to block k (32-bit cluster addresses)
  {
    const uint32_t local = (uint32_t)__cvta_generic_to_shared(buf + pad(c0));
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      uint32_t remote;
      asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local), "r"(k));
      asm volatile("st.shared::cluster.v2.u64 [%0], {%1, %2};" ::"r"(remote),
                   "l"(A::bits(x[k])), "l"(A::bits(x[8 + k]))
                   : "memory");
    }
  }
  cluster.sync();

  const int jb = rank * BLK;
  load16<512>(x, vb, tid);
  ct_pass(ar, x, tw, 3, jb + tid, 512);
  store16<512>(x, vb, tid);
  __syncthreads();
  const int lb = warp * SEG + lane;
  load16<32>(x, vb, lb);
  ct_pass(ar, x, tw, 7, jb + lb, 32);
  store16<32>(x, vb, lb);
  __syncwarp();
  const int lc = (tid >> 1) * 32 + (tid & 1);
  load16<2>(x, vb, lc);
  ct_pass(ar, x, tw, 11, jb + lc, 2);
  const bool odd = tid & 1;
  const int je = jb + (tid >> 1) * 32;
  // stage 15 twiddle of element je + 2 (k + odd): 2^15 + je / 2 + odd + k
  const W *tw15 = tw + (1 << 15) + (je >> 1) + (odd ? 1 : 0);
  // butterflies k (even lane) and k+1 (odd lane) of each pair: one
  // exchange brings each lane the operand it lacks, one sends back the half
  // of the result the other lane owns, and no product is computed twice
#pragma unroll
  for (int k = 0; k < 16; k += 2) {
    // even lane holds X_k, X_{k+1}; odd lane holds Y_k, Y_{k+1}
    const V give = odd ? x[k] : x[k + 1];
    const V got = __shfl_xor_sync(0xffffffffu, give, 1);
    const V X = odd ? got : x[k], Y = odd ? x[k + 1] : got;
    const W w = A::ldtw(tw15, k);
    // outputs of this lane's butterfly, fully reduced
    V ra = X, rb = Y;
    ar.ct(ra, rb, w);
    ra = ar.full(ra);
    rb = ar.full(rb);
    // even lane keeps ra = X'_k and sends rb = Y'_k; odd keeps rb = Y'_{k+1}, sends ra
    const V back = __shfl_xor_sync(0xffffffffu, odd ? ra : rb, 1);
    x[k] = odd ? back : ra;       // even: X'_k;  odd: Y'_k (from even)
    x[k + 1] = odd ? rb : back;   // even: X'_{k+1} (from odd);  odd: Y'_{k+1}
  }
  // each lane rewrites the words it read in pass C, then the warp finishes
  // its 512-word segment in lane-interleaved pairs
  {
    uint64_t *p = buf + pad(lc);
#pragma unroll
    for (int k = 0; k < 16; ++k) p[pad_step<2>() * k] = A::to_word(x[k]);
  }
  __syncwarp();
  const int it = epi.one_poly ? (int)item : (int)(item >> 1);
  const int b = epi.one_poly ? 1 : (int)(item & 1), i = (int)job.out_off;
  const uint32_t ginv = galois_inverse(epi.items.g[epi.items.at(it)]);
  const uint64_t q = epi.primes[i];
  const ulonglong2 pi = epi.pinv[i];
  const ulonglong2 qi = epi.qinv ? epi.qinv[i] : make_ulonglong2(0, 0);
  // the constant of the post-operation (poly 0 only)
  const bool with_c = epi.has_cadd && b == 0;
  const uint64_t cadd_i = with_c ? epi.cadd[i] : 0;
  const uint64_t *accl = epi.acc + (((size_t)it * 2 + b) * epi.lk + i) * kN;
  const uint64_t *addl = b ? epi.add1 : epi.add0;
  if (addl) addl += epi.items.ct(it) * epi.add_stride + (size_t)i * kN;
  uint64_t *outl =
      epi.out + epi.items.out(it, epi.out_stride) +
      ((size_t)(epi.one_poly ? 0 : b) * epi.l_out + i) * kN;
  // pairs of evaluations per lane, four pairs' loads issued together
#pragma unroll
  for (int r0 = 0; r0 < SEG / 64; r0 += 4) {
    ulonglong2 av[4], dv[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int j = jb + warp * SEG + 2 * (lane + 32 * (r0 + u));
      av[u] = *reinterpret_cast<const ulonglong2 *>(accl + j);
      dv[u] = addl ? *reinterpret_cast<const ulonglong2 *>(addl + j) : make_ulonglong2(0, 0);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int kk = warp * SEG + 2 * (lane + 32 * (r0 + u));
      const uint32_t j = (uint32_t)(jb + kk);
      const uint64_t *bk = buf + pad(kk);  // kk even: kk + 1 is in the same block
      uint64_t w0 = shoup(sub_mod(av[u].x, bk[0], q), pi.x, pi.y, q);
      uint64_t w1 = shoup(sub_mod(av[u].y, bk[1], q), pi.x, pi.y, q);
      if (epi.qinv) {
        w0 = shoup(w0, qi.x, qi.y, q);
        w1 = shoup(w1, qi.x, qi.y, q);
      }
      if (epi.dbl) {
        w0 = add_mod(w0, w0, q);
        w1 = add_mod(w1, w1, q);
      }
      if (addl) {
        w0 = epi.add_neg ? sub_mod(w0, dv[u].x, q) : add_mod(w0, dv[u].x, q);
        w1 = epi.add_neg ? sub_mod(w1, dv[u].y, q) : add_mod(w1, dv[u].y, q);
      }
      if (with_c) {
        w0 = add_mod(w0, cadd_i, q);
        w1 = add_mod(w1, cadd_i, q);
      }
      if (ginv == 1) {
        *reinterpret_cast<ulonglong2 *>(outl + j) = make_ulonglong2(w0, w1);
      } else {
        // j even: auto_src(j + 1) = auto_src(j) ^ 1, so the pair lands on one
        // aligned pair of words, in order or swapped
        const uint32_t d = auto_src(j, ginv);
        *reinterpret_cast<ulonglong2 *>(outl + (d & ~1u)) =
            (d & 1u) ? make_ulonglong2(w1, w0) : make_ulonglong2(w0, w1);
      }
    }
  }
}

}  // namespace md

// epi: null for a plain transform, else the ModDown the forward transform
// finishes
int launch_ntt_impl(b2f_context *ctx, const uint64_t *in, long long in_stride,
                    uint64_t *out, long long out_stride, const LimbJob *jobs,
                    int jobs_per_item, int items, int inverse,
                    const ulonglong2 *scales, const ModDownOut *epi, cudaStream_t s) {
  if (items <= 0 || jobs_per_item <= 0) return B2F_OK;
  if ((((uintptr_t)in | (uintptr_t)out) & 31) || ((in_stride | out_stride) & 3)) {
    set_error("launch_ntt: limbs must be 32-byte aligned (in %p, out %p, strides %lld, %lld)",
              (const void *)in, (const void *)out, in_stride, out_stride);
    return B2F_ERR_ARG;
  }
  // one bit per device: the attribute calls are idempotent, so threads that
  // race on a device's first launch only repeat them
  static std::atomic<uint64_t> configured{0};
  const uint64_t bit = 1ull << (ctx->device & 63);
  if (!(configured.load(std::memory_order_acquire) & bit)) {
    // 16-CTA clusters are beyond the portable size of 8: opt in per kernel
    B2F_CUDA(cudaFuncSetAttribute(ntt_fwd_kernel<IntArith>,
                                  cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    B2F_CUDA(cudaFuncSetAttribute(ntt_inv_kernel<IntArith>,
                                  cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    B2F_CUDA(cudaFuncSetAttribute(ntt_fwd_kernel<FpArith>,
                                  cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    B2F_CUDA(cudaFuncSetAttribute(ntt_inv_kernel<FpArith>,
                                  cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    // the 8-CTA kernel's 68 KiB of shared memory are above the default 48
    B2F_CUDA(cudaFuncSetAttribute(md::ntt_moddown_kernel<IntArith>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, md::SMEM_BYTES));
    B2F_CUDA(cudaFuncSetAttribute(md::ntt_moddown_kernel<FpArith>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, md::SMEM_BYTES));
    configured.fetch_or(bit, std::memory_order_release);
  }
  const bool fp = ctx->fp64;
  NttParams P;
  P.in = in;
  P.out = out;
  P.in_stride = in_stride;
  P.out_stride = out_stride;
  P.jobs = jobs;
  P.tw = fp ? (const void *)(inverse ? ctx->d_twd_inv : ctx->d_twd_fwd)
            : (const void *)(inverse ? ctx->d_tw_inv : ctx->d_tw_fwd);
  P.primes = ctx->d_primes;
  P.qinv = ctx->d_qinv;
  P.scales = scales ? scales : ctx->d_ninv;
  P.jobs_per_item = jobs_per_item;
  P.items = items;
  const int cl = epi ? md::CL : CL;
  const long long blocks = (long long)items * jobs_per_item * cl;
  if (blocks > 0x7fffffffLL) {
    set_error("launch_ntt: batch too large (%lld limbs)", blocks / cl);
    return B2F_ERR_ARG;
  }
  const unsigned g = (unsigned)blocks;
  if (inverse) {
    if (fp)
      ntt_inv_kernel<FpArith><<<g, NT, SMEM_BYTES, s>>>(P);
    else
      ntt_inv_kernel<IntArith><<<g, NT, SMEM_BYTES, s>>>(P);
  } else if (epi) {
    if (fp)
      md::ntt_moddown_kernel<FpArith><<<g, md::NT, md::SMEM_BYTES, s>>>(P, *epi);
    else
      md::ntt_moddown_kernel<IntArith><<<g, md::NT, md::SMEM_BYTES, s>>>(P, *epi);
  } else {
    if (fp)
      ntt_fwd_kernel<FpArith><<<g, NT, SMEM_BYTES, s>>>(P);
    else
      ntt_fwd_kernel<IntArith><<<g, NT, SMEM_BYTES, s>>>(P);
  }
  B2F_LAUNCHED("ntt kernel launch");
  return B2F_OK;
}

}  // namespace

int launch_ntt(b2f_context *ctx, const uint64_t *in, long long in_stride,
               uint64_t *out, long long out_stride, const LimbJob *jobs,
               int jobs_per_item, int items, int inverse,
               const ulonglong2 *scales, cudaStream_t s) {
  return launch_ntt_impl(ctx, in, in_stride, out, out_stride, jobs, jobs_per_item,
                         items, inverse, scales, nullptr, s);
}

int ntt_moddown(b2f_context *ctx, uint64_t *conv, int items, int q_limbs, int lk,
                const uint64_t *acc, const uint64_t *add0, const uint64_t *add1,
                long long add_stride, uint64_t *out, long long out_stride,
                const ulonglong2 *qinv, const ItemKeys &keys, cudaStream_t s,
                const uint64_t *z, const EpiPostOp *post, bool second_only) {
  std::vector<int> key = {0, q_limbs, 0};
  std::vector<LimbJob> jobs(q_limbs);
  for (int i = 0; i < q_limbs; ++i)
    jobs[i] = LimbJob{(uint32_t)i, (uint32_t)i, (uint16_t)i, (uint16_t)i};
  const LimbJob *d = job_table(ctx, key, jobs);
  if (!d) return B2F_ERR_NOMEM;
  ModDownOut E;
  E.acc = acc;
  E.add0 = add0;
  E.add1 = add1;
  E.add_stride = add_stride;
  E.out = out;
  E.out_stride = out_stride;
  E.pinv = ctx->d_moddown_pinv;
  E.qinv = qinv;
  E.primes = ctx->d_primes;
  E.items = keys;
  E.lk = lk;
  E.l_out = q_limbs;
  E.z = z;
  E.zconv = ctx->d_md_conv_f64;
  E.zK = (z != nullptr) ? ctx->K : 0;
  E.lift = 0;
  E.zlast = nullptr;
  E.qlast_mod = nullptr;
  E.q_last = 0;
  E.mods = ctx->d_mod;
  E.dbl = post ? post->dbl : 0;
  E.add_neg = post ? post->add_neg : 0;
  E.has_cadd = post ? post->has_cadd : 0;
  if (E.has_cadd)
    for (int i = 0; i < q_limbs; ++i) E.cadd[i] = post->cadd[i];
  if (E.zK > 0 && !(ctx->fp64 && ctx->K <= 4 && ctx->d_md_conv_f64)) {
    set_error("ntt_moddown: the in-transform conversion needs binary64 and K <= 4");
    return B2F_ERR_UNSUPPORTED;
  }
  const long long st = (long long)q_limbs * kN;
  if (second_only) {  // the second poly of every item: conv [item][2][q_limbs]
    if (z) {
      set_error("ntt_moddown: one-poly ModDown takes its conversion from conv");
      return B2F_ERR_UNSUPPORTED;
    }
    E.one_poly = 1;
    return launch_ntt_impl(ctx, conv + st, 2 * st, conv + st, 2 * st, d, q_limbs, items, 0,
                           nullptr, &E, s);
  }
  return launch_ntt_impl(ctx, conv, st, conv, st, d, q_limbs, 2 * items, 0, nullptr, &E, s);
}

int ntt_rescale(b2f_context *ctx, const uint64_t *last, const uint64_t *in, uint64_t *out,
                int num_polys, int l, cudaStream_t s) {
  const int lo = l - 1;
  std::vector<LimbJob> jobs(lo);
  for (int i = 0; i < lo; ++i) jobs[i] = LimbJob{0u, (uint32_t)i, (uint16_t)i, (uint16_t)i};
  const LimbJob *d = job_table(ctx, {9, l}, jobs);
  if (!d) return B2F_ERR_NOMEM;
  return ntt_rescale_jobs(ctx, last, in, out, num_polys, l, d, s);
}

int ntt_rescale_jobs(b2f_context *ctx, const uint64_t *last, const uint64_t *in,
                     uint64_t *out, int num_polys, int l, const LimbJob *d, cudaStream_t s) {
  const int lo = l - 1;
  const LevelTables &T = ctx->levels[l];
  ModDownOut E;
  E.acc = in;
  E.add0 = E.add1 = nullptr;
  E.add_stride = 0;
  E.out = out;
  E.out_stride = 2LL * lo * kN;
  E.pinv = T.rescale_inv;
  E.qinv = nullptr;
  E.primes = ctx->d_primes;
  E.items = ItemKeys{{}, {1u}, {}, 1};
  E.lk = l;
  E.l_out = lo;
  E.z = nullptr;
  E.zconv = nullptr;
  E.zK = 0;
  E.lift = 1;
  E.zlast = last;
  E.qlast_mod = T.rescale_qlast;
  E.q_last = ctx->primes[l - 1];
  E.mods = ctx->d_mod;
  E.dbl = 0;
  E.add_neg = 0;
  E.has_cadd = 0;
  return launch_ntt_impl(ctx, last, 0, out, 0, d, lo, num_polys, 0, nullptr, &E, s);
}

int ntt_polys(b2f_context *ctx, uint64_t *data, int num_polys, int q_limbs,
              int p_limbs, int inverse, cudaStream_t s) {
  const int limbs = q_limbs + p_limbs;
  std::vector<int> key = {0, q_limbs, p_limbs};
  std::vector<LimbJob> jobs(limbs);
  for (int i = 0; i < limbs; ++i) {
    int pi = prime_of(ctx, q_limbs, i);
    jobs[i] = LimbJob{(uint32_t)i, (uint32_t)i, (uint16_t)pi, (uint16_t)pi};
  }
  const LimbJob *d = job_table(ctx, key, jobs);
  if (!d) return B2F_ERR_NOMEM;
  const long long st = (long long)limbs * kN;
  return launch_ntt(ctx, data, st, data, st, d, limbs, num_polys, inverse,
                    nullptr, s);
}

}  // namespace b2f

using namespace b2f;

extern "C" int b2f_ntt(b2f_context *ctx, uint64_t *data, int num_polys,
                       int q_limbs, int p_limbs, int inverse, void *stream) {
  B2F_RANGE("b2f_ntt");
  B2F_CHECK_ARG(ctx && data, "b2f_ntt: null argument");
  B2F_CHECK_ARG(num_polys >= 0 && q_limbs >= 0 && q_limbs <= ctx->L &&
                    p_limbs >= 0 && p_limbs <= ctx->K && q_limbs + p_limbs > 0,
                "b2f_ntt: bad limb counts q=%d p=%d (L=%d K=%d)", q_limbs,
                p_limbs, ctx->L, ctx->K);
  B2F_CHECK_ARG(((uintptr_t)data & 31) == 0, "b2f_ntt: data must be 32-byte aligned");
  return ntt_polys(ctx, data, num_polys, q_limbs, p_limbs, inverse,
                   (cudaStream_t)stream);
}
