// Fast base conversion (ModUp step 2, ModDown step 4b) on the 5th-generation
// tensor cores: tcgen05.mma kind::i8 with the accumulator in tensor memory.
//
// For T targets and w input limbs, out_t[n] = sum_i x_i[n] c_{t,i} mod p_t
// is, over the bytes of the inputs (k = 8i + a) and of the constants
// c_{t,i} 2^(8a) mod p_t (output byte b), one integer matrix product per
// tile of 128 coefficients:
//   D[n][(t, b)] = sum_k X[n][k] C[(t, b)][k],   out_t[n] = sum_b D 2^(8b)
// (each D below 2^23, the recombined value below 2^79, one Barrett-style
// reduction).  The coefficients are the M dimension (128 TMEM lanes) and
// (target, output byte) the N dimension, so the eight byte sums of every
// output of a coefficient sit in one lane: the warp that reads that lane
// quarter (tcgen05.ld 32x32b.x8, eight columns per target) recombines them in
// registers and stores 32 consecutive coefficients at once.
//
// Operands are K-major u8 in the no-swizzle canonical layout: 8 rows x 16
// bytes per 128-byte core matrix, 8-row groups 128 bytes apart (SBO), 16-byte
// K chunks one group-column apart (LBO).  Each thread stages its coefficient's
// input words as one row (two words per 16-byte store); the constant rows are
// re-laid from the mma.sync table once per block.  One thread issues the MMAs
// (M = 128, N <= 256 per instruction, 32 bytes of K per instruction) and
// commits them to an mbarrier; every wait is bounded and counted.  Two
// threads per coefficient: warps w and w + 4 read the same TMEM lane quarter
// and split the targets; the next tile's words are loaded during the
// current tile's MMA and epilogue.
#include "b2f_internal.h"

namespace b2f {
namespace {

constexpr int UC_M = 128;         // coefficients per tile (TMEM lanes, MMA M)
constexpr int UC_THREADS = 256;   // two threads per coefficient (warps w, w + 4 share lanes)
constexpr int UC_TILES = 8;       // 128-coefficient tiles per block
constexpr long long UC_WAIT_LIMIT = 1ll << 24;

__device__ int g_conv_wait_errors;

__device__ __forceinline__ uint32_t saddr(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void uc_mbar_init(uint64_t *bar) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(saddr(bar)));
  asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}
__device__ __forceinline__ bool uc_mbar_wait(uint64_t *bar, uint32_t parity) {
  for (long long it = 0; it < UC_WAIT_LIMIT; ++it) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(saddr(bar)), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}
// tensor memory: allocation by one whole warp, address written to shared memory
__device__ __forceinline__ void tmem_alloc(uint32_t *dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(
                   saddr(dst)),
               "r"(ncols));
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::);
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(taddr),
               "r"(ncols));
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
}
// shared-memory writes of this thread visible to the tensor cores' reads
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}
// K-major, no swizzle: start, leading (K chunk) and stride (8-row group)
// byte offsets in 16-byte units, descriptor version 1
__device__ __forceinline__ uint64_t smem_desc(const void *p, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr(p) >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46);
}
// D (tmem) = A B (+ D when accumulate); u8 x u8 -> s32
__device__ __forceinline__ void umma_u8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}\n" ::"r"(
          tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u));
}
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(
          saddr(bar))
      : "memory");
}
// eight consecutive columns of this warp's 32 lanes; complete after tmem_wait
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t *r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
}

// (hi 2^64 + lo) mod p for hi < 2^16 (as in the mma.sync conversion)
__device__ __forceinline__ uint64_t umul_lo32(uint64_t a, uint32_t b) {
  return (uint64_t)(uint32_t)a * b + (((uint64_t)(uint32_t)(a >> 32) * b) << 32);
}
__device__ __forceinline__ uint64_t umul_hi32(uint64_t a, uint32_t b) {
  return ((uint64_t)(uint32_t)(a >> 32) * b + (((uint64_t)(uint32_t)a * b) >> 32)) >> 32;
}
__device__ __forceinline__ uint64_t uc_reduce79(uint64_t hi, uint64_t lo, const Red79 &R) {
  const uint64_t p = R.p;
  const uint64_t qe = umul_hi32(lo, (uint32_t)R.mu);
  const uint64_t r0 = lo - umul_lo32(p, (uint32_t)qe);
  const uint32_t h = (uint32_t)hi;
  const uint64_t y1 = umul_lo32(R.r, h) - umul_lo32(p, (uint32_t)umul_hi32(R.rs, h));
  uint64_t v = r0 + y1;  // < 4p
  v = v >= 2 * p ? v - 2 * p : v;
  return v >= p ? v - p : v;
}

// Shared memory of a block: barrier and TMEM address (128 bytes), then the
// coefficient tile X (kp / 16 chunks of 2048 bytes) and the constants C
// (kp / 16 chunks of (N / 8) x 128 bytes).
inline size_t conv_umma_smem(int kp, int N) {
  return 128 + (size_t)(kp / 16) * 2048 + (size_t)(kp / 16) * (N / 8) * 128;
}

// x: limb 0 of the w input limbs (N apart); A: the mma.sync constant table
// (conv_bytes: row G*64 + (b/2)*16 + (b%2)*8 + t%8 for target t = 8G + t%8,
// output byte b; kp bytes a row); T targets; out(t), red(t) as in
// conv_mma_block.  The block converts tiles [n_begin, n_begin + 128 UC_TILES).
template <class Out, class Rd>
__device__ __forceinline__ void conv_umma_block(const uint64_t *__restrict__ x, int w,
                                                const uint8_t *__restrict__ A, int T, int kp,
                                                Out out, Rd red, int n_begin) {
  extern __shared__ __align__(128) uint8_t ucs[];
  uint64_t *mbar = reinterpret_cast<uint64_t *>(ucs);
  uint32_t *tptr = reinterpret_cast<uint32_t *>(ucs + 16);
  uint8_t *Xs = ucs + 128;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int N = 8 * ((T + 1) & ~1);  // a multiple of 16
  const int kch = kp / 16;           // 16-byte K chunks (even)
  uint8_t *Cs = Xs + kch * 2048;
  const uint32_t c_lbo = (uint32_t)(N / 8) * 128;
  // constants, re-laid as rows (t, b) = 8t + b
  for (int idx = tid; idx < N * kch; idx += UC_THREADS) {
    const int r = idx / kch, c = idx - r * kch, t = r >> 3, b = r & 7;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (t < T) {
      const size_t orow = (size_t)(t >> 3) * 64 + (b >> 1) * 16 + (b & 1) * 8 + (t & 7);
      v = __ldg(reinterpret_cast<const uint4 *>(A + orow * kp) + c);
    }
    *reinterpret_cast<uint4 *>(Cs + c * c_lbo + (r >> 3) * 128 + (r & 7) * 16) = v;
  }
  const uint32_t ncols = N <= 32 ? 32 : N <= 64 ? 64 : N <= 128 ? 128 : N <= 256 ? 256 : 512;
  if (warp == 0) tmem_alloc(tptr, ncols);
  if (tid == 0) uc_mbar_init(mbar);
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tptr;
  // s32 accumulate, u8 x u8, both K-major, M = 128
  const uint32_t idesc_m = (2u << 4) | (8u << 24);
  uint32_t parity = 0;
  bool lost = false;
  // this thread's coefficient of a tile as one K-major row (words 2c, 2c+1 in
  // chunk c); the next tile's words are loaded while this tile computes
  // thread (r, h): coefficient r of the tile, chunks c = h, h + 2, ...
  constexpr int WMAX = 8;
  const int r = tid & (UC_M - 1), h = tid >> 7;
  uint64_t xw[WMAX];
  auto load_tile = [&](int n0) {
#pragma unroll
    for (int j = 0; j < WMAX / 2; ++j) {
      const int c = 2 * j + h, i0 = 2 * c, i1 = i0 + 1;
      if (c < kch) {
        xw[2 * j] = i0 < w ? x[(size_t)i0 * kN + n0 + r] : 0;
        xw[2 * j + 1] = i1 < w ? x[(size_t)i1 * kN + n0 + r] : 0;
      }
    }
  };
  load_tile(n_begin);
  for (int tile = 0; tile < UC_TILES && !lost; ++tile) {
    const int n0 = n_begin + tile * UC_M;
#pragma unroll
    for (int j = 0; j < WMAX / 2; ++j) {
      const int c = 2 * j + h;
      if (c < kch)
        *reinterpret_cast<ulonglong2 *>(Xs + c * 2048 + (r >> 3) * 128 + (r & 7) * 16) =
            make_ulonglong2(xw[2 * j], xw[2 * j + 1]);
    }
    fence_async_smem();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      for (int nc = 0; nc < N; nc += 256) {
        const int nn = min(256, N - nc);
        const uint32_t idesc = idesc_m | ((uint32_t)(nn >> 3) << 17);
        for (int s = 0; s < kch / 2; ++s)
          umma_u8(tmem + nc, smem_desc(Xs + 2 * s * 2048, 2048, 128),
                  smem_desc(Cs + 2 * s * c_lbo + (nc / 8) * 128, c_lbo, 128), idesc, s > 0);
      }
      umma_commit(mbar);
    }
    if (tile + 1 < UC_TILES) load_tile(n0 + UC_M);
    lost = __syncthreads_or(!uc_mbar_wait(mbar, parity));
    parity ^= 1;
    if (lost) break;
    tc_fence_after();
    // lanes 32 (warp % 4) .. + 31 = coefficients n0 + r; warps w and w + 4
    // take alternate groups of four targets (32 columns per wait)
    const uint32_t trow = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    for (int t0 = 4 * h; t0 < T; t0 += 8) {
      uint32_t d[4][8];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (t0 + u < T) tmem_ld8(trow + 8 * (t0 + u), d[u]);
      tmem_wait();
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int t = t0 + u;
        if (t < T) {
          uint64_t lo4 = d[u][0], hi4 = d[u][4];
          lo4 += (uint64_t)d[u][1] << 8;
          hi4 += (uint64_t)d[u][5] << 8;
          lo4 += (uint64_t)d[u][2] << 16;
          hi4 += (uint64_t)d[u][6] << 16;
          lo4 += (uint64_t)d[u][3] << 24;
          hi4 += (uint64_t)d[u][7] << 24;
          const uint64_t lo = lo4 + (hi4 << 32);
          const uint64_t hi = (hi4 >> 32) + (lo < lo4);
          out(t)[n0 + r] = uc_reduce79(hi, lo, red(t));
        }
      }
    }
    tc_fence_before();
    __syncthreads();  // TMEM and the tile are free for the next tile
  }
  if (lost) {
    if (tid == 0) {
      atomicAdd(&g_conv_wait_errors, 1);
      uc_mbar_wait(mbar, parity ^ 1);  // the MMAs in flight, once more bounded
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
  }
  if (warp == 0) tmem_dealloc(tmem, ncols);
}

// ModUp step 2.  grid (N / (128 TILES), beta, cts), 128 threads
__global__ void __launch_bounds__(UC_THREADS) modup_conv_umma_kernel(
    const uint64_t *__restrict__ xt, uint64_t *__restrict__ ext,
    const uint8_t *__restrict__ bytes, size_t bytes_stride, const Red79 *__restrict__ reds,
    int l, int K, int L, int alpha, int kp) {
  const int j = blockIdx.y, ct = blockIdx.z, beta = gridDim.y, lk = l + K;
  const int lo = j * alpha, hi = min(lo + alpha, l), w = hi - lo;
  uint64_t *dst = ext + ((size_t)ct * beta + j) * lk * kN;
  conv_umma_block(
      xt + ((size_t)ct * l + lo) * kN, w, bytes + j * bytes_stride, lk - w, kp,
      [=](int tau) { return dst + (size_t)(tau < lo ? tau : tau + w) * kN; },
      [=](int tau) {
        const int t = tau < lo ? tau : tau + w;
        return reds[t < l ? t : L + (t - l)];
      },
      blockIdx.x * UC_M * UC_TILES);
}

// ModDown step 4b.  grid (N / (128 TILES), 2, cts), 128 threads
__global__ void __launch_bounds__(UC_THREADS) moddown_conv_umma_kernel(
    const uint64_t *__restrict__ acc, uint64_t *__restrict__ conv_out,
    const uint8_t *__restrict__ bytes, const Red79 *__restrict__ reds, int l, int K, int kp) {
  const int b = blockIdx.y, ct = blockIdx.z, lk = l + K;
  uint64_t *o = conv_out + (((size_t)ct * 2 + b) * l) * kN;
  conv_umma_block(
      acc + (((size_t)ct * 2 + b) * lk + l) * kN, K, bytes, l, kp,
      [=](int t) { return o + (size_t)t * kN; }, [=](int t) { return reds[t]; },
      blockIdx.x * UC_M * UC_TILES);
}

int set_umma_smem(const void *kern, size_t bytes) {
  if (bytes > 48 * 1024)
    B2F_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)bytes));
  return B2F_OK;
}

}  // namespace

// ModUp conversion on tcgen05; -1 (nothing launched) when a digit has more
// than 64 targets (N > 512 TMEM columns), so the caller takes mma.sync.
int launch_modup_conv_umma(b2f_context *ctx, const uint64_t *xt, uint64_t *ext, int l,
                           int cts, cudaStream_t s) {
  const LevelTables &LT = ctx->levels[l];
  const int K = ctx->K, lk = l + K, alpha = ctx->alpha, kp = conv_kpad(alpha);
  const int w_min = l - (LT.beta - 1) * alpha;
  const int t_max = lk - w_min;
  if (t_max > 64 || kp > 128) return -1;
  const size_t sm = conv_umma_smem(kp, 8 * ((t_max + 1) & ~1));
  int rc;
  if ((rc = set_umma_smem((const void *)modup_conv_umma_kernel, sm))) return rc;
  const dim3 grid(kN / (UC_M * UC_TILES), LT.beta, cts);
  modup_conv_umma_kernel<<<grid, UC_THREADS, sm, s>>>(xt, ext, LT.modup_bytes,
                                                      LT.modup_bytes_stride, ctx->d_red79, l,
                                                      K, ctx->L, alpha, kp);
  B2F_LAUNCHED("modup_conv_umma_kernel");
  return B2F_OK;
}

// ModDown conversion (P to Q_l) on tcgen05; -1 when l > 64 or K > 16.
int launch_moddown_conv_umma(b2f_context *ctx, const uint64_t *acc, uint64_t *conv, int l,
                             int cts, cudaStream_t s, int polys) {
  const int K = ctx->K, kp = conv_kpad(K);
  if (l > 64 || kp > 128) return -1;
  const size_t sm = conv_umma_smem(kp, 8 * ((l + 1) & ~1));
  int rc;
  if ((rc = set_umma_smem((const void *)moddown_conv_umma_kernel, sm))) return rc;
  const dim3 grid(kN / (UC_M * UC_TILES), polys, cts);
  moddown_conv_umma_kernel<<<grid, UC_THREADS, sm, s>>>(acc, conv, ctx->d_moddown_bytes,
                                                        ctx->d_red79, l, K, kp);
  B2F_LAUNCHED("moddown_conv_umma_kernel");
  return B2F_OK;
}

}  // namespace b2f

extern "C" int b2f_set_conv_path(b2f_context *ctx, int path) {
  B2F_CHECK_ARG(ctx, "b2f_set_conv_path: null context");
  B2F_CHECK_ARG(path >= 0 && path <= 2, "b2f_set_conv_path: path %d is not 0, 1 or 2", path);
  ctx->conv_path = path;
  return B2F_OK;
}

extern "C" int b2f_conv_wait_errors(void) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, b2f::g_conv_wait_errors, sizeof(int)) != cudaSuccess) return -1;
  return v;
}
