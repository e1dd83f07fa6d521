// BSGS multiply-accumulate on the u8 tensor cores.
//
// The chunk sums of a hoisted BSGS transform,
//   out[ct][p][g] = sum_b pt[g][b] * baby[ct][b][p]   (mod q, per coefficient)
// are, for one coefficient of one limb, a small matrix product: giants x
// babies times babies x (ciphertext, poly).  Splitting every 64-bit residue
// into its 8 bytes turns it into an exact integer product on the u8 tensor
// cores:
//   P[(i, g)][(j, ct, p)] = sum_b byte_i(pt[g][b]) * byte_j(baby[ct][b][p])
//   out[ct][p][g] = sum_{i, j} 2^(8 (i + j)) P[(i, g)][(j, ct, p)]  mod q.
//
// Operand layout in mma.sync m16n8k32 (u8 x u8 -> s32): row tile a of the
// 64-row A operand holds byte 2a (rows 0-7) and byte 2a + 1 (rows 8-15) of
// the 8 giants; column tile j of the B operand holds byte j of 8
// (ciphertext, poly) columns.  A warp owns one coefficient and 8 columns, so
// every byte-pair sum of an output lands in the registers of one thread
// (group id = giant, thread-in-group = column pair) and the recombination
// needs no shuffle or shared-memory exchange.  Tile (a, j) accumulates into
// register set 2a + j: the tensor cores themselves sum over the row tiles of
// one diagonal, the babies and the baby stages, so after the last stage
//   D_s = set[s].rows(gid) + set[s - 1].rows(gid + 8) = sum_{i+j=s} P[i][j]
// (below 8 * 1024 * 255^2 < 2^32 for up to 1024 babies), and
//   value = sum_s D_s 2^(8s)  (< 2^128 when baby_count * q^2 is, checked on
// the host) needs one Barrett reduction.  14 sets = 56 registers keep a
// thread at 125 registers: 16 warps per SM.
//
// Data path: the words arrive coefficient-major (N contiguous per limb).  A
// block of 16 warps stages 16 coefficients (one 128-byte line per row) x 32
// babies of the chunk's plaintext rows and of 4 ciphertexts' babies in shared
// memory with 8-byte cp.async, baby-contiguous per (coefficient, row): rows
// padded to 272 bytes so the fragment loads (two 16-byte loads per four
// babies) are free of bank conflicts, coefficient slices 16 bytes apart
// modulo 128 so the words of one 32-byte sector land in distinct banks; three
// stages in flight.  The byte transposition into fragments is a 4 x 4 byte
// transpose (8 byte permutes per 4 registers).
#include "b2f_internal.h"

namespace b2f {
namespace {

constexpr int MM_KC = 32;          // babies per pipeline stage (one k-step)
constexpr int MM_ROW = MM_KC + 2;  // words per staged row
constexpr int MM_TILES = 16;       // coefficient tiles per block

// T coefficients per tile x NCB column blocks of 8: one warp per pair, 16
// warps per SM (one block of 16 warps or two of 8), 128 registers a thread.
template <int T, int NCB>
struct MmaShape {
  static constexpr int WARPS = T * NCB;
  static_assert(WARPS == 8 || WARPS == 16, "8 or 16 warps a block");
  static constexpr int THREADS = 32 * WARPS;
  static constexpr int BLOCKS_PER_SM = 16 / WARPS;
  static constexpr int COLS = 8 * NCB;                  // (ciphertext, poly) columns
  static constexpr int CTS = 4 * NCB;                   // ciphertexts per block
  static constexpr int PT_TS = 8 * MM_ROW + 2;          // words per coefficient slice
  static constexpr int BB_TS = COLS * MM_ROW + 2;
  static constexpr int STAGE_WORDS = T * (PT_TS + BB_TS);
  static constexpr int STAGES = 210 * 1024 / BLOCKS_PER_SM / (STAGE_WORDS * 8);
  static constexpr size_t SMEM = (size_t)STAGES * STAGE_WORDS * 8;
  static_assert(STAGES >= 2, "stage buffers exceed the shared-memory budget");
  static_assert((MM_ROW * 8) % 16 == 0 && (PT_TS * 8) % 16 == 0 && (BB_TS * 8) % 16 == 0 &&
                    (STAGE_WORDS * 8) % 16 == 0,
                "16-byte fragment loads need 16-byte aligned rows");
  static_assert((PT_TS * 8) % 128 == 16 && (BB_TS * 8) % 128 == 16,
                "coefficient slices 16 bytes apart modulo 128");
};

__device__ __forceinline__ void cp_async8(uint64_t *dst, const uint64_t *src, bool valid) {
  const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
  // src-size 0 fills the 8 bytes with zeros and reads nothing
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;\n" ::"r"(d), "l"(src),
               "r"(valid ? 8 : 0));
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;\n" ::);
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// d = a b (fresh accumulators)
__device__ __forceinline__ void mma_u8_zero(uint32_t (&d)[4], uint32_t a0, uint32_t a1,
                                            uint32_t a2, uint32_t a3, uint32_t b0,
                                            uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};\n"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

// c += a b
__device__ __forceinline__ void mma_u8_acc(uint32_t (&c)[4], uint32_t a0, uint32_t a1,
                                           uint32_t a2, uint32_t a3, uint32_t b0,
                                           uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// One 32-baby step: row tile a (bytes 2a, 2a + 1 of the plaintexts) times
// column tile j (byte j of the babies) accumulates into acc[2a + j].  With
// FIRST (the first baby step of a tile) the first tile of every diagonal
// starts its sums from zero.
template <bool FIRST>
__device__ __forceinline__ void mma_diagonals(uint32_t (&acc)[14][4], const uint32_t (&A0)[8],
                                              const uint32_t (&A1)[8], const uint32_t (&B0)[8],
                                              const uint32_t (&B1)[8]) {
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int d = 2 * a + j;
      if (FIRST && a == (d <= 7 ? 0 : (d - 6) / 2))
        mma_u8_zero(acc[d], A0[2 * a], A0[2 * a + 1], A1[2 * a], A1[2 * a + 1], B0[j], B1[j]);
      else
        mma_u8_acc(acc[d], A0[2 * a], A0[2 * a + 1], A1[2 * a], A1[2 * a + 1], B0[j], B1[j]);
    }
}

// r[k] = byte k of x0, x1, x2, x3 (in that order, low byte first), k = 0..3
__device__ __forceinline__ void byte_transpose4(uint32_t x0, uint32_t x1, uint32_t x2,
                                                uint32_t x3, uint32_t *r) {
  const uint32_t e0 = __byte_perm(x0, x1, 0x5140);  // x0.b0 x1.b0 x0.b1 x1.b1
  const uint32_t e1 = __byte_perm(x0, x1, 0x7362);  // x0.b2 x1.b2 x0.b3 x1.b3
  const uint32_t f0 = __byte_perm(x2, x3, 0x5140);
  const uint32_t f1 = __byte_perm(x2, x3, 0x7362);
  r[0] = __byte_perm(e0, f0, 0x5410);
  r[1] = __byte_perm(e0, f0, 0x7632);
  r[2] = __byte_perm(e1, f1, 0x5410);
  r[3] = __byte_perm(e1, f1, 0x7632);
}

// Four consecutive staged words (16-byte aligned) -> R[k] = byte k of each,
// k = 0..7.
__device__ __forceinline__ void load_bytes4(const uint64_t *p, uint32_t *R) {
  const uint4 v0 = *reinterpret_cast<const uint4 *>(p);
  const uint4 v1 = *reinterpret_cast<const uint4 *>(p + 2);
  byte_transpose4(v0.x, v0.z, v1.x, v1.z, R);      // low words: bytes 0-3
  byte_transpose4(v0.y, v0.w, v1.y, v1.w, R + 4);  // high words: bytes 4-7
}

// value = sum_s D[s] 2^(8s) as (hi, lo); the host guarantees value < 2^128
__device__ __forceinline__ void combine_diagonals(const uint32_t (&D)[15], uint64_t &hi,
                                                  uint64_t &lo) {
  uint64_t W[4];
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    W[w] = D[4 * w];
#pragma unroll
    for (int d = 4 * w + 1; d < 4 * w + 4 && d < 15; ++d)
      W[w] += (uint64_t)D[d] << (8 * (d - 4 * w));
  }
  lo = W[0] + (W[1] << 32);
  hi = (W[1] >> 32) + W[2] + (W[3] << 32) + (lo < W[0]);
}

// grid (ceil(cts / (4 NCB)), N / (T * TILES), l), 32 T NCB threads,
// MmaShape<T, NCB>::SMEM bytes.  Warp w computes coefficient w / NCB of each
// tile for column block w % NCB.  Limb i reduces modulo prime i for i < ql
// and prime L + i - ql after it.
template <int T, int NCB>
__global__ void __launch_bounds__(32 * T * NCB, 16 / (T * NCB)) mac_mma_kernel(
    const uint64_t *__restrict__ babies, int baby_count, int cts,
    const uint64_t *__restrict__ pts, int g0, int G, int l,
    uint64_t *__restrict__ out, int out_giants, int giant_major,
    const Mod *__restrict__ mods, int ql, int L) {
  using S = MmaShape<T, NCB>;
  extern __shared__ __align__(16) uint64_t smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gid = lane >> 2, tq = lane & 3;
  const int wt = warp / NCB, cb = warp % NCB;
  const int cg = blockIdx.x, limb = blockIdx.z;
  const size_t pw = (size_t)l * kN, cw = 2 * pw;
  const int kchunks = (baby_count + MM_KC - 1) / MM_KC;
  const int stages = MM_TILES * kchunks;
  const int tile0 = blockIdx.y * MM_TILES;

  // copy roles: coefficient lt of the tile; in copy round k the thread
  // copies baby lb of row group k * RSTEP + lrow (plaintext row groups are
  // giants, baby row groups (ciphertext, poly) columns, 32 babies each), so
  // every copy of a stage is a fixed base + the stage's offset + a row stride
  constexpr int RPR = S::THREADS / T;  // staged rows per copy round
  static_assert(RPR % 32 == 0, "copy rounds cover whole 32-baby row groups");
  constexpr int RSTEP = RPR / 32;
  const int lt = tid % T, lr = tid / T, lb = lr & 31, lrow = lr >> 5;
  const int valid_cts = min(S::CTS, cts - cg * S::CTS);
  // rows past the last baby are zero-filled: their source stays at a valid
  // address (baby min(lb, B - 1) of the first baby chunk) and reads nothing
  const int lb_c = min(lb, baby_count - 1);
  const size_t gstride = (size_t)baby_count * pw, cstride = (size_t)baby_count * cw;
  const uint64_t *pt_base =
      pts + ((size_t)g0 * baby_count + lb_c) * pw + (size_t)limb * kN + lt;
  const uint64_t *bb_base =
      babies + ((size_t)cg * S::CTS * baby_count + lb_c) * cw + (size_t)limb * kN + lt;
  uint64_t *const pt_dst = smem + lt * S::PT_TS + lb;
  uint64_t *const bb_dst = smem + T * S::PT_TS + lt * S::BB_TS + lb;

  // issue cursor: tile, baby chunk and buffer of the next stage to load
  int i_tile = 0, i_kc = 0, i_buf = 0, i_left = stages;
  auto issue = [&]() {
    if (i_left > 0) {
      const int kb = i_kc * MM_KC;
      const size_t n0 = (size_t)(tile0 + i_tile) * T;
      const bool ok = kb + lb < baby_count;
      const size_t poff = (ok ? (size_t)kb * pw : 0) + n0;
      const size_t boff = (ok ? (size_t)kb * cw : 0) + n0;
      const size_t so = (size_t)i_buf * S::STAGE_WORDS;
#pragma unroll
      for (int k = 0; k < 8 / RSTEP; ++k) {  // plaintext rows: 8 giants x 32 babies
        const int g = k * RSTEP + lrow;
        if (g < G) cp_async8(pt_dst + so + g * MM_ROW, pt_base + g * gstride + poff, ok);
      }
#pragma unroll
      for (int k = 0; k < S::COLS / RSTEP; ++k) {  // baby rows: COLS x 32 babies
        const int c = k * RSTEP + lrow, ct = c >> 1;
        if (ct < valid_cts)
          cp_async8(bb_dst + so + c * MM_ROW, bb_base + ct * cstride + (c & 1) * pw + boff, ok);
      }
      --i_left;
      if (++i_kc == kchunks) i_kc = 0, ++i_tile;
      if (++i_buf == S::STAGES) i_buf = 0;
    }
    cp_async_commit();
  };

  const Mod M = mods[limb < ql ? limb : L + limb - ql];
  // acc[s]: the tiles (a, j) with 2a + j = s summed by the tensor cores over
  // babies and stages; c0, c1 (rows gid: byte 2a) add to diagonal s,
  // c2, c3 (rows gid + 8: byte 2a + 1) to diagonal s + 1
  uint32_t acc[14][4];

  for (int k = 0; k < S::STAGES - 1; ++k) issue();
  int c_tile = 0, c_kc = 0, c_buf = 0;
  for (int s = 0; s < stages; ++s) {
    cp_async_wait<S::STAGES - 2>();
    __syncthreads();
    issue();
    const uint64_t *st = smem + (size_t)c_buf * S::STAGE_WORDS;
    const uint64_t *prow = st + wt * S::PT_TS + gid * MM_ROW + tq * 4;
    const uint64_t *brow =
        st + T * S::PT_TS + wt * S::BB_TS + (cb * 8 + gid) * MM_ROW + tq * 4;
    uint32_t A0[8], A1[8], B0[8], B1[8];
    load_bytes4(prow, A0);
    load_bytes4(prow + 16, A1);
    load_bytes4(brow, B0);
    load_bytes4(brow + 16, B1);
    if (c_kc == 0)
      mma_diagonals<true>(acc, A0, A1, B0, B1);
    else
      mma_diagonals<false>(acc, A0, A1, B0, B1);
    if (c_kc == kchunks - 1) {
      // this thread's outputs: giant gid, ciphertext cg*CTS + cb*4 + tq, polys 0, 1
      const int ct = cg * S::CTS + cb * 4 + tq;
      const size_t n = (size_t)(tile0 + c_tile) * T + wt;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t D[15];
        D[0] = acc[0][h];
#pragma unroll
        for (int d = 1; d < 14; ++d) D[d] = acc[d][h] + acc[d - 1][h + 2];
        D[14] = acc[13][h + 2];
        uint64_t hi, lo;
        combine_diagonals(D, hi, lo);
        if (gid < G && ct < cts) {
          const size_t slot = giant_major ? (size_t)(g0 + gid) * cts + ct
                                          : (size_t)ct * out_giants + g0 + gid;
          out[slot * cw + h * pw + (size_t)limb * kN + n] = reduce128(hi, lo, M);
        }
      }
    }
    if (++c_kc == kchunks) c_kc = 0, ++c_tile;
    if (++c_buf == S::STAGES) c_buf = 0;
  }
  cp_async_wait<0>();
}

int ceil_log2(int x) {
  int b = 0;
  while ((1 << b) < x) ++b;
  return b;
}

}  // namespace

// True when the tensor-core MAC runs this call: it is exact (every limb's
// prime q has baby_count * (q - 1)^2 < 2^128, so the recombined byte sums fit
// the 128-bit Barrett input, and baby_count <= 1024, so the diagonal sums fit
// 32 bits) and the batch has at least two ciphertexts (one ciphertext fills
// a quarter of the 8 columns of a tile: the CUDA-core kernel is faster there,
// 1.2 against 1.7 ms at the linear block's chunk on B200).
bool mac_mma_eligible(const b2f_context *ctx, int baby_count, int l, int ql, int cts) {
  if (ctx->mac_path == 1 || baby_count > 1024 || cts < 2) return false;
  int bits = 0;
  for (int i = 0; i < l; ++i) {
    const uint64_t q = ctx->primes[i < ql ? i : ctx->L + i - ql];
    bits = std::max(bits, 64 - __builtin_clzll(q - 1));
  }
  return 2 * bits + ceil_log2(baby_count) <= 128;
}

template <int T, int NCB>
static int launch_shape(b2f_context *ctx, const uint64_t *babies, int baby_count,
                        const uint64_t *pts, int g0, int G, int l, uint64_t *out,
                        int out_giants, int cts, int giant_major, int ql, cudaStream_t s) {
  using S = MmaShape<T, NCB>;
  static_assert(kN % (T * MM_TILES) == 0, "tiles must cover N");
  static bool attr_set[64] = {};
  if (!attr_set[ctx->device & 63]) {
    B2F_CUDA(cudaFuncSetAttribute(mac_mma_kernel<T, NCB>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, (int)S::SMEM));
    attr_set[ctx->device & 63] = true;
  }
  const dim3 grid((cts + S::CTS - 1) / S::CTS, kN / (T * MM_TILES), l);
  mac_mma_kernel<T, NCB><<<grid, S::THREADS, S::SMEM, s>>>(babies, baby_count, cts, pts, g0, G, l,
                                                    out, out_giants, giant_major, ctx->d_mod,
                                                    ql, ctx->L);
  B2F_LAUNCHED("mac_mma_kernel");
  return B2F_OK;
}

int launch_mac_mma(b2f_context *ctx, const uint64_t *babies, int baby_count,
                   const uint64_t *pts, int g0, int G, int l, uint64_t *out,
                   int out_giants, int cts, int giant_major, int ql, cudaStream_t s) {
  return launch_shape<16, 1>(ctx, babies, baby_count, pts, g0, G, l, out, out_giants, cts,
                             giant_major, ql, s);
}

}  // namespace b2f
