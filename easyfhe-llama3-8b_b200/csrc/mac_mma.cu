// BSGS multiply-accumulate on the u8 tensor cores, operands staged by TMA.
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
// the host) needs one Barrett reduction.  14 sets = 56 registers: 16 warps
// per SM.
//
// Data path: the words arrive coefficient-major (N contiguous per limb).  Per
// stage one thread issues two TMA tile loads: 16 coefficients x 8 giants x 32
// babies of the chunk's plaintext rows and 16 coefficients x 8 (ciphertext,
// poly) columns x 32 babies, 32 KB each.  The tensor maps order their
// dimensions (coefficient, limb, giant or column, baby), so a box lands as
// 128-byte rows (16 coefficients) in the order baby-major, giant/column-minor,
// and the 128-byte swizzle XORs a word's 16-byte chunk with its giant/column:
// the 32 lanes' 8-byte fragment loads (giant = group id, baby = 4 thread-in-
// group values) meet 4 to a bank instead of 32.  Out-of-range giants, babies
// and ciphertexts arrive as zeros.  Three stages, each with a "full" mbarrier
// (the two loads landed) and an "empty" one (all 16 warps have their
// fragments in registers): warps run unsynchronised, up to two stages apart,
// and the issuing thread waits only before it refills a buffer.  A tile's
// outputs are staged in shared memory and stored as 128-byte rows (for 4+
// ciphertexts).  Every wait is bounded and a timeout ends the block with an
// error count.  The byte transposition into fragments is a 4 x 4 byte
// transpose (8 byte permutes per 4 registers).
#include <cuda.h>
#include <cudaTypedefs.h>

#include "b2f_internal.h"

namespace b2f {
namespace {

constexpr int MM_T = 16;                       // coefficients per tile (one 128-byte row)
constexpr int MM_KC = 32;                      // babies per stage (one k-step)
constexpr int MM_TILES = 16;                   // coefficient tiles per block
constexpr int MM_STAGES = 3;
constexpr int MM_THREADS = 512;                // one warp per coefficient of the tile
constexpr int MM_BOX = MM_T * 8 * MM_KC * 8;   // bytes of one box (32 KB)
constexpr int MM_STAGE = 2 * MM_BOX;           // plaintext box, then baby box
constexpr int MM_WARPS = MM_THREADS / 32;
constexpr int MM_OUT_ROWS = 8 * 4 * 2;               // (giant, ciphertext, poly) of a block
constexpr int MM_OUT = MM_OUT_ROWS * MM_T * 8;       // bytes of one staged output tile
constexpr size_t MM_SMEM = (size_t)MM_STAGES * MM_STAGE + 128 + 2 * MM_OUT + 1024;
constexpr long long MM_WAIT_LIMIT = 1ll << 24;  // try_wait polls before a stage is declared lost
static_assert(MM_THREADS == 32 * MM_T, "one warp per coefficient");
static_assert(MM_SMEM <= 227 * 1024, "stage buffers exceed shared memory");

__device__ int g_mac_wait_errors;

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, int count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_addr(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done;
}
// bounded wait for the phase of `parity` to complete
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
  for (long long it = 0; it < MM_WAIT_LIMIT; ++it)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}
// TMA tile loads into shared memory, completion counted on `bar`
__device__ __forceinline__ void tma_load_4d(void *dst, const CUtensorMap *map, int c0, int c1,
                                            int c2, int c3, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3, %4, %5}], [%6];\n" ::"r"(smem_addr(dst)),
      "l"((uint64_t)map), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_addr(bar))
      : "memory");
}
__device__ __forceinline__ void tma_load_5d(void *dst, const CUtensorMap *map, int c0, int c1,
                                            int c2, int c3, int c4, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3, %4, %5, %6}], [%7];\n" ::"r"(smem_addr(dst)),
      "l"((uint64_t)map), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4), "r"(smem_addr(bar))
      : "memory");
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
      if (FIRST && a == (d <= 7 ? 0 : (d - 6) / 2))  // the first tile of diagonal d
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

// The staged words of four consecutive babies (1024 bytes apart in a box)
// -> R[k] = byte k of each, k = 0..7.
__device__ __forceinline__ void load_bytes4(const uint8_t *p, uint32_t *R) {
  const uint2 w0 = *reinterpret_cast<const uint2 *>(p);
  const uint2 w1 = *reinterpret_cast<const uint2 *>(p + 1024);
  const uint2 w2 = *reinterpret_cast<const uint2 *>(p + 2048);
  const uint2 w3 = *reinterpret_cast<const uint2 *>(p + 3072);
  byte_transpose4(w0.x, w1.x, w2.x, w3.x, R);      // low words: bytes 0-3
  byte_transpose4(w0.y, w1.y, w2.y, w3.y, R + 4);  // high words: bytes 4-7
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

// grid (ceil(cts / 4), N / (16 * TILES), l), 512 threads, MM_SMEM bytes.
// Warp w computes coefficient w of each 16-coefficient tile for the block's 4
// ciphertexts (8 columns).  Limb i reduces modulo prime i for i < ql and
// prime L + i - ql after it.  tm_pt: the launch's G giants' plaintext rows,
// dims (coefficient, limb, giant, baby); tm_bb: the babies, dims
// (coefficient, limb, poly, ciphertext, baby).
template <bool STAGE_OUT>
__global__ void __launch_bounds__(MM_THREADS, 1) mac_mma_kernel(
    const __grid_constant__ CUtensorMap tm_pt, const __grid_constant__ CUtensorMap tm_bb,
    int baby_count, int cts, int g0, int G, int l, uint64_t *__restrict__ out, int out_giants,
    int giant_major, const Mod *__restrict__ mods, int ql, int L) {
  extern __shared__ uint8_t smem_raw[];
  // 128-byte swizzled boxes need 1024-byte aligned destinations
  uint8_t *const sbase = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t *const full = reinterpret_cast<uint64_t *>(sbase + MM_STAGES * MM_STAGE);
  uint64_t *const empty = full + MM_STAGES;
  uint64_t *const staged = empty + MM_STAGES;  // two: a tile's outputs all staged
  // two output tiles [row = (giant * 4 + ciphertext) * 2 + poly][16 coefficients]
  uint64_t *const obuf = reinterpret_cast<uint64_t *>(sbase + MM_STAGES * MM_STAGE + 128);
  const int tid = threadIdx.x, lane = tid & 31, wt = tid >> 5;
  const int gid = lane >> 2, tq = lane & 3;
  const int cg = blockIdx.x, limb = blockIdx.z;
  const size_t pw = (size_t)l * kN, cw = 2 * pw;
  const int kchunks = (baby_count + MM_KC - 1) / MM_KC;
  const int stages = MM_TILES * kchunks;
  const int tile0 = blockIdx.y * MM_TILES;

  if (tid == 0) {
    for (int i = 0; i < MM_STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], MM_WARPS);
    }
    mbar_init(&staged[0], MM_WARPS);
    mbar_init(&staged[1], MM_WARPS);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  __syncthreads();

  // issue cursor, used by thread 0 alone; false when the buffer never came
  // free (a bounded wait on its empty barrier timed out)
  int i_tile = 0, i_kc = 0, i_buf = 0, issued = 0;
  auto issue = [&]() -> bool {
    if (tid == 0 && issued < stages) {
      // the previous use of this buffer (stage issued - STAGES) must be read
      if (issued >= MM_STAGES &&
          !mbar_wait(&empty[i_buf], (uint32_t)(issued / MM_STAGES - 1) & 1))
        return false;
      uint8_t *st = sbase + i_buf * MM_STAGE;
      const int n0 = (tile0 + i_tile) * MM_T, kb = i_kc * MM_KC;
      mbar_expect_tx(&full[i_buf], MM_STAGE);
      tma_load_4d(st, &tm_pt, n0, limb, 0, kb, &full[i_buf]);
      tma_load_5d(st + MM_BOX, &tm_bb, n0, limb, 0, cg * 4, kb, &full[i_buf]);
      ++issued;
      if (++i_kc == kchunks) i_kc = 0, ++i_tile;
      if (++i_buf == MM_STAGES) i_buf = 0;
    }
    return true;
  };
  for (int k = 0; k < MM_STAGES - 1; ++k) issue();

  const Mod M = mods[limb < ql ? limb : L + limb - ql];
  // word (coefficient wt, giant or column gid, baby b) of a box: row b * 8 +
  // gid of 128 bytes, its 16-byte chunk XORed with gid; this lane's four
  // babies tq*4 .. tq*4 + 3 (and + 16) are 1024 bytes apart
  const uint32_t frag =
      gid * 128 + (((((uint32_t)wt >> 1) ^ gid) << 4) | ((wt & 1) << 3)) + tq * 4096;
  uint32_t acc[14][4];
  int c_tile = 0, c_kc = 0, c_buf = 0;
  uint32_t parity = 0;
  // a lost stage (bounded wait timed out) at stage s: count it; the issuing
  // thread lets its loads still in flight (stages s .. issued - 1, one per
  // buffer, so their parities are exact) land before the block's shared
  // memory is released
  auto give_up = [&](int s) {
    if (lane == 0) atomicAdd(&g_mac_wait_errors, 1);
    if (tid == 0)
      for (int k = s; k < issued; ++k)
        mbar_wait(&full[k % MM_STAGES], (uint32_t)(k / MM_STAGES) & 1);
  };
  for (int s = 0; s < stages; ++s) {
    if (!__all_sync(0xffffffffu, mbar_wait(&full[c_buf], parity))) {  // warp-uniform
      give_up(s);
      return;
    }
    const uint8_t *st = sbase + c_buf * MM_STAGE;
    uint32_t A0[8], A1[8], B0[8], B1[8];
    load_bytes4(st + frag, A0);
    load_bytes4(st + frag + 16 * 1024, A1);
    load_bytes4(st + MM_BOX + frag, B0);
    load_bytes4(st + MM_BOX + frag + 16 * 1024, B1);
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[c_buf]);  // this warp is done with the buffer
    // stage s + 2 into the buffer of stage s - 1; warp 0 reconverges on
    // thread 0's outcome before its mma.sync
    const bool issued_ok = __shfl_sync(0xffffffffu, issue(), 0);
    if (!issued_ok) {
      give_up(s + 1);
      return;
    }
    if (c_kc == 0)
      mma_diagonals<true>(acc, A0, A1, B0, B1);
    else
      mma_diagonals<false>(acc, A0, A1, B0, B1);
    if (c_kc == kchunks - 1) {
      // this thread's outputs: giant gid, ciphertext cg*4 + tq, polys 0, 1 at
      // coefficient wt.  STAGE_OUT (4+ ciphertexts): into the tile's staging
      // buffer; once all 16 warps have staged theirs, each warp stores 4 rows
      // of 16 coefficients (128 bytes), 16x fewer store transactions than a
      // word per row.  Below 4 ciphertexts the rendezvous costs more than it
      // saves (it holds back the warp that issues the loads): direct stores.
      uint64_t *ob = obuf + (c_tile & 1) * (MM_OUT_ROWS * MM_T);
      const int my_ct = cg * 4 + tq;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t D[15];
        D[0] = acc[0][h];
#pragma unroll
        for (int d = 1; d < 14; ++d) D[d] = acc[d][h] + acc[d - 1][h + 2];
        D[14] = acc[13][h + 2];
        uint64_t hi, lo;
        combine_diagonals(D, hi, lo);
        const uint64_t v = reduce128(hi, lo, M);
        if (STAGE_OUT) {
          ob[((gid * 4 + tq) * 2 + h) * MM_T + wt] = v;
        } else if (gid < G && my_ct < cts) {  // fewer than 4 ciphertexts: store directly
          const size_t slot = giant_major ? (size_t)(g0 + gid) * cts + my_ct
                                          : (size_t)my_ct * out_giants + g0 + gid;
          out[slot * cw + h * pw + (size_t)limb * kN + (size_t)(tile0 + c_tile) * MM_T + wt] =
              v;
        }
      }
    }
    if (STAGE_OUT && c_kc == kchunks - 1) {
      uint64_t *ob = obuf + (c_tile & 1) * (MM_OUT_ROWS * MM_T);
      __syncwarp();
      if (lane == 0) mbar_arrive(&staged[c_tile & 1]);
      if (!__all_sync(0xffffffffu, mbar_wait(&staged[c_tile & 1], (c_tile >> 1) & 1))) {
        give_up(s + 1);
        return;
      }
      const size_t n0 = (size_t)(tile0 + c_tile) * MM_T;
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int row = 4 * wt + 2 * k + (lane >> 4), t = lane & 15;
        const int g = row >> 3, ct = cg * 4 + ((row >> 1) & 3), h = row & 1;
        if (g < G && ct < cts) {
          const size_t slot = giant_major ? (size_t)(g0 + g) * cts + ct
                                          : (size_t)ct * out_giants + g0 + g;
          out[slot * cw + h * pw + (size_t)limb * kN + n0 + t] = ob[row * MM_T + t];
        }
      }
    }
    if (++c_kc == kchunks) c_kc = 0, ++c_tile;
    if (++c_buf == MM_STAGES) c_buf = 0, parity ^= 1;
  }
}

int ceil_log2(int x) {
  int b = 0;
  while ((1 << b) < x) ++b;
  return b;
}

using TensorMapEncoder = PFN_cuTensorMapEncodeTiled_v12000;

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// against the driver library); null when the driver does not provide it
TensorMapEncoder tensor_map_encoder() {
  static const TensorMapEncoder fn = [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return (TensorMapEncoder) nullptr;
    return reinterpret_cast<TensorMapEncoder>(p);
  }();
  return fn;
}

}  // namespace

// True when the tensor-core MAC runs this call's launches of 4 or more
// giants: it is exact (every limb's prime q has baby_count * (q - 1)^2 <
// 2^128, so the recombined byte sums fit the 128-bit Barrett input, and
// baby_count <= 1024, so the diagonal sums fit 32 bits) and the tiles are
// full enough to beat the CUDA cores: at least two ciphertexts (of a tile's
// 4), 16 babies (of a 32-baby step) and, per launch, 4 giants (of 8).  The
// bootstrap's transforms (4-8 babies, 4 giants) stay on the CUDA cores.
bool mac_mma_eligible(const b2f_context *ctx, int baby_count, int l, int ql, int cts) {
  if (ctx->mac_path == 1 || baby_count > 1024 || baby_count < 16 || cts < 2) return false;
  int bits = 0;
  for (int i = 0; i < l; ++i) {
    const uint64_t q = ctx->primes[i < ql ? i : ctx->L + i - ql];
    bits = std::max(bits, 64 - __builtin_clzll(q - 1));
  }
  return 2 * bits + ceil_log2(baby_count) <= 128;
}

// Launches the G <= 8 giants from g0 on; -1 (nothing launched) when the
// operands cannot be described as tensor maps (a base address that is not
// 16-byte aligned, or no tensor-map encoder), so the caller takes the
// CUDA-core kernel.
int launch_mac_mma(b2f_context *ctx, const uint64_t *babies, int baby_count,
                   const uint64_t *pts, int g0, int G, int l, uint64_t *out,
                   int out_giants, int cts, int giant_major, int ql, cudaStream_t s) {
  static_assert(kN % (MM_T * MM_TILES) == 0, "tiles must cover N");
  const TensorMapEncoder enc = tensor_map_encoder();
  if (!enc) return -1;
  const cuuint64_t pw = (cuuint64_t)l * kN, B = (cuuint64_t)baby_count;
  const cuuint32_t unit[5] = {1, 1, 1, 1, 1};
  CUtensorMap tm_pt, tm_bb;
  // plaintext rows [giant][baby][limb][N] from giant g0: dims (n, limb, giant, baby)
  const cuuint64_t pdim[4] = {(cuuint64_t)kN, (cuuint64_t)l, (cuuint64_t)G, B};
  const cuuint64_t pstride[3] = {kN * 8ull, B * pw * 8, pw * 8};
  const cuuint32_t pbox[4] = {MM_T, 1, 8, MM_KC};
  if (enc(&tm_pt, CU_TENSOR_MAP_DATA_TYPE_UINT64, 4,
          const_cast<uint64_t *>(pts) + (size_t)g0 * baby_count * pw, pdim, pstride, pbox, unit,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
          CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return -1;
  // babies [ct][baby][poly][limb][N]: dims (n, limb, poly, ct, baby)
  const cuuint64_t bdim[5] = {(cuuint64_t)kN, (cuuint64_t)l, 2, (cuuint64_t)cts, B};
  const cuuint64_t bstride[4] = {kN * 8ull, pw * 8, B * 2 * pw * 8, 2 * pw * 8};
  const cuuint32_t bbox[5] = {MM_T, 1, 2, 4, MM_KC};
  if (enc(&tm_bb, CU_TENSOR_MAP_DATA_TYPE_UINT64, 5, const_cast<uint64_t *>(babies), bdim,
          bstride, bbox, unit, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
          CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return -1;
  static bool attr_set[64] = {};
  if (!attr_set[ctx->device & 63]) {
    B2F_CUDA(cudaFuncSetAttribute(mac_mma_kernel<true>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, (int)MM_SMEM));
    B2F_CUDA(cudaFuncSetAttribute(mac_mma_kernel<false>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, (int)MM_SMEM));
    attr_set[ctx->device & 63] = true;
  }
  const dim3 grid((cts + 3) / 4, kN / (MM_T * MM_TILES), l);
  if (cts >= 4)
    mac_mma_kernel<true><<<grid, MM_THREADS, MM_SMEM, s>>>(tm_pt, tm_bb, baby_count, cts, g0,
                                                           G, l, out, out_giants, giant_major,
                                                           ctx->d_mod, ql, ctx->L);
  else
    mac_mma_kernel<false><<<grid, MM_THREADS, MM_SMEM, s>>>(tm_pt, tm_bb, baby_count, cts, g0,
                                                            G, l, out, out_giants, giant_major,
                                                            ctx->d_mod, ql, ctx->L);
  B2F_LAUNCHED("mac_mma_kernel");
  return B2F_OK;
}

}  // namespace b2f

extern "C" int b2f_mac_wait_errors(void) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, b2f::g_mac_wait_errors, sizeof(int)) != cudaSuccess) return -1;
  return v;
}
