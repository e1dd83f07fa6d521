// Butterfly roofline of this GPU: the rate of the NTT's lazy forward
// butterfly, in the arithmetic the context's NTT uses (64-bit integer Shoup,
// or binary64 when every prime is below 2^50), when nothing but registers is
// involved (16 independent values per thread, one twiddle, every SM full).
// The NTT kernels are bound by this multiply work on CUDA cores rather than
// by HBM, so bench.py reports their butterfly rate against the rate measured
// here.
#include "b2f_internal.h"
#include "modarith.cuh"
#include "ntt_arith.cuh"

namespace b2f {
namespace {

template <class A>
__global__ void __launch_bounds__(256) butterfly_peak_kernel(uint64_t *out,
                                                             const uint64_t *primes,
                                                             const double *qinv,
                                                             ulonglong2 w_int, int iters) {
  const A ar(primes, qinv, 0);
  const typename A::W w = A::scale(w_int);
  typename A::V x[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) x[i] = A::from_word((threadIdx.x * 16 + i + blockIdx.x) % primes[0]);
  for (int it = 0; it < iters; ++it) {
#pragma unroll
    for (int i = 0; i < 8; ++i) ct_bfly(ar, x[i], x[i + 8], w);
  }
  uint64_t s = 0;
#pragma unroll
  for (int i = 0; i < 16; ++i) s ^= A::bits(x[i]);
  out[(size_t)blockIdx.x * blockDim.x + threadIdx.x] = s;
}

// The same for mac_kernel's inner step: 8 giants x 2 polys of 128-bit
// accumulators, babies taken two at a time (2 x 8 x 2 multiply-adds per
// step), every accumulator reduced every 16 steps (32 babies), all from
// registers.
__global__ void __launch_bounds__(256) mac_peak_kernel(uint64_t *out, const Mod *mods,
                                                       int iters) {
  const Mod M = mods[0];
  U128 acc[8][2];
  uint64_t w[8], c[4];
#pragma unroll
  for (int g = 0; g < 8; ++g) {
    acc[g][0] = acc[g][1] = U128{0, 0};
    w[g] = (0x9E3779B97F4A7C15ull * (g + 1) + threadIdx.x) % M.q;
  }
#pragma unroll
  for (int u = 0; u < 4; ++u) c[u] = (0xD1B54A32D192ED03ull * (u + 7) + blockIdx.x) % M.q;
  for (int it = 0; it < iters; ++it) {
#pragma unroll
    for (int u = 0; u < 2; ++u)
#pragma unroll
      for (int g = 0; g < 8; ++g) {
        mac128(acc[g][0], c[2 * u], w[g]);
        mac128(acc[g][1], c[2 * u + 1], w[g]);
      }
    if ((it & 15) == 15) {
#pragma unroll
      for (int g = 0; g < 8; ++g) {
        acc[g][0] = U128{reduce128(acc[g][0].hi, acc[g][0].lo, M), 0};
        acc[g][1] = U128{reduce128(acc[g][1].hi, acc[g][1].lo, M), 0};
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) c[u] ^= (uint64_t)it;  // keeps the inputs live
  }
  uint64_t s = 0;
#pragma unroll
  for (int g = 0; g < 8; ++g) s ^= acc[g][0].lo ^ acc[g][1].hi;
  out[(size_t)blockIdx.x * blockDim.x + threadIdx.x] = s;
}

}  // namespace
}  // namespace b2f

using namespace b2f;

extern "C" int b2f_mac_peak(b2f_context *ctx, int iters, double *per_second,
                            void *stream) {
  B2F_CHECK_ARG(ctx && per_second && iters > 0, "b2f_mac_peak: bad argument");
  cudaStream_t s = (cudaStream_t)stream;
  int sms = 0;
  B2F_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, ctx->device));
  const int blocks = sms * 8, threads = 256;
  uint64_t *out = nullptr;
  B2F_CUDA(cudaMallocAsync(&out, sizeof(uint64_t) * blocks * threads, s));
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  float ms = 0.f;
  cudaError_t err = cudaEventCreate(&e0);
  if (err == cudaSuccess) err = cudaEventCreate(&e1);
  if (err == cudaSuccess) {
    mac_peak_kernel<<<blocks, threads, 0, s>>>(out, ctx->d_mod, iters);  // warm-up
    note_launch();
    cudaEventRecord(e0, s);
    mac_peak_kernel<<<blocks, threads, 0, s>>>(out, ctx->d_mod, iters);
    note_launch();
    cudaEventRecord(e1, s);
    err = cudaEventSynchronize(e1);
  }
  if (err == cudaSuccess) err = cudaEventElapsedTime(&ms, e0, e1);
  if (e0) cudaEventDestroy(e0);
  if (e1) cudaEventDestroy(e1);
  cudaFreeAsync(out, s);
  if (err != cudaSuccess) return cuda_status(err, "b2f_mac_peak");
  *per_second = (double)blocks * threads * iters * 32 / (ms * 1e-3);
  return B2F_OK;
}

// mac_mma_kernel's tensor-core step from registers alone: each warp issues
// `iters` rounds of the 32 independent mma.sync m16n8k32 u8 tiles (4 row x
// 8 column tiles) that one 32-baby step of that kernel issues; the operands
// change every round so nothing is hoisted.  4096 byte multiply-adds per mma.
__global__ void __launch_bounds__(256, 1) mma_u8_peak_kernel(uint32_t *out, int iters) {
  int acc[4][8][4] = {};
  uint32_t a[4], b[2];
#pragma unroll
  for (int r = 0; r < 4; ++r) a[r] = 0x01010101u * (threadIdx.x + r);
  b[0] = 0x02020202u ^ blockIdx.x;
  b[1] = 0x03030303u ^ threadIdx.x;
  for (int it = 0; it < iters; ++it) {
#pragma unroll
    for (int t = 0; t < 4; ++t)
#pragma unroll
      for (int j = 0; j < 8; ++j)
        asm volatile(
            "mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 "
            "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
            : "+r"(acc[t][j][0]), "+r"(acc[t][j][1]), "+r"(acc[t][j][2]), "+r"(acc[t][j][3])
            : "r"(a[t & 3]), "r"(a[(t + 1) & 3]), "r"(a[(t + 2) & 3]), "r"(a[(t + 3) & 3]),
              "r"(b[j & 1]), "r"(b[(j + 1) & 1]));
    a[0] += 0x01000001u;
    a[2] ^= (uint32_t)it;
    b[1] ^= (uint32_t)it;
  }
  uint32_t sum = 0;
#pragma unroll
  for (int t = 0; t < 4; ++t)
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int r = 0; r < 4; ++r) sum += (uint32_t)acc[t][j][r] * (r + 1);
  out[(size_t)blockIdx.x * blockDim.x + threadIdx.x] = sum;
}

extern "C" int b2f_mma_u8_peak(b2f_context *ctx, int iters, double *per_second,
                               void *stream) {
  B2F_CHECK_ARG(ctx && per_second && iters > 0, "b2f_mma_u8_peak: bad argument");
  cudaStream_t s = (cudaStream_t)stream;
  int sms = 0;
  B2F_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, ctx->device));
  const int blocks = sms * 4, threads = 256;
  uint32_t *out = nullptr;
  B2F_CUDA(cudaMallocAsync(&out, sizeof(uint32_t) * blocks * threads, s));
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  float ms = 0.f;
  cudaError_t err = cudaEventCreate(&e0);
  if (err == cudaSuccess) err = cudaEventCreate(&e1);
  if (err == cudaSuccess) {
    mma_u8_peak_kernel<<<blocks, threads, 0, s>>>(out, iters);  // warm-up
    note_launch();
    cudaEventRecord(e0, s);
    mma_u8_peak_kernel<<<blocks, threads, 0, s>>>(out, iters);
    note_launch();
    cudaEventRecord(e1, s);
    err = cudaEventSynchronize(e1);
  }
  if (err == cudaSuccess) err = cudaEventElapsedTime(&ms, e0, e1);
  if (e0) cudaEventDestroy(e0);
  if (e1) cudaEventDestroy(e1);
  cudaFreeAsync(out, s);
  if (err != cudaSuccess) return cuda_status(err, "b2f_mma_u8_peak");
  *per_second = (double)blocks * (threads / 32) * iters * 32 * 4096.0 / (ms * 1e-3);
  return B2F_OK;
}

extern "C" int b2f_butterfly_peak(b2f_context *ctx, int iters, double *per_second,
                                  void *stream) {
  B2F_CHECK_ARG(ctx && per_second && iters > 0, "b2f_butterfly_peak: bad argument");
  cudaStream_t s = (cudaStream_t)stream;
  int sms = 0;
  B2F_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, ctx->device));
  const int blocks = sms * 8, threads = 256;
  uint64_t *out = nullptr;
  B2F_CUDA(cudaMallocAsync(&out, sizeof(uint64_t) * blocks * threads, s));
  const uint64_t q = ctx->primes[0];
  const uint64_t w = 0x2545F4914F6CDD1Dull % q;
  const uint64_t ws = (uint64_t)(((unsigned __int128)w << 64) / q);
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  float ms = 0.f;
  cudaError_t err = cudaEventCreate(&e0);
  if (err == cudaSuccess) err = cudaEventCreate(&e1);
  if (err == cudaSuccess) {
    const ulonglong2 wi = make_ulonglong2(w, ws);
    auto run = [&]() {
      if (ctx->fp64)
        butterfly_peak_kernel<FpArith><<<blocks, threads, 0, s>>>(out, ctx->d_primes,
                                                                  ctx->d_qinv, wi, iters);
      else
        butterfly_peak_kernel<IntArith><<<blocks, threads, 0, s>>>(out, ctx->d_primes,
                                                                   ctx->d_qinv, wi, iters);
    };
    run();  // warm-up
    cudaEventRecord(e0, s);
    run();
    cudaEventRecord(e1, s);
    err = cudaEventSynchronize(e1);
  }
  if (err == cudaSuccess) err = cudaEventElapsedTime(&ms, e0, e1);
  if (e0) cudaEventDestroy(e0);
  if (e1) cudaEventDestroy(e1);
  cudaFreeAsync(out, s);
  if (err != cudaSuccess) return cuda_status(err, "b2f_butterfly_peak");
  *per_second = (double)blocks * threads * iters * 8 / (ms * 1e-3);
  return B2F_OK;
}
