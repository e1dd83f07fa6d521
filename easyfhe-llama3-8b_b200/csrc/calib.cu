// Butterfly roofline of this GPU: the rate of the NTT's lazy forward
// butterfly, in the arithmetic the context's NTT uses (64-bit integer Shoup,
// or binary64 when every prime is below 2^50), when nothing but registers is
// involved (16 independent values per thread, one twiddle, every SM full).
// The NTT kernels are bound by this multiply work on CUDA cores rather than
// by HBM, so bench.py reports their butterfly rate against the rate measured
// here.
#include "b2f_internal.h"
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

}  // namespace
}  // namespace b2f

using namespace b2f;

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
