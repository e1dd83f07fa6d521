// Integer-multiply roofline of this GPU: the rate of the NTT's lazy Shoup
// butterfly when nothing but registers is involved (16 independent values per
// thread, one twiddle, every SM full).  The NTT kernels are bound by this
// 64-bit multiply work on CUDA cores rather than by HBM, so bench.py reports
// their butterfly rate against the rate measured here.
#include "b2f_internal.h"

namespace b2f {
namespace {

__global__ void __launch_bounds__(256) butterfly_peak_kernel(uint64_t *out, uint64_t q,
                                                             uint64_t w, uint64_t ws,
                                                             int iters) {
  uint64_t x[16];
  const uint64_t q2 = 2 * q;
#pragma unroll
  for (int i = 0; i < 16; ++i) x[i] = (threadIdx.x * 16 + i + blockIdx.x) % q;
  for (int it = 0; it < iters; ++it) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      uint64_t &a = x[i], &b = x[i + 8];
      const uint64_t u = a >= q2 ? a - q2 : a;
      const uint64_t t = b * w - __umul64hi(b, ws) * q;
      a = u + t;
      b = u - t + q2;
    }
  }
  uint64_t s = 0;
#pragma unroll
  for (int i = 0; i < 16; ++i) s ^= x[i];
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
    butterfly_peak_kernel<<<blocks, threads, 0, s>>>(out, q, w, ws, iters);  // warm-up
    cudaEventRecord(e0, s);
    butterfly_peak_kernel<<<blocks, threads, 0, s>>>(out, q, w, ws, iters);
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
