// Client-side key material and symmetric encryption on the GPU.
//
// Randomness is ChaCha20 (Bernstein 2008; 64-bit block counter, 64-bit
// nonce used as the stream id) keyed by the 64-bit session seed.  Sampling:
//   uniform mod q  : coefficient k uses 128 bits (words 2(k%4), 2(k%4)+1 of
//                    block k/4) reduced mod q;
//   error          : centred binomial with eta = 21 from word k%8 of block
//                    k/8 (variance 10.5);
//   stream ids     : (tag << 56) | (a << 32) | (b << 16) | c, with tags
//                    1 secret, 2 key uniform, 3 key error, 4 encryption
//                    uniform, 5 encryption error.
// Key switching key from s_from to s_to, digits of the top level:
//   key[j][1][t] = a,  key[j][0][t] = -a s_to + e + [t in D_j] (P mod q_t) s_from.
// Rotation keys switch s to sigma_{g^-1}(s) (the automorphism is applied
// after the key switch); the relinearisation key switches s^2 to s.
#include "b2f_internal.h"

namespace b2f {
namespace {

constexpr int TPB = 256;

__host__ __device__ __forceinline__ uint32_t rotl32(uint32_t v, int c) {
  return (v << c) | (v >> (32 - c));
}
#define B2F_QR(a, b, c, d)          \
  a += b; d ^= a; d = rotl32(d, 16); \
  c += d; b ^= c; b = rotl32(b, 12); \
  a += b; d ^= a; d = rotl32(d, 8);  \
  c += d; b ^= c; b = rotl32(b, 7);

__host__ __device__ inline void chacha_block(uint64_t seed, uint64_t stream,
                                             uint64_t counter, uint64_t out[8]) {
  uint32_t s[16] = {0x61707865u, 0x3320646eu, 0x79622d32u, 0x6b206574u,
                    (uint32_t)seed, (uint32_t)(seed >> 32), 0, 0, 0, 0, 0, 0,
                    (uint32_t)counter, (uint32_t)(counter >> 32),
                    (uint32_t)stream, (uint32_t)(stream >> 32)};
  uint32_t x[16];
  for (int i = 0; i < 16; ++i) x[i] = s[i];
  for (int i = 0; i < 10; ++i) {
    B2F_QR(x[0], x[4], x[8], x[12]);
    B2F_QR(x[1], x[5], x[9], x[13]);
    B2F_QR(x[2], x[6], x[10], x[14]);
    B2F_QR(x[3], x[7], x[11], x[15]);
    B2F_QR(x[0], x[5], x[10], x[15]);
    B2F_QR(x[1], x[6], x[11], x[12]);
    B2F_QR(x[2], x[7], x[8], x[13]);
    B2F_QR(x[3], x[4], x[9], x[14]);
  }
  for (int i = 0; i < 8; ++i)
    out[i] = (uint64_t)(x[2 * i] + s[2 * i]) |
             ((uint64_t)(x[2 * i + 1] + s[2 * i + 1]) << 32);
}

__host__ __device__ inline uint64_t stream_id(uint64_t tag, uint64_t a,
                                              uint64_t b, uint64_t c) {
  return (tag << 56) | ((a & 0xFFFFFFull) << 32) | ((b & 0xFFFFull) << 16) |
         (c & 0xFFFFull);
}
enum { TAG_SECRET = 1, TAG_KEY_A = 2, TAG_KEY_E = 3, TAG_ENC_A = 4, TAG_ENC_E = 5 };

__device__ __forceinline__ uint64_t uniform_at(uint64_t seed, uint64_t stream,
                                               int k, const Mod &M) {
  uint64_t blk[8];
  chacha_block(seed, stream, (uint64_t)(k >> 2), blk);
  const int p = k & 3;
  return reduce128(blk[2 * p], blk[2 * p + 1], M);
}
__device__ __forceinline__ int cbd_at(uint64_t seed, uint64_t stream, int k) {
  uint64_t blk[8];
  chacha_block(seed, stream, (uint64_t)(k >> 3), blk);
  const uint64_t w = blk[k & 7];
  return __popcll(w & 0x1FFFFFull) - __popcll((w >> 21) & 0x1FFFFFull);
}
__device__ __forceinline__ uint64_t signed_residue(long long v, uint64_t q) {
  if (v >= 0) return (uint64_t)v % q;
  uint64_t r = (uint64_t)(-v) % q;
  return r ? q - r : 0;
}

// error polys of every digit, coefficient form, into key[j][0][t]
__global__ void __launch_bounds__(TPB) key_error_kernel(
    uint64_t *key, uint64_t seed, uint32_t tag, const uint64_t *primes, int np) {
  const int k = blockIdx.x * TPB + threadIdx.x;
  const int j = blockIdx.y;
  const int e = cbd_at(seed, stream_id(TAG_KEY_E, tag, j, 0), k);
  uint64_t *b = key + (size_t)j * 2 * np * kN;
  for (int t = 0; t < np; ++t) b[(size_t)t * kN + k] = signed_residue(e, primes[t]);
}

// grid (N/TPB, np, digits)
__global__ void __launch_bounds__(TPB) key_finish_kernel(
    uint64_t *key, const uint64_t *s_from, const uint64_t *s_to, uint64_t seed,
    uint32_t tag, const Mod *mods, const uint64_t *pmod, int L, int np,
    int alpha) {
  const int k = blockIdx.x * TPB + threadIdx.x;
  const int t = blockIdx.y, j = blockIdx.z;
  const Mod M = mods[t];
  const uint64_t a = uniform_at(seed, stream_id(TAG_KEY_A, tag, j, t), k, M);
  uint64_t *b = key + ((size_t)j * 2 * np + t) * kN + k;
  const size_t idx = (size_t)t * kN + k;
  uint64_t v = sub_mod(*b, mul_mod(a, s_to[idx], M), M.q);
  const int lo = j * alpha, hi = min(lo + alpha, L);
  if (t >= lo && t < hi) v = add_mod(v, mul_mod(pmod[t], s_from[idx], M), M.q);
  *b = v;
  b[(size_t)np * kN] = a;
}

__global__ void __launch_bounds__(TPB) secret_residue_kernel(
    const int8_t *s, uint64_t *out, const uint64_t *primes) {
  const int k = blockIdx.x * TPB + threadIdx.x;
  const int t = blockIdx.y;
  out[(size_t)t * kN + k] = signed_residue(s[k], primes[t]);
}

__global__ void __launch_bounds__(TPB) square_kernel(const uint64_t *a,
                                                     uint64_t *out,
                                                     const Mod *mods) {
  const int k = blockIdx.x * TPB + threadIdx.x;
  const int t = blockIdx.y;
  const size_t idx = (size_t)t * kN + k;
  out[idx] = mul_mod(a[idx], a[idx], mods[t]);
}

__global__ void __launch_bounds__(TPB) enc_error_kernel(uint64_t *c0, uint64_t seed,
                                                        uint64_t nonce,
                                                        const uint64_t *primes, int l) {
  const int k = blockIdx.x * TPB + threadIdx.x;
  const int e = cbd_at(seed, stream_id(TAG_ENC_E, nonce, nonce >> 24, 0), k);
  for (int i = 0; i < l; ++i) c0[(size_t)i * kN + k] = signed_residue(e, primes[i]);
}

// grid (N/TPB, l): c1 = a; c0 = e - a s + m
__global__ void __launch_bounds__(TPB) enc_finish_kernel(
    uint64_t *ct, const uint64_t *m, const uint64_t *s, uint64_t seed,
    uint64_t nonce, const Mod *mods, int l) {
  const int k = blockIdx.x * TPB + threadIdx.x;
  const int i = blockIdx.y;
  const Mod M = mods[i];
  const uint64_t a =
      uniform_at(seed, stream_id(TAG_ENC_A, nonce, nonce >> 24, i), k, M);
  const size_t idx = (size_t)i * kN + k;
  uint64_t v = sub_mod(ct[idx], mul_mod(a, s[idx], M), M.q);
  ct[idx] = add_mod(v, m[idx], M.q);
  ct[(size_t)l * kN + idx] = a;
}

__global__ void __launch_bounds__(TPB) decrypt_kernel(const uint64_t *ct,
                                                      const uint64_t *s,
                                                      uint64_t *m, const Mod *mods,
                                                      int l) {
  const int k = blockIdx.x * TPB + threadIdx.x;
  const int i = blockIdx.y;
  const Mod M = mods[i];
  const size_t idx = (size_t)i * kN + k;
  m[idx] = add_mod(ct[idx], mul_mod(ct[(size_t)l * kN + idx], s[idx], M), M.q);
}

__global__ void __launch_bounds__(TPB) permute_kernel(const uint64_t *in,
                                                      uint64_t *out, uint32_t g) {
  const int k = blockIdx.x * TPB + threadIdx.x;
  const size_t limb = blockIdx.y;
  uint32_t e = 2 * (__brev((uint32_t)k) >> 16) + 1;
  uint32_t e2 = (uint32_t)(((uint64_t)e * g) & (2 * kN - 1));
  out[limb * kN + k] = in[limb * kN + (__brev((e2 - 1) >> 1) >> 16)];
}

}  // namespace
}  // namespace b2f

using namespace b2f;

extern "C" {

int b2f_sample_secret(int log_n, uint64_t seed, int hamming, int8_t *s) {
  B2F_CHECK_ARG(s && log_n >= 1 && log_n <= 20, "b2f_sample_secret: bad argument");
  const uint64_t n = 1ull << log_n;
  B2F_CHECK_ARG(hamming >= 0 && (uint64_t)hamming <= n,
                "b2f_sample_secret: hamming weight %d > N", hamming);
  uint64_t blk[8];
  for (uint64_t k = 0; k < n; ++k) s[k] = 0;
  if (hamming == 0) {
    const uint64_t st = stream_id(TAG_SECRET, 1, 0, 0);
    for (uint64_t k = 0; k < n; ++k) {
      if (k % 8 == 0) chacha_block(seed, st, k / 8, blk);
      s[k] = (int8_t)((int)(blk[k % 8] % 3) - 1);
    }
    return B2F_OK;
  }
  std::vector<uint32_t> perm(n);
  for (uint64_t k = 0; k < n; ++k) perm[k] = (uint32_t)k;
  const uint64_t st = stream_id(TAG_SECRET, 0, 0, 0);
  for (uint64_t i = 0; i < (uint64_t)hamming; ++i) {
    if (i % 8 == 0) chacha_block(seed, st, i / 8, blk);
    const uint64_t w = blk[i % 8];
    const uint64_t j = i + (w >> 1) % (n - i);
    std::swap(perm[i], perm[j]);
    s[perm[i]] = (w & 1) ? -1 : 1;
  }
  return B2F_OK;
}

int b2f_secret_to_ntt(b2f_context *ctx, const int8_t *s_coeff, uint64_t *s_ntt,
                      void *stream) {
  B2F_CHECK_ARG(ctx && s_coeff && s_ntt, "b2f_secret_to_ntt: null argument");
  cudaStream_t st = (cudaStream_t)stream;
  int8_t *d = nullptr;
  B2F_CUDA(cudaMallocAsync(&d, kN, st));
  cudaError_t e = cudaMemcpyAsync(d, s_coeff, kN, cudaMemcpyHostToDevice, st);
  int rc = B2F_OK;
  if (e != cudaSuccess) rc = cuda_status(e, "b2f_secret_to_ntt copy");
  if (!rc) {
    secret_residue_kernel<<<dim3(kN / TPB, ctx->L + ctx->K), TPB, 0, st>>>(
        d, s_ntt, ctx->d_primes);
    note_launch();
    e = cudaGetLastError();
    if (e != cudaSuccess) rc = cuda_status(e, "secret_residue_kernel");
  }
  if (!rc) rc = ntt_polys(ctx, s_ntt, 1, ctx->L, ctx->K, 0, st);
  cudaFreeAsync(d, st);
  if (!rc) {
    e = cudaStreamSynchronize(st);  // the host secret may go away after return
    if (e != cudaSuccess) rc = cuda_status(e, "b2f_secret_to_ntt sync");
  }
  return rc;
}

int b2f_keygen_switch(b2f_context *ctx, const uint64_t *s_from,
                      const uint64_t *s_to, uint64_t seed, uint32_t tag,
                      uint64_t *key, void *stream) {
  B2F_RANGE("b2f_keygen_switch");
  B2F_CHECK_ARG(ctx && s_from && s_to && key, "b2f_keygen_switch: null argument");
  cudaStream_t st = (cudaStream_t)stream;
  const int np = ctx->L + ctx->K;
  key_error_kernel<<<dim3(kN / TPB, ctx->digits), TPB, 0, st>>>(key, seed, tag,
                                                                ctx->d_primes, np);
  B2F_LAUNCHED("key_error_kernel");
  // NTT of the error limbs: digit j poly 0 is the item, all np limbs
  std::vector<LimbJob> jobs(np);
  for (int t = 0; t < np; ++t)
    jobs[t] = LimbJob{(uint32_t)t, (uint32_t)t, (uint16_t)t, (uint16_t)t, 0};
  const LimbJob *d = job_table(ctx, {5}, jobs);
  if (!d) return B2F_ERR_NOMEM;
  const long long stride = 2LL * np * kN;
  int rc = launch_ntt(ctx, key, stride, key, stride, d, np, ctx->digits, 0,
                      nullptr, st);
  if (rc) return rc;
  key_finish_kernel<<<dim3(kN / TPB, np, ctx->digits), TPB, 0, st>>>(
      key, s_from, s_to, seed, tag, ctx->d_mod, ctx->d_pmod, ctx->L, np,
      ctx->alpha);
  B2F_LAUNCHED("key_finish_kernel");
  return B2F_OK;
}

int b2f_keygen_rotation(b2f_context *ctx, const uint64_t *s_ntt, uint64_t galois,
                        uint64_t seed, uint64_t *key, void *stream) {
  B2F_RANGE("b2f_keygen_rotation");
  B2F_CHECK_ARG(ctx && s_ntt && key, "b2f_keygen_rotation: null argument");
  const uint64_t m = 2ull * kN;
  B2F_CHECK_ARG((galois & 1) && galois < m, "b2f_keygen_rotation: bad galois");
  uint64_t ginv = 0;
  for (uint64_t x = 1; x < m; x += 2)
    if ((x * galois) % m == 1) {
      ginv = x;
      break;
    }
  cudaStream_t st = (cudaStream_t)stream;
  const int np = ctx->L + ctx->K;
  uint64_t *s_to = nullptr;
  B2F_CUDA(cudaMallocAsync(&s_to, (size_t)np * kN * 8, st));
  permute_kernel<<<dim3(kN / TPB, np), TPB, 0, st>>>(s_ntt, s_to, (uint32_t)ginv);
  int rc = B2F_OK;
  note_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) rc = cuda_status(e, "permute_kernel");
  if (!rc) rc = b2f_keygen_switch(ctx, s_ntt, s_to, seed, (uint32_t)galois, key, st);
  cudaFreeAsync(s_to, st);
  return rc;
}

int b2f_keygen_relin(b2f_context *ctx, const uint64_t *s_ntt, uint64_t seed,
                     uint64_t *key, void *stream) {
  B2F_RANGE("b2f_keygen_relin");
  B2F_CHECK_ARG(ctx && s_ntt && key, "b2f_keygen_relin: null argument");
  cudaStream_t st = (cudaStream_t)stream;
  const int np = ctx->L + ctx->K;
  uint64_t *s2 = nullptr;
  B2F_CUDA(cudaMallocAsync(&s2, (size_t)np * kN * 8, st));
  square_kernel<<<dim3(kN / TPB, np), TPB, 0, st>>>(s_ntt, s2, ctx->d_mod);
  int rc = B2F_OK;
  note_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) rc = cuda_status(e, "square_kernel");
  if (!rc) rc = b2f_keygen_switch(ctx, s2, s_ntt, seed, 0u, key, st);
  cudaFreeAsync(s2, st);
  return rc;
}

int b2f_encrypt(b2f_context *ctx, const uint64_t *m_ntt, int l,
                const uint64_t *s_ntt, uint64_t seed, uint64_t nonce,
                uint64_t *ct, void *stream) {
  B2F_RANGE("b2f_encrypt");
  B2F_CHECK_ARG(ctx && m_ntt && s_ntt && ct, "b2f_encrypt: null argument");
  B2F_CHECK_ARG(l >= 1 && l <= ctx->L, "b2f_encrypt: bad limbs %d", l);
  cudaStream_t st = (cudaStream_t)stream;
  enc_error_kernel<<<kN / TPB, TPB, 0, st>>>(ct, seed, nonce, ctx->d_primes, l);
  B2F_LAUNCHED("enc_error_kernel");
  int rc = ntt_polys(ctx, ct, 1, l, 0, 0, st);
  if (rc) return rc;
  enc_finish_kernel<<<dim3(kN / TPB, l), TPB, 0, st>>>(ct, m_ntt, s_ntt, seed, nonce,
                                                       ctx->d_mod, l);
  B2F_LAUNCHED("enc_finish_kernel");
  return B2F_OK;
}

int b2f_decrypt(b2f_context *ctx, const uint64_t *ct, int l, const uint64_t *s_ntt,
                uint64_t *m_ntt, void *stream) {
  B2F_RANGE("b2f_decrypt");
  B2F_CHECK_ARG(ctx && ct && s_ntt && m_ntt, "b2f_decrypt: null argument");
  B2F_CHECK_ARG(l >= 1 && l <= ctx->L, "b2f_decrypt: bad limbs %d", l);
  decrypt_kernel<<<dim3(kN / TPB, l), TPB, 0, (cudaStream_t)stream>>>(
      ct, s_ntt, m_ntt, ctx->d_mod, l);
  B2F_LAUNCHED("decrypt_kernel");
  return B2F_OK;
}

}  // extern "C"
