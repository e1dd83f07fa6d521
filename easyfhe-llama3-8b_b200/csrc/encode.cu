// CKKS encoding / decoding (special FFT of Cheon-Kim-Kim-Song 2017) and the
// feature-major BSGS diagonal packers.
//
// Every floating-point product and sum is an explicit round-to-nearest
// operation (__dmul_rn / __dadd_rn / __dsub_rn, no FMA contraction), in the
// same order as the CPU restatement, so encoded residues are bit-identical.
// Butterfly stages with half-length >= 1024 run as one global pass each;
// the remaining stages of a row run inside one CTA on a 2048-slot chunk in
// shared memory.
#include "b2f_internal.h"

namespace b2f {
namespace {

constexpr int TPB = 256;
constexpr int CHUNK = 2048;  // complex slots per shared-memory chunk

__device__ __forceinline__ double2 cmul(double2 a, double2 b) {
  return make_double2(__dsub_rn(__dmul_rn(a.x, b.x), __dmul_rn(a.y, b.y)),
                      __dadd_rn(__dmul_rn(a.x, b.y), __dmul_rn(a.y, b.x)));
}
__device__ __forceinline__ double2 cadd(double2 a, double2 b) {
  return make_double2(__dadd_rn(a.x, b.x), __dadd_rn(a.y, b.y));
}
__device__ __forceinline__ double2 csubd(double2 a, double2 b) {
  return make_double2(__dsub_rn(a.x, b.x), __dsub_rn(a.y, b.y));
}

// One butterfly of stage `len`.  inverse: (u,v) -> (u+v, (u-v) ksi[idx]),
// idx = (lenq - rot[j] % lenq) * M/lenq; forward: (u, v ksi) -> (u+w, u-w),
// idx = (rot[j] % lenq) * M/lenq.
__device__ __forceinline__ void fft_bfly(double2 &a, double2 &b, int j, int len,
                                         bool inverse, const double2 *ksi,
                                         const uint32_t *rot) {
  const uint32_t lenq = (uint32_t)len << 2, gap = (2u * kN) / lenq;
  const uint32_t r = __ldg(rot + j) % lenq;
  if (inverse) {
    const double2 w = __ldg(ksi + (size_t)(lenq - r) * gap);
    double2 u = cadd(a, b), d = csubd(a, b);
    a = u;
    b = cmul(d, w);
  } else {
    const double2 w = __ldg(ksi + (size_t)r * gap);
    double2 v = cmul(b, w);
    double2 u = a;
    a = cadd(u, v);
    b = csubd(u, v);
  }
}

// one global stage; grid (slots/2/TPB, rows)
__global__ void __launch_bounds__(TPB) fft_stage_kernel(
    double2 *v, int slots, int len, int inverse, const double2 *ksi,
    const uint32_t *rot) {
  const int t = blockIdx.x * TPB + threadIdx.x;
  if (t >= slots / 2) return;
  const int lenh = len >> 1;
  const int i = (t / lenh) * len, j = t % lenh;
  double2 *row = v + (size_t)blockIdx.y * slots;
  double2 a = row[i + j], b = row[i + j + lenh];
  fft_bfly(a, b, j, len, inverse != 0, ksi, rot);
  row[i + j] = a;
  row[i + j + lenh] = b;
}

// stages with len <= ch on one ch-slot chunk; grid (slots/ch, rows), ch/2 threads
__global__ void __launch_bounds__(CHUNK / 2) fft_chunk_kernel(
    double2 *v, int slots, int ch, int inverse, const double2 *ksi,
    const uint32_t *rot) {
  __shared__ double2 sm[CHUNK];
  double2 *base = v + (size_t)blockIdx.y * slots + (size_t)blockIdx.x * ch;
  for (int x = threadIdx.x; x < ch; x += blockDim.x) sm[x] = base[x];
  __syncthreads();
  const int t = threadIdx.x;
  if (inverse) {
    for (int len = ch; len >= 2; len >>= 1) {
      const int lenh = len >> 1, i = (t / lenh) * len, j = t % lenh;
      double2 a = sm[i + j], b = sm[i + j + lenh];
      fft_bfly(a, b, j, len, true, ksi, rot);
      sm[i + j] = a;
      sm[i + j + lenh] = b;
      __syncthreads();
    }
  } else {
    for (int len = 2; len <= ch; len <<= 1) {
      const int lenh = len >> 1, i = (t / lenh) * len, j = t % lenh;
      double2 a = sm[i + j], b = sm[i + j + lenh];
      fft_bfly(a, b, j, len, false, ksi, rot);
      sm[i + j] = a;
      sm[i + j + lenh] = b;
      __syncthreads();
    }
  }
  for (int x = threadIdx.x; x < ch; x += blockDim.x) base[x] = sm[x];
}

int run_fft(b2f_context *ctx, double2 *v, int rows, int slots, bool inverse,
            cudaStream_t s) {
  const int ch = slots < CHUNK ? slots : CHUNK;
  const dim3 gs((slots / 2 + TPB - 1) / TPB, rows);
  if (inverse) {
    for (int len = slots; len > ch; len >>= 1) {
      fft_stage_kernel<<<gs, TPB, 0, s>>>(v, slots, len, 1, ctx->d_ksi,
                                          ctx->d_rot_group);
      B2F_LAUNCHED("fft_stage_kernel");
    }
    if (ch >= 2) {
      fft_chunk_kernel<<<dim3(slots / ch, rows), ch / 2, 0, s>>>(
          v, slots, ch, 1, ctx->d_ksi, ctx->d_rot_group);
      B2F_LAUNCHED("fft_chunk_kernel");
    }
  } else {
    if (ch >= 2) {
      fft_chunk_kernel<<<dim3(slots / ch, rows), ch / 2, 0, s>>>(
          v, slots, ch, 0, ctx->d_ksi, ctx->d_rot_group);
      B2F_LAUNCHED("fft_chunk_kernel");
    }
    for (int len = 2 * ch; len <= slots; len <<= 1) {
      fft_stage_kernel<<<gs, TPB, 0, s>>>(v, slots, len, 0, ctx->d_ksi,
                                          ctx->d_rot_group);
      B2F_LAUNCHED("fft_stage_kernel");
    }
  }
  return B2F_OK;
}

__device__ __forceinline__ uint64_t pow2_mod(int e, const Mod &M) {
  uint64_t r = 1, b = 2;
  while (e) {
    if (e & 1) r = mul_mod(r, b, M);
    b = mul_mod(b, b, M);
    e >>= 1;
  }
  return r;
}

// exact residue of an integral double
__device__ __forceinline__ uint64_t double_mod(double v, const Mod &M) {
  if (v == 0.0) return 0;
  const bool neg = v < 0.0;
  const double a = fabs(v);
  uint64_t r;
  if (a < 9223372036854775808.0) {
    r = reduce128(0, (uint64_t)a, M);
  } else {
    int e;
    const double f = frexp(a, &e);
    const uint64_t mant = (uint64_t)ldexp(f, 53);
    r = mul_mod(reduce128(0, mant, M), pow2_mod(e - 53, M), M);
  }
  return neg ? (r ? M.q - r : 0) : r;
}

__device__ __forceinline__ uint32_t bitrev_n(uint32_t x, int bits) {
  return __brev(x) >> (32 - bits);
}

// bit-reverse, scale by 1/slots then by `scale`, round, reduce per limb.
// grid (N/TPB, limbs, rows); values v [rows][slots]; out [rows][limbs][N]
__global__ void __launch_bounds__(TPB) encode_round_kernel(
    const double2 *__restrict__ v, int slots, int log_slots, double inv_slots,
    double scale, uint64_t *__restrict__ out, int limbs, int q_limbs, int L,
    const Mod *__restrict__ mods) {
  const int k = blockIdx.x * TPB + threadIdx.x;
  const int t = blockIdx.y, r = blockIdx.z;
  const int half = kN / 2, gap = half / slots;
  double c = 0.0;
  if (k % gap == 0) {
    const int j = (k % half) / gap;
    const double2 z = v[(size_t)r * slots + bitrev_n((uint32_t)j, log_slots)];
    const double x = k < half ? z.x : z.y;
    c = rint(__dmul_rn(__dmul_rn(x, inv_slots), scale));
  }
  const Mod M = mods[t < q_limbs ? t : L + (t - q_limbs)];
  out[((size_t)r * limbs + t) * kN + k] = double_mod(c, M);
}

// decode: CRT of limbs 0 (and 1) in coefficient form, centred, / scale,
// written bit-reversed into v [slots]
__global__ void __launch_bounds__(TPB) decode_gather_kernel(
    const uint64_t *__restrict__ coef, int use, int slots, int log_slots,
    double scale, double2 *__restrict__ v, uint64_t q0, uint64_t q1,
    ulonglong2 q0inv_mod_q1) {
  const int j = blockIdx.x * TPB + threadIdx.x;
  if (j >= slots) return;
  const int half = kN / 2, gap = half / slots;
  double out[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int k = j * gap + h * half;
    const uint64_t a0 = coef[k];
    double val;
    if (use == 1) {
      val = a0 > q0 / 2 ? -(double)(q0 - a0) : (double)a0;
    } else {
      const uint64_t a1 = coef[kN + k];
      const uint64_t hh = shoup(sub_mod(a1, a0 % q1, q1), q0inv_mod_q1.x,
                                q0inv_mod_q1.y, q1);
      // v = a0 + q0 * hh as 128 bits; Q = q0 q1
      U128 vv = {a0, 0};
      mac128(vv, q0, hh);
      U128 Q = {0, 0};
      mac128(Q, q0, q1);
      // Q/2
      const uint64_t half_hi = Q.hi >> 1, half_lo = (Q.lo >> 1) | (Q.hi << 63);
      const bool negv = vv.hi > half_hi || (vv.hi == half_hi && vv.lo > half_lo);
      if (negv) {
        // Q - v
        const uint64_t lo = Q.lo - vv.lo;
        const uint64_t hi = Q.hi - vv.hi - (Q.lo < vv.lo);
        val = -((double)hi * 18446744073709551616.0 + (double)lo);
      } else {
        val = (double)vv.hi * 18446744073709551616.0 + (double)vv.lo;
      }
    }
    out[h] = val / scale;
  }
  v[bitrev_n((uint32_t)j, log_slots)] = make_double2(out[0], out[1]);
}

// ---- packers (feature-major BSGS diagonals) ----
// row(g,b)[s] = W[(f - g B) mod D, (f + b) mod D], f = s / lanes
__global__ void __launch_bounds__(TPB) pack_dense_kernel(
    const void *__restrict__ weight, int dtype, int D, int lanes, int B,
    int giant_base, int slots, double2 *__restrict__ out) {
  const int s = blockIdx.x * TPB + threadIdx.x;
  if (s >= slots) return;
  const int row = blockIdx.y;
  const int g = giant_base + row / B, b = row % B;
  const int f = s / lanes;
  int of = (f - g * B) % D;
  if (of < 0) of += D;
  const int inf = (f + b) % D;
  const size_t w = (size_t)of * D + inf;
  double2 v;
  if (dtype == 2) {
    v = reinterpret_cast<const double2 *>(weight)[w];
  } else if (dtype == 1) {
    v = make_double2((double)reinterpret_cast<const float *>(weight)[w], 0.0);
  } else {
    v = make_double2(reinterpret_cast<const double *>(weight)[w], 0.0);
  }
  out[(size_t)row * slots + s] = v;
}

struct StructSources {
  const void *src[3];
  long long rs[3], cs[3];
};

// same formula through the structured map; arithmetic in the reference
// kernel's order: (sum of selected source values) * (row_scale * col_scale)
__global__ void __launch_bounds__(TPB) pack_structured_kernel(
    StructSources S, int count, int dtype, const int64_t *__restrict__ rsrc,
    const int64_t *__restrict__ rrow, const double *__restrict__ rscale,
    const int64_t *__restrict__ isrc, const int64_t *__restrict__ irow,
    const double *__restrict__ iscale, const int64_t *__restrict__ column,
    const double *__restrict__ cscale, int D, int lanes, int B, int giant_base,
    int slots, double2 *__restrict__ out) {
  const int s = blockIdx.x * TPB + threadIdx.x;
  if (s >= slots) return;
  const int row = blockIdx.y;
  const int g = giant_base + row / B, b = row % B;
  const int f = s / lanes;
  int of = (f - g * B) % D;
  if (of < 0) of += D;
  const int inf = (f + b) % D;
  const int64_t col = column[inf];
  double re = 0.0, im = 0.0;
  if (col >= 0) {
    const int64_t rs = rsrc[of], is = isrc[of];
    for (int k = 0; k < count; ++k) {
      if (rs == k) {
        const long long idx = rrow[of] * S.rs[k] + col * S.cs[k];
        re = __dadd_rn(re, dtype ? (double)reinterpret_cast<const float *>(S.src[k])[idx]
                                 : reinterpret_cast<const double *>(S.src[k])[idx]);
      }
      if (is == k) {
        const long long idx = irow[of] * S.rs[k] + col * S.cs[k];
        im = __dadd_rn(im, dtype ? (double)reinterpret_cast<const float *>(S.src[k])[idx]
                                 : reinterpret_cast<const double *>(S.src[k])[idx]);
      }
    }
  }
  const double cs = cscale[inf];
  re = __dmul_rn(re, __dmul_rn(rscale[of], cs));
  im = __dmul_rn(im, __dmul_rn(iscale[of], cs));
  out[(size_t)row * slots + s] = make_double2(re, im);
}

bool pow2(int x) { return x > 0 && (x & (x - 1)) == 0; }
int log2i(int x) {
  int r = 0;
  while ((1 << r) < x) ++r;
  return r;
}

}  // namespace
}  // namespace b2f

using namespace b2f;

extern "C" {

size_t b2f_encode_workspace(const b2f_context *ctx, int num_rows, int slots) {
  if (!ctx || num_rows < 0 || slots < 1) return 0;
  return (size_t)num_rows * slots * sizeof(double2) + 256;
}

int b2f_encode(b2f_context *ctx, const double *values, int num_rows, int slots,
               double scale, int q_limbs, int p_limbs, uint64_t *out, void *ws,
               size_t ws_bytes, void *stream) {
  B2F_RANGE("b2f_encode");
  B2F_CHECK_ARG(ctx && values && out, "b2f_encode: null argument");
  B2F_CHECK_ARG(pow2(slots) && slots <= kN / 2, "b2f_encode: slots %d must be a "
                "power of two <= N/2", slots);
  B2F_CHECK_ARG(q_limbs >= 1 && q_limbs <= ctx->L && p_limbs >= 0 &&
                    p_limbs <= ctx->K,
                "b2f_encode: bad limbs q=%d p=%d", q_limbs, p_limbs);
  B2F_CHECK_ARG(scale > 0.0 && std::isfinite(scale), "b2f_encode: bad scale");
  if (num_rows <= 0) return B2F_OK;
  cudaStream_t s = (cudaStream_t)stream;
  const size_t need = b2f_encode_workspace(ctx, num_rows, slots);
  void *owned = nullptr;
  if (!ws) {
    B2F_CUDA(cudaMallocAsync(&owned, need, s));
    ws = owned;
  } else {
    B2F_CHECK_ARG(ws_bytes >= need, "b2f_encode: workspace %zu < %zu", ws_bytes, need);
  }
  double2 *v = static_cast<double2 *>(ws);
  int rc = B2F_OK;
  cudaError_t e = cudaMemcpyAsync(v, values, (size_t)num_rows * slots * 16,
                                  cudaMemcpyDeviceToDevice, s);
  if (e != cudaSuccess) rc = cuda_status(e, "b2f_encode copy");
  if (!rc) rc = run_fft(ctx, v, num_rows, slots, true, s);
  const int limbs = q_limbs + p_limbs;
  if (!rc) {
    encode_round_kernel<<<dim3(kN / TPB, limbs, num_rows), TPB, 0, s>>>(
        v, slots, log2i(slots), 1.0 / (double)slots, scale, out, limbs, q_limbs,
        ctx->L, ctx->d_mod);
    note_launch();
    e = cudaGetLastError();
    if (e != cudaSuccess) rc = cuda_status(e, "encode_round_kernel");
  }
  if (!rc) rc = ntt_polys(ctx, out, num_rows, q_limbs, p_limbs, 0, s);
  if (owned) cudaFreeAsync(owned, s);
  return rc;
}

size_t b2f_decode_workspace(const b2f_context *ctx, int slots) {
  if (!ctx) return 0;
  (void)slots;
  return 2 * (size_t)kN * 8 + 256;
}

int b2f_decode(b2f_context *ctx, const uint64_t *pt, int l, int slots,
               double scale, double *values, void *ws, size_t ws_bytes,
               void *stream) {
  B2F_RANGE("b2f_decode");
  B2F_CHECK_ARG(ctx && pt && values, "b2f_decode: null argument");
  B2F_CHECK_ARG(pow2(slots) && slots <= kN / 2, "b2f_decode: bad slots %d", slots);
  B2F_CHECK_ARG(l >= 1 && l <= ctx->L, "b2f_decode: bad limbs %d", l);
  cudaStream_t s = (cudaStream_t)stream;
  const size_t need = b2f_decode_workspace(ctx, slots);
  void *owned = nullptr;
  if (!ws) {
    B2F_CUDA(cudaMallocAsync(&owned, need, s));
    ws = owned;
  } else {
    B2F_CHECK_ARG(ws_bytes >= need, "b2f_decode: workspace %zu < %zu", ws_bytes, need);
  }
  uint64_t *coef = static_cast<uint64_t *>(ws);
  const int use = l < 2 ? l : 2;
  int rc = B2F_OK;
  cudaError_t e = cudaMemcpyAsync(coef, pt, (size_t)use * kN * 8,
                                  cudaMemcpyDeviceToDevice, s);
  if (e != cudaSuccess) rc = cuda_status(e, "b2f_decode copy");
  if (!rc) rc = ntt_polys(ctx, coef, 1, use, 0, 1, s);
  if (!rc) {
    const uint64_t q0 = ctx->primes[0], q1 = ctx->L > 1 ? ctx->primes[1] : 3;
    unsigned __int128 r = 1;
    // q0^-1 mod q1 by Fermat
    {
      uint64_t base = q0 % q1, ex = q1 - 2, acc = 1;
      while (ex) {
        if (ex & 1) acc = (uint64_t)(((unsigned __int128)acc * base) % q1);
        base = (uint64_t)(((unsigned __int128)base * base) % q1);
        ex >>= 1;
      }
      r = acc;
    }
    const uint64_t inv = (uint64_t)r;
    const ulonglong2 invp =
        make_ulonglong2(inv, (uint64_t)(((unsigned __int128)inv << 64) / q1));
    decode_gather_kernel<<<(slots + TPB - 1) / TPB, TPB, 0, s>>>(
        coef, use, slots, log2i(slots), scale, reinterpret_cast<double2 *>(values),
        q0, q1, invp);
    note_launch();
    e = cudaGetLastError();
    if (e != cudaSuccess) rc = cuda_status(e, "decode_gather_kernel");
  }
  if (!rc) rc = run_fft(ctx, reinterpret_cast<double2 *>(values), 1, slots, false, s);
  if (owned) cudaFreeAsync(owned, s);
  return rc;
}

int b2f_pack_diagonals(b2f_context *ctx, const void *weight, int dtype,
                       int dimension, int token_lanes, int baby_steps,
                       int giant_base, int giant_count, int slots, double *out,
                       void *stream) {
  B2F_RANGE("b2f_pack_diagonals");
  B2F_CHECK_ARG(ctx && weight && out, "b2f_pack_diagonals: null argument");
  B2F_CHECK_ARG(dtype >= 0 && dtype <= 2, "b2f_pack_diagonals: bad dtype %d", dtype);
  B2F_CHECK_ARG(slots > 0 && dimension > 0 && token_lanes > 0 &&
                    (long long)dimension * token_lanes == slots,
                "TokenLane GPU packing requires dimension*token_lanes == slots, "
                "got %d*%d != %d", dimension, token_lanes, slots);
  B2F_CHECK_ARG(baby_steps > 0 && giant_base >= 0 && giant_count > 0,
                "baby_steps/giant_count must be positive and giant_base "
                "non-negative");
  const int rows = giant_count * baby_steps;
  pack_dense_kernel<<<dim3((slots + TPB - 1) / TPB, rows), TPB, 0,
                      (cudaStream_t)stream>>>(weight, dtype, dimension, token_lanes,
                                              baby_steps, giant_base, slots,
                                              reinterpret_cast<double2 *>(out));
  B2F_LAUNCHED("pack_dense_kernel");
  return B2F_OK;
}

int b2f_pack_structured(b2f_context *ctx, const void *const *sources,
                        const int64_t *strides, int source_count, int dtype,
                        const int64_t *real_source, const int64_t *real_row,
                        const double *real_scale, const int64_t *imag_source,
                        const int64_t *imag_row, const double *imag_scale,
                        const int64_t *column, const double *column_scale,
                        int dimension, int token_lanes, int baby_steps,
                        int giant_base, int giant_count, int slots, double *out,
                        void *stream) {
  B2F_RANGE("b2f_pack_structured");
  B2F_CHECK_ARG(ctx && sources && strides && out && real_source && real_row &&
                    real_scale && imag_source && imag_row && imag_scale &&
                    column && column_scale,
                "b2f_pack_structured: null argument");
  B2F_CHECK_ARG(source_count >= 1 && source_count <= 3,
                "structured GPU packer requires one to three sources.");
  B2F_CHECK_ARG(dtype == 0 || dtype == 1,
                "structured GPU sources must use float32 or float64");
  B2F_CHECK_ARG(slots > 0 && dimension > 0 && token_lanes > 0 &&
                    (long long)dimension * token_lanes == slots,
                "structured TokenLane packing requires dimension*token_lanes "
                "== slots, got %d*%d != %d", dimension, token_lanes, slots);
  B2F_CHECK_ARG(baby_steps > 0 && giant_base >= 0 && giant_count > 0,
                "baby_steps/giant_count must be positive and giant_base "
                "non-negative");
  StructSources S{};
  for (int k = 0; k < 3; ++k) {
    const int kk = k < source_count ? k : 0;
    S.src[k] = sources[kk];
    B2F_CHECK_ARG(S.src[k], "b2f_pack_structured: source %d is null", kk);
    S.rs[k] = strides[2 * kk];
    S.cs[k] = strides[2 * kk + 1];
  }
  const int rows = giant_count * baby_steps;
  pack_structured_kernel<<<dim3((slots + TPB - 1) / TPB, rows), TPB, 0,
                           (cudaStream_t)stream>>>(
      S, source_count, dtype, real_source, real_row, real_scale, imag_source,
      imag_row, imag_scale, column, column_scale, dimension, token_lanes,
      baby_steps, giant_base, slots, reinterpret_cast<double2 *>(out));
  B2F_LAUNCHED("pack_structured_kernel");
  return B2F_OK;
}

}  // extern "C"
