// Level management, limb-wise arithmetic and the baby-step/giant-step
// plaintext x ciphertext multiply-accumulate.
#include "b2f_internal.h"

namespace b2f {
size_t rotate_workspace(const b2f_context *ctx, int cts, int l);
namespace {

constexpr int TPB = 256;
constexpr int GMAX = 8;  // giants accumulated per MAC pass

__device__ __forceinline__ uint32_t brv16(uint32_t x) { return __brev(x) >> 16; }

// rescale step 2: centred lift of the last limb (coefficient form) to q_i
// grid (N/TPB, l-1, polys)
__global__ void __launch_bounds__(TPB) rescale_lift_kernel(
    const uint64_t *__restrict__ last, uint64_t *__restrict__ lifted,
    const uint64_t *__restrict__ primes, const uint64_t *__restrict__ qlast_mod,
    int l, uint64_t q_last) {
  const int n = blockIdx.x * TPB + threadIdx.x;
  const int i = blockIdx.y, p = blockIdx.z;
  const uint64_t v = last[(size_t)p * kN + n];
  const uint64_t qi = primes[i];
  uint64_t r = v % qi;
  if (v > (q_last - 1) / 2) r = sub_mod(r, qlast_mod[i], qi);
  lifted[((size_t)p * (l - 1) + i) * kN + n] = r;
}

// rescale step 4: out = (in - lifted) * q_last^-1
__global__ void __launch_bounds__(TPB) rescale_combine_kernel(
    const uint64_t *__restrict__ in, const uint64_t *__restrict__ lifted,
    uint64_t *__restrict__ out, const uint64_t *__restrict__ primes,
    const ulonglong2 *__restrict__ inv, int l) {
  const int n = blockIdx.x * TPB + threadIdx.x;
  const int i = blockIdx.y, p = blockIdx.z;
  const uint64_t q = primes[i];
  const ulonglong2 w = inv[i];
  const uint64_t a = in[((size_t)p * l + i) * kN + n];
  const uint64_t b = lifted[((size_t)p * (l - 1) + i) * kN + n];
  out[((size_t)p * (l - 1) + i) * kN + n] = shoup(sub_mod(a, b, q), w.x, w.y, q);
}

// ModRaise step 2: limb 0 of every poly holds coefficients mod q_0; write
// their centred lift modulo q_t into limbs t = 1 .. l_out-1.
// grid (N/TPB, l_out-1, polys)
__global__ void __launch_bounds__(TPB) modraise_lift_kernel(
    uint64_t *__restrict__ data, const uint64_t *__restrict__ primes, int l_out) {
  const int n = blockIdx.x * TPB + threadIdx.x;
  const int t = blockIdx.y + 1, p = blockIdx.z;
  const uint64_t q0 = primes[0], qt = primes[t];
  const uint64_t v = data[(size_t)p * l_out * kN + n];
  uint64_t r;
  if (v > (q0 - 1) / 2) {
    const uint64_t m = (q0 - v) % qt;
    r = m ? qt - m : 0;
  } else {
    r = v % qt;
  }
  data[((size_t)p * l_out + t) * kN + n] = r;
}

// Tensor product of ciphertext pairs: (a0 b0, a0 b1 + a1 b0, a1 b1), the
// middle term accumulated in 128 bits and reduced once.  grid (N/TPB, l, cts)
__global__ void __launch_bounds__(TPB) tensor_kernel(
    const uint64_t *__restrict__ a, const uint64_t *__restrict__ b,
    uint64_t *__restrict__ out, const Mod *__restrict__ mods, int l) {
  const int n = blockIdx.x * TPB + threadIdx.x;
  const int i = blockIdx.y, ct = blockIdx.z;
  const size_t lim = (size_t)l * kN, off = (size_t)i * kN + n;
  const size_t in = (size_t)ct * 2 * lim + off;
  const Mod M = mods[i];
  const uint64_t a0 = a[in], a1 = a[in + lim], b0 = b[in], b1 = b[in + lim];
  U128 mid = {0, 0};
  mac128(mid, a0, b1);
  mac128(mid, a1, b0);
  const size_t o = (size_t)ct * 3 * lim + off;
  out[o] = mul_mod(a0, b0, M);
  out[o + lim] = reduce128(mid.hi, mid.lo, M);
  out[o + 2 * lim] = mul_mod(a1, b1, M);
}

// grid (N/TPB, l, polys); limb i is prime i below ql, prime L + i - ql after
// it (the extended basis Q_ql u P; ql = l outside it)
__global__ void __launch_bounds__(TPB) elementwise_kernel(
    int op, const uint64_t *__restrict__ a, const uint64_t *__restrict__ b,
    uint64_t *__restrict__ out, const Mod *__restrict__ mods, int l,
    int b_polys, int ql, int L) {
  const int n = blockIdx.x * TPB + threadIdx.x;
  const int i = blockIdx.y, p = blockIdx.z;
  const size_t ia = ((size_t)p * l + i) * kN + n;
  const size_t ib = ((size_t)(b_polys == 1 ? 0 : p) * l + i) * kN + n;
  const Mod M = mods[i < ql ? i : L + i - ql];
  const uint64_t x = a[ia], y = b[ib];
  uint64_t r;
  if (op == 0)
    r = add_mod(x, y, M.q);
  else if (op == 1)
    r = sub_mod(x, y, M.q);
  else
    r = mul_mod(x, y, M);
  out[ia] = r;
}

__global__ void __launch_bounds__(TPB) mul_i_kernel(
    const uint64_t *__restrict__ a, uint64_t *__restrict__ out,
    const ulonglong2 *__restrict__ factor, const uint64_t *__restrict__ primes,
    int l, int negative) {
  const int k = blockIdx.x * TPB + threadIdx.x;
  const int i = blockIdx.y, p = blockIdx.z;
  const size_t idx = ((size_t)p * l + i) * kN + k;
  const uint64_t q = primes[i];
  const ulonglong2 w = factor[i];
  const uint32_t e = 2 * brv16(k) + 1;
  // evaluation at psi^e of X^(N/2) is omega^e, omega = psi^(N/2) (order 4)
  const bool minus = ((e & 3) == 3) != (negative != 0);
  uint64_t r = shoup(a[idx], w.x, w.y, q);
  out[idx] = (minus && r) ? q - r : r;
}

struct ScalarArgs {
  ulonglong2 mul[64];
  uint64_t add[64];
  int has_mul, has_add, add_poly;
};

__global__ void __launch_bounds__(TPB) scalar_kernel(
    const uint64_t *__restrict__ a, uint64_t *__restrict__ out,
    const uint64_t *__restrict__ primes, int l, ScalarArgs S) {
  const int k = blockIdx.x * TPB + threadIdx.x;
  const int i = blockIdx.y, p = blockIdx.z;
  const size_t idx = ((size_t)p * l + i) * kN + k;
  const uint64_t q = primes[i];
  uint64_t r = a[idx];
  if (S.has_mul) r = shoup(r, S.mul[i].x, S.mul[i].y, q);
  const bool add_here = S.add_poly == -1 || S.add_poly == p ||
                        (S.add_poly == -2 && (p & 1) == 0);
  if (S.has_add && add_here) r = add_mod(r, S.add[i], q);
  out[idx] = r;
}

// out[c][p][i] = sum_k w_k[i] * term_k[c][p][i] (mod q_i): ciphertexts
// (or batches) of different limb counts combined with per-limb scalar weights
// in one pass.  The weights travel by value (Barrett products: the kernel is
// bound by reading the terms).  grid (N/TPB, l, cts * polys)
constexpr int LC_MAX = 8;    // terms
constexpr int LC_LMAX = 40;  // limbs
struct LinTerms {
  const uint64_t *in[LC_MAX];
  int limbs[LC_MAX];
  int count;
  uint64_t w[LC_MAX][LC_LMAX];
};
__global__ void __launch_bounds__(TPB) linear_combination_kernel(
    const LinTerms T, uint64_t *__restrict__ out, const Mod *__restrict__ mods, int l) {
  const int n = blockIdx.x * TPB + threadIdx.x;
  const int i = blockIdx.y, cp = blockIdx.z;  // cp = ciphertext * polys + poly
  const Mod M = mods[i];
  U128 acc = {0, 0};
  for (int k = 0; k < T.count; ++k)
    mac128(acc, T.in[k][((size_t)cp * T.limbs[k] + i) * kN + n], T.w[k][i]);
  out[((size_t)cp * l + i) * kN + n] = reduce128(acc.hi, acc.lo, M);
}

// out[ct][g] (2 polys, l limbs; giant-major [g][ct] when giant_major) =
// sum_b pt[g0+g][b] * babies[ct][b].  grid (cts, N/TPB, l): the ciphertexts
// of a batch are the fastest grid axis, so they read each plaintext tile
// while it is in L2 and the plaintext rows stream from HBM once per batch.
// Up to GMAX giants per launch; babies are taken two at a time with every
// load of the pair issued before its multiplies.  l is the limbs of the
// layout; limb i is prime i for i < ql and prime L + i - ql after it (the
// extended basis Q_ql u P: ql = l outside it).
__global__ void __launch_bounds__(TPB) mac_kernel(
    const uint64_t *__restrict__ babies, int baby_count,
    const uint64_t *__restrict__ pts, int g0, int G, int l,
    uint64_t *__restrict__ out, int out_giants, int giant_major,
    const Mod *__restrict__ mods, int ql, int L) {
  constexpr int BU = 2;
  const int n = blockIdx.y * TPB + threadIdx.x;
  const int i = blockIdx.z, ct = blockIdx.x, cts = gridDim.x;
  const Mod M = mods[i < ql ? i : L + i - ql];
  const size_t limb = (size_t)i * kN + n;
  const size_t ct_words = 2 * (size_t)l * kN, pt_words = (size_t)l * kN;
  const uint64_t *bb = babies + (size_t)ct * baby_count * ct_words + limb;
  const uint64_t *pp = pts + (size_t)g0 * baby_count * pt_words + limb;
  U128 acc[GMAX][2];
#pragma unroll
  for (int g = 0; g < GMAX; ++g) acc[g][0] = acc[g][1] = U128{0, 0};
  for (int b = 0; b < baby_count; b += BU) {
    uint64_t c0[BU], c1[BU], w[BU][GMAX];
#pragma unroll
    for (int u = 0; u < BU; ++u) {
      if (b + u < baby_count) {
        c0[u] = bb[(size_t)(b + u) * ct_words];
        c1[u] = bb[(size_t)(b + u) * ct_words + pt_words];
#pragma unroll
        for (int g = 0; g < GMAX; ++g)
          if (g < G) w[u][g] = __ldg(pp + ((size_t)g * baby_count + b + u) * pt_words);
      }
    }
#pragma unroll
    for (int u = 0; u < BU; ++u) {
      if (b + u < baby_count) {
#pragma unroll
        for (int g = 0; g < GMAX; ++g) {
          if (g < G) {
            mac128(acc[g][0], c0[u], w[u][g]);
            mac128(acc[g][1], c1[u], w[u][g]);
          }
        }
      }
    }
    // keep the 128-bit sums far from overflow for long baby runs
    if (((b + BU) & 31) == 0) {
#pragma unroll
      for (int g = 0; g < GMAX; ++g)
        if (g < G) {
          acc[g][0] = U128{reduce128(acc[g][0].hi, acc[g][0].lo, M), 0};
          acc[g][1] = U128{reduce128(acc[g][1].hi, acc[g][1].lo, M), 0};
        }
    }
  }
#pragma unroll
  for (int g = 0; g < GMAX; ++g)
    if (g < G) {
      const size_t slot = giant_major ? (size_t)(g0 + g) * cts + ct
                                      : (size_t)ct * out_giants + g0 + g;
      uint64_t *o = out + slot * ct_words + limb;
      o[0] = reduce128(acc[g][0].hi, acc[g][0].lo, M);
      o[pt_words] = reduce128(acc[g][1].hi, acc[g][1].lo, M);
    }
}

// out[g] = sum over i in group g of ct[i] * pt[i]; cts [count][2][limbs],
// pts rows of pt_stride limbs (the first `limbs` used).  grid (N/TPB, limbs,
// groups); limb t is prime t < q_limbs ? t : L + t - q_limbs.
__global__ void __launch_bounds__(TPB) pairwise_mac_kernel(
    const uint64_t *__restrict__ cts, const uint64_t *__restrict__ pts,
    uint64_t *__restrict__ out, int per_group, int limbs, int q_limbs,
    int pt_stride, int L, const Mod *__restrict__ mods) {
  const int n = blockIdx.x * TPB + threadIdx.x;
  const int t = blockIdx.y, g = blockIdx.z;
  const Mod M = mods[t < q_limbs ? t : L + (t - q_limbs)];
  const size_t ct_words = 2 * (size_t)limbs * kN;
  U128 a0 = {0, 0}, a1 = {0, 0};
  for (int j = 0; j < per_group; ++j) {
    const size_t i = (size_t)g * per_group + j;
    const uint64_t w = __ldg(pts + (i * pt_stride + t) * kN + n);
    const uint64_t *c = cts + i * ct_words + (size_t)t * kN + n;
    mac128(a0, c[0], w);
    mac128(a1, c[(size_t)limbs * kN], w);
    if ((j & 31) == 31) {
      a0 = U128{reduce128(a0.hi, a0.lo, M), 0};
      a1 = U128{reduce128(a1.hi, a1.lo, M), 0};
    }
  }
  uint64_t *o = out + (size_t)g * ct_words + (size_t)t * kN + n;
  o[0] = reduce128(a0.hi, a0.lo, M);
  o[(size_t)limbs * kN] = reduce128(a1.hi, a1.lo, M);
}

int launch_mac(b2f_context *ctx, const uint64_t *babies, int baby_count,
               const uint64_t *pts, int giant_count, int l, uint64_t *out,
               int cts, cudaStream_t s, int giant_major = 0, int ql = -1) {
  if (ql < 0) ql = l;
  const bool mma = mac_mma_eligible(ctx, baby_count, l, ql, cts);
  for (int g0 = 0; g0 < giant_count; g0 += GMAX) {
    const int G = std::min(GMAX, giant_count - g0);
    if (mma && G >= 4) {
      const int rc = launch_mac_mma(ctx, babies, baby_count, pts, g0, G, l, out,
                                    giant_count, cts, giant_major, ql, s);
      if (rc > 0) return rc;
      if (rc == 0) continue;
    }
    mac_kernel<<<dim3(cts, kN / TPB, l), TPB, 0, s>>>(
        babies, baby_count, pts, g0, G, l, out, giant_count, giant_major,
        ctx->d_mod, ql, ctx->L);
    B2F_LAUNCHED("mac_kernel");
  }
  return B2F_OK;
}

}  // namespace
}  // namespace b2f

using namespace b2f;

extern "C" {

size_t b2f_rescale_workspace(const b2f_context *ctx, int num_polys, int l) {
  if (!ctx || l < 2 || num_polys < 0) return 0;
  return ((size_t)num_polys * kN + (size_t)num_polys * (l - 1) * kN) * 8 + 512;
}

int b2f_rescale(b2f_context *ctx, const uint64_t *in, uint64_t *out,
                int num_polys, int l, void *ws, size_t ws_bytes, void *stream) {
  B2F_RANGE("b2f_rescale");
  B2F_CHECK_ARG(ctx && in && out && num_polys >= 0, "b2f_rescale: null argument");
  B2F_CHECK_ARG(l >= 2 && l <= ctx->L, "b2f_rescale: needs 2..%d limbs, got %d",
                ctx->L, l);
  B2F_CHECK_ARG(in != out, "b2f_rescale: in-place rescale is not supported");
  if (!num_polys) return B2F_OK;
  cudaStream_t s = (cudaStream_t)stream;
  const size_t need = b2f_rescale_workspace(ctx, num_polys, l);
  void *owned = nullptr;
  if (!ws) {
    B2F_CUDA(cudaMallocAsync(&owned, need, s));
    ws = owned;
  } else {
    B2F_CHECK_ARG(ws_bytes >= need, "b2f_rescale: workspace %zu < %zu", ws_bytes,
                  need);
  }
  uint64_t *last = static_cast<uint64_t *>(ws);
  int rc;
  {
    std::vector<LimbJob> j = {
        LimbJob{(uint32_t)(l - 1), 0u, (uint16_t)(l - 1), (uint16_t)(l - 1), 0}};
    const LimbJob *d = job_table(ctx, {4, l}, j);
    rc = d ? launch_ntt(ctx, in, (long long)l * kN, last, kN, d, 1, num_polys, 1,
                        nullptr, s)
           : B2F_ERR_NOMEM;
  }
  // lift, NTT and combine in one launch (ntt_rescale)
  if (!rc) rc = ntt_rescale(ctx, last, in, out, num_polys, l, s);
  if (owned) cudaFreeAsync(owned, s);
  return rc;
}

int b2f_modraise(b2f_context *ctx, const uint64_t *in, int num_polys, int l_out,
                 uint64_t *out, void *stream) {
  B2F_RANGE("b2f_modraise");
  B2F_CHECK_ARG(ctx && in && out && num_polys >= 0, "b2f_modraise: null argument");
  B2F_CHECK_ARG(l_out >= 1 && l_out <= ctx->L, "b2f_modraise: bad target limbs %d", l_out);
  B2F_CHECK_ARG(in != out, "b2f_modraise: in-place ModRaise is not supported");
  if (!num_polys) return B2F_OK;
  cudaStream_t s = (cudaStream_t)stream;
  std::vector<LimbJob> j = {LimbJob{0u, 0u, 0, 0, 0}};
  const LimbJob *d = job_table(ctx, {6}, j);
  if (!d) return B2F_ERR_NOMEM;
  int rc = launch_ntt(ctx, in, kN, out, (long long)l_out * kN, d, 1, num_polys, 1,
                      nullptr, s);
  if (rc) return rc;
  if (l_out > 1) {
    modraise_lift_kernel<<<dim3(kN / TPB, l_out - 1, num_polys), TPB, 0, s>>>(
        out, ctx->d_primes, l_out);
    B2F_LAUNCHED("modraise_lift_kernel");
  }
  return ntt_polys(ctx, out, num_polys, l_out, 0, 0, s);
}

int b2f_drop_limbs(b2f_context *ctx, const uint64_t *in, uint64_t *out,
                   int num_polys, int l_in, int l_out, void *stream) {
  B2F_CHECK_ARG(ctx && in && out && num_polys >= 0, "b2f_drop_limbs: null argument");
  B2F_CHECK_ARG(l_out >= 1 && l_out <= l_in && l_in <= ctx->L,
                "b2f_drop_limbs: cannot go from %d to %d limbs", l_in, l_out);
  if (!num_polys) return B2F_OK;
  B2F_CUDA(cudaMemcpy2DAsync(out, (size_t)l_out * kN * 8, in, (size_t)l_in * kN * 8,
                             (size_t)l_out * kN * 8, num_polys,
                             cudaMemcpyDeviceToDevice, (cudaStream_t)stream));
  return B2F_OK;
}

int b2f_elementwise(b2f_context *ctx, int op, const uint64_t *a,
                    const uint64_t *b, uint64_t *out, int num_polys, int l,
                    int b_polys, void *stream) {
  B2F_CHECK_ARG(ctx && a && b && out, "b2f_elementwise: null argument");
  B2F_CHECK_ARG(op >= 0 && op <= 2, "b2f_elementwise: unknown op %d", op);
  B2F_CHECK_ARG(l >= 1 && l <= ctx->L + ctx->K, "b2f_elementwise: bad limbs %d", l);
  B2F_CHECK_ARG(b_polys == 1 || b_polys == num_polys,
                "b2f_elementwise: b_polys must be 1 or num_polys");
  if (num_polys <= 0) return B2F_OK;
  elementwise_kernel<<<dim3(kN / TPB, l, num_polys), TPB, 0, (cudaStream_t)stream>>>(
      op, a, b, out, ctx->d_mod, l, b_polys, l, ctx->L);
  B2F_LAUNCHED("elementwise_kernel");
  return B2F_OK;
}

int b2f_elementwise_ext(b2f_context *ctx, int op, const uint64_t *a,
                        const uint64_t *b, uint64_t *out, int num_polys, int q_limbs,
                        int p_limbs, void *stream) {
  B2F_CHECK_ARG(ctx && a && b && out, "b2f_elementwise_ext: null argument");
  B2F_CHECK_ARG(op >= 0 && op <= 2, "b2f_elementwise_ext: unknown op %d", op);
  B2F_CHECK_ARG(q_limbs >= 1 && q_limbs <= ctx->L && p_limbs >= 0 && p_limbs <= ctx->K,
                "b2f_elementwise_ext: bad limbs q=%d p=%d", q_limbs, p_limbs);
  if (num_polys <= 0) return B2F_OK;
  const int l = q_limbs + p_limbs;
  elementwise_kernel<<<dim3(kN / TPB, l, num_polys), TPB, 0, (cudaStream_t)stream>>>(
      op, a, b, out, ctx->d_mod, l, num_polys, q_limbs, ctx->L);
  B2F_LAUNCHED("elementwise_kernel");
  return B2F_OK;
}

int b2f_mul_i(b2f_context *ctx, const uint64_t *a, uint64_t *out, int num_polys,
              int l, int negative, void *stream) {
  B2F_CHECK_ARG(ctx && a && out, "b2f_mul_i: null argument");
  B2F_CHECK_ARG(l >= 1 && l <= ctx->L, "b2f_mul_i: bad limbs %d", l);
  if (num_polys <= 0) return B2F_OK;
  mul_i_kernel<<<dim3(kN / TPB, l, num_polys), TPB, 0, (cudaStream_t)stream>>>(
      a, out, ctx->d_i_factor, ctx->d_primes, l, negative);
  B2F_LAUNCHED("mul_i_kernel");
  return B2F_OK;
}

int b2f_tensor(b2f_context *ctx, const uint64_t *a, const uint64_t *b,
               uint64_t *out, int num_cts, int l, void *stream) {
  B2F_RANGE("b2f_tensor");
  B2F_CHECK_ARG(ctx && a && b && out && num_cts >= 0, "b2f_tensor: null argument");
  B2F_CHECK_ARG(l >= 1 && l <= ctx->L, "b2f_tensor: bad limbs %d", l);
  B2F_CHECK_ARG(out != a && out != b, "b2f_tensor: output overlaps an input");
  if (!num_cts) return B2F_OK;
  tensor_kernel<<<dim3(kN / TPB, l, num_cts), TPB, 0, (cudaStream_t)stream>>>(
      a, b, out, ctx->d_mod, l);
  B2F_LAUNCHED("tensor_kernel");
  return B2F_OK;
}

int b2f_linear_combination(b2f_context *ctx, int num_terms,
                           const uint64_t *const *terms, const int *term_limbs,
                           const uint64_t *weights, int num_cts, int polys, int l,
                           uint64_t *out, void *stream) {
  B2F_RANGE("b2f_linear_combination");
  B2F_CHECK_ARG(ctx && terms && term_limbs && weights && out,
                "b2f_linear_combination: null argument");
  B2F_CHECK_ARG(num_terms >= 1 && num_cts >= 0 && polys >= 1 && polys <= 3 && l >= 1 &&
                    l <= ctx->L,
                "b2f_linear_combination: bad shape (terms=%d, l=%d, cts=%d, polys=%d)",
                num_terms, l, num_cts, polys);
  if (num_terms > LC_MAX || l > LC_LMAX) {
    set_error("b2f_linear_combination: at most %d terms of %d limbs", LC_MAX, LC_LMAX);
    return B2F_ERR_UNSUPPORTED;
  }
  LinTerms T{};
  T.count = num_terms;
  for (int k = 0; k < num_terms; ++k) {
    B2F_CHECK_ARG(terms[k] && term_limbs[k] >= l && term_limbs[k] <= ctx->L,
                  "b2f_linear_combination: term %d has %d limbs, fewer than %d", k,
                  term_limbs[k], l);
    T.in[k] = terms[k];
    T.limbs[k] = term_limbs[k];
    for (int i = 0; i < l; ++i) T.w[k][i] = weights[(size_t)k * l + i] % ctx->primes[i];
  }
  if (!num_cts) return B2F_OK;
  linear_combination_kernel<<<dim3(kN / TPB, l, num_cts * polys), TPB, 0,
                              (cudaStream_t)stream>>>(T, out, ctx->d_mod, l);
  B2F_LAUNCHED("linear_combination_kernel");
  return B2F_OK;
}

int b2f_scalar_op(b2f_context *ctx, const uint64_t *a, uint64_t *out,
                  int num_polys, int l, const uint64_t *mul_residues,
                  const uint64_t *add_residues, int add_poly, void *stream) {
  B2F_CHECK_ARG(ctx && a && out, "b2f_scalar_op: null argument");
  B2F_CHECK_ARG(l >= 1 && l <= ctx->L && l <= 64, "b2f_scalar_op: bad limbs %d", l);
  B2F_CHECK_ARG(add_poly >= -2 && add_poly < num_polys,
                "b2f_scalar_op: add_poly %d outside [-2, %d)", add_poly, num_polys);
  if (num_polys <= 0) return B2F_OK;
  ScalarArgs S{};
  S.has_mul = mul_residues != nullptr;
  S.has_add = add_residues != nullptr;
  S.add_poly = add_poly;
  for (int i = 0; i < l; ++i) {
    const uint64_t q = ctx->primes[i];
    if (S.has_mul) {
      uint64_t w = mul_residues[i] % q;
      S.mul[i] = make_ulonglong2(
          w, (uint64_t)(((unsigned __int128)w << 64) / q));
    }
    if (S.has_add) S.add[i] = add_residues[i] % q;
  }
  scalar_kernel<<<dim3(kN / TPB, l, num_polys), TPB, 0, (cudaStream_t)stream>>>(
      a, out, ctx->d_primes, l, S);
  B2F_LAUNCHED("scalar_kernel");
  return B2F_OK;
}

int b2f_mac(b2f_context *ctx, const uint64_t *babies, int baby_count,
            const uint64_t *pts, int giant_count, int l, uint64_t *out,
            int num_cts, void *stream) {
  B2F_RANGE("b2f_mac");
  B2F_CHECK_ARG(ctx && babies && pts && out, "b2f_mac: null argument");
  B2F_CHECK_ARG(l >= 1 && l <= ctx->L, "b2f_mac: bad limbs %d", l);
  B2F_CHECK_ARG(baby_count >= 1 && giant_count >= 1 && num_cts >= 0,
                "b2f_mac: bad counts");
  if (!num_cts) return B2F_OK;
  return launch_mac(ctx, babies, baby_count, pts, giant_count, l, out, num_cts,
                    (cudaStream_t)stream);
}

int b2f_mac_ext(b2f_context *ctx, const uint64_t *babies, int baby_count,
                const uint64_t *pts, int giant_count, int q_limbs, int p_limbs,
                uint64_t *out, int num_cts, void *stream) {
  B2F_RANGE("b2f_mac_ext");
  B2F_CHECK_ARG(ctx && babies && pts && out, "b2f_mac_ext: null argument");
  B2F_CHECK_ARG(q_limbs >= 1 && q_limbs <= ctx->L && p_limbs >= 0 && p_limbs <= ctx->K,
                "b2f_mac_ext: bad limbs q=%d p=%d", q_limbs, p_limbs);
  B2F_CHECK_ARG(baby_count >= 1 && giant_count >= 1 && num_cts >= 0,
                "b2f_mac_ext: bad counts");
  if (!num_cts) return B2F_OK;
  return launch_mac(ctx, babies, baby_count, pts, giant_count, q_limbs + p_limbs, out,
                    num_cts, (cudaStream_t)stream, 0, q_limbs);
}

int b2f_set_giant_chain(b2f_context *ctx, int mode) {
  B2F_CHECK_ARG(ctx, "b2f_set_giant_chain: null context");
  B2F_CHECK_ARG(mode == 0 || mode == 1, "b2f_set_giant_chain: mode %d is not 0 or 1", mode);
  ctx->giant_chain = mode;
  return B2F_OK;
}

int b2f_set_mac_path(b2f_context *ctx, int path) {
  B2F_CHECK_ARG(ctx, "b2f_set_mac_path: null context");
  B2F_CHECK_ARG(path == 0 || path == 1, "b2f_set_mac_path: path %d is not 0 or 1", path);
  ctx->mac_path = path;
  return B2F_OK;
}

int b2f_mac_uses_tensor_cores(const b2f_context *ctx, int baby_count, int giant_count,
                              int q_limbs, int p_limbs, int num_cts) {
  if (!ctx || baby_count < 1 || giant_count < 1 || q_limbs < 1 || q_limbs > ctx->L ||
      p_limbs < 0 || p_limbs > ctx->K)
    return 0;
  return mac_mma_eligible(ctx, baby_count, q_limbs + p_limbs, q_limbs, num_cts) &&
                 std::min(GMAX, giant_count) >= 4
             ? 1
             : 0;
}

int b2f_pairwise_mac(b2f_context *ctx, const uint64_t *cts, const uint64_t *pts,
                     int count, int groups, int q_limbs, int p_limbs,
                     int pt_limb_stride, uint64_t *out, void *stream) {
  B2F_RANGE("b2f_pairwise_mac");
  B2F_CHECK_ARG(ctx && cts && pts && out, "b2f_pairwise_mac: null argument");
  B2F_CHECK_ARG(count >= 1 && groups >= 1 && count % groups == 0,
                "b2f_pairwise_mac: %d pairs do not split into %d groups", count, groups);
  B2F_CHECK_ARG(q_limbs >= 1 && q_limbs <= ctx->L && p_limbs >= 0 && p_limbs <= ctx->K,
                "b2f_pairwise_mac: bad limbs q=%d p=%d", q_limbs, p_limbs);
  const int limbs = q_limbs + p_limbs;
  B2F_CHECK_ARG(pt_limb_stride >= limbs, "b2f_pairwise_mac: plaintext rows of %d limbs "
                "are shorter than %d", pt_limb_stride, limbs);
  pairwise_mac_kernel<<<dim3(kN / TPB, limbs, groups), TPB, 0, (cudaStream_t)stream>>>(
      cts, pts, out, count / groups, limbs, q_limbs, pt_limb_stride, ctx->L, ctx->d_mod);
  B2F_LAUNCHED("pairwise_mac_kernel");
  return B2F_OK;
}

size_t b2f_bsgs_mac_batch_workspace(const b2f_context *ctx, int num_cts,
                                    int giant_count, int l) {
  if (!ctx || l < 1 || l > ctx->L || num_cts < 0 || giant_count < 1) return 0;
  const size_t ct_words = 2 * (size_t)l * kN * std::max(num_cts, 1);
  const size_t horner = ct_words * 8 + rotate_workspace(ctx, num_cts, l);
  const size_t chain = giant_chain_workspace(ctx, std::max(num_cts, 1), l);
  return giant_count * ct_words * 8 + std::max(horner, chain) + 512;
}

size_t b2f_bsgs_mac_workspace(const b2f_context *ctx, int l) {
  if (!ctx || l < 1 || l > ctx->L) return 0;
  return 0;  // depends on giant_count: b2f_bsgs_mac_batch_workspace
}

int b2f_bsgs_mac_batch(b2f_context *ctx, const uint64_t *babies, int num_cts,
                       int baby_count, const uint64_t *pts, int giant_count,
                       int l, uint64_t giant_galois, const uint64_t *giant_key,
                       uint64_t *out, void *ws, size_t ws_bytes, void *stream) {
  B2F_RANGE("b2f_bsgs_mac_batch");
  B2F_CHECK_ARG(ctx && babies && pts && out, "b2f_bsgs_mac: null argument");
  B2F_CHECK_ARG(l >= 1 && l <= ctx->L, "b2f_bsgs_mac: bad limbs %d", l);
  B2F_CHECK_ARG(baby_count >= 1 && giant_count >= 1 && num_cts >= 0,
                "b2f_bsgs_mac: bad counts");
  B2F_CHECK_ARG(giant_count == 1 || giant_key,
                "b2f_bsgs_mac: giant_count > 1 needs the giant rotation key");
  if (!num_cts) return B2F_OK;
  cudaStream_t s = (cudaStream_t)stream;
  const size_t ct_words = 2 * (size_t)l * kN;
  const size_t batch_words = ct_words * num_cts;
  const size_t rot_ws = rotate_workspace(ctx, num_cts, l);
  const size_t need = b2f_bsgs_mac_batch_workspace(ctx, num_cts, giant_count, l);
  void *owned = nullptr;
  if (!ws) {
    B2F_CUDA(cudaMallocAsync(&owned, need, s));
    ws = owned;
  } else {
    B2F_CHECK_ARG(ws_bytes >= need, "b2f_bsgs_mac: workspace %zu < %zu", ws_bytes,
                  need);
  }
  // inner[g] (all ciphertexts of giant g contiguous), then a rotation buffer
  uint64_t *inner = static_cast<uint64_t *>(ws);
  uint64_t *rot = inner + giant_count * batch_words;
  void *rws = rot + batch_words;
  int rc = launch_mac(ctx, babies, baby_count, pts, giant_count, l, inner, num_cts,
                      s, 1);
  if (!rc && giant_count == 1) {
    cudaError_t e = cudaMemcpyAsync(out, inner, batch_words * 8,
                                    cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess) rc = cuda_status(e, "b2f_bsgs_mac copy");
  }
  if (!rc && giant_count > 1 && ctx->giant_chain == 0) {
    // Horner kept in Q_l u P: one ModDown per chain
    rc = giant_chain_ext(ctx, inner, 0, (long long)batch_words, (long long)ct_words, num_cts,
                         giant_count, l, giant_galois, giant_key, out, rot,
                         need - giant_count * batch_words * 8, s);
    if (owned) cudaFreeAsync(owned, s);
    return rc;
  }
  // Horner over the giants: acc = inner[G-1]; acc = rot(acc) + inner[g]
  const uint64_t *acc = inner + (size_t)(giant_count - 1) * batch_words;
  for (int g = giant_count - 2; !rc && g >= 0; --g) {
    rc = b2f_rotate(ctx, acc, rot, num_cts, l, giant_galois, giant_key, rws, rot_ws,
                    s);
    if (rc) break;
    uint64_t *dst = g == 0 ? out : inner + (size_t)(g + 1) * batch_words;
    rc = b2f_elementwise(ctx, 0, rot, inner + (size_t)g * batch_words, dst,
                         2 * num_cts, l, 2 * num_cts, s);
    acc = dst;
  }
  if (owned) cudaFreeAsync(owned, s);
  return rc;
}

int b2f_bsgs_mac(b2f_context *ctx, const uint64_t *babies, int baby_count,
                 const uint64_t *pts, int giant_count, int l,
                 uint64_t giant_galois, const uint64_t *giant_key,
                 uint64_t *out, void *ws, size_t ws_bytes, void *stream) {
  return b2f_bsgs_mac_batch(ctx, babies, 1, baby_count, pts, giant_count, l,
                            giant_galois, giant_key, out, ws, ws_bytes, stream);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Rescale that allocates nothing (b2f_rescale_noalloc).
//
// For callers that cannot allocate device memory: a process whose HBM is
// owned by another allocator (a framework that reserved the device up front
// and hands out only its own blocks), or a step with a fixed memory budget
// that may not call cudaMalloc/cudaMallocAsync.  The scratch lives in a
// file-scope __device__ array instead; every GPU that loads this library
// holds it (16 MiB) until the process exits.
// ---------------------------------------------------------------------------
namespace b2f {
namespace {

// scratch: the last limb of every poly in coefficient form (num_polys N
// words); the rescale's forward transform lifts it to the other primes in its
// input stage and writes the result straight to `out`
constexpr size_t kNoAllocBytes = 16u << 20;
constexpr size_t kNoAllocWords = kNoAllocBytes / sizeof(uint64_t);
__device__ __align__(256) uint64_t g_noalloc_scratch[kNoAllocWords];
// NTT job tables of the two transforms: row 0 the last limb, row 1 limbs
// 0..l-2 (l <= 64)
__device__ __align__(256) LimbJob g_noalloc_jobs[2][64];

struct NoAllocDevice {
  bool ready = false;
  uint64_t *scratch = nullptr;
  LimbJob *jobs = nullptr;
};
std::mutex g_noalloc_mu;
NoAllocDevice g_noalloc_dev[64];

__global__ void noalloc_jobs_kernel(LimbJob *jobs, int l) {
  const int i = threadIdx.x;
  if (i == 0)
    jobs[0] = LimbJob{(uint32_t)(l - 1), 0u, (uint16_t)(l - 1), (uint16_t)(l - 1), 0};
  if (i < l - 1) jobs[64 + i] = LimbJob{0u, (uint32_t)i, (uint16_t)i, (uint16_t)i, 0};
}

// The host-side names of the arrays above are stand-ins, not device
// addresses: look the addresses up once per device, with that device
// current, and hand those to the kernels.
int noalloc_setup(const b2f_context *ctx, NoAllocDevice **out) {
  std::lock_guard<std::mutex> g(g_noalloc_mu);
  NoAllocDevice &d = g_noalloc_dev[ctx->device & 63];
  if (!d.ready) {
    int prev = 0;
    B2F_CUDA(cudaGetDevice(&prev));
    if (prev != ctx->device) B2F_CUDA(cudaSetDevice(ctx->device));
    cudaError_t e1 = cudaGetSymbolAddress((void **)&d.scratch, g_noalloc_scratch);
    cudaError_t e2 = cudaGetSymbolAddress((void **)&d.jobs, g_noalloc_jobs);
    if (prev != ctx->device) cudaSetDevice(prev);
    if (e1 != cudaSuccess) return cuda_status(e1, "cudaGetSymbolAddress(scratch)");
    if (e2 != cudaSuccess) return cuda_status(e2, "cudaGetSymbolAddress(jobs)");
    d.ready = true;
  }
  *out = &d;
  return B2F_OK;
}

}  // namespace
}  // namespace b2f

extern "C" int b2f_rescale_noalloc(b2f_context *ctx, const uint64_t *in,
                                   uint64_t *out, int num_polys, int l,
                                   void *stream) {
  B2F_CHECK_ARG(ctx && in && out && num_polys >= 0,
                "b2f_rescale_noalloc: null argument");
  B2F_CHECK_ARG(l >= 2 && l <= ctx->L && l <= 64,
                "b2f_rescale_noalloc: needs 2..%d limbs, got %d", ctx->L, l);
  B2F_CHECK_ARG(in != out, "b2f_rescale_noalloc: in-place rescale is not supported");
  const size_t need = (size_t)num_polys * kN;
  B2F_CHECK_ARG(need <= kNoAllocWords,
                "b2f_rescale_noalloc: %d polys need %zu bytes of scratch, more than "
                "its fixed %zu (num_polys must be <= %zu)",
                num_polys, need * 8, kNoAllocBytes, kNoAllocWords / kN);
  int cur = -1;
  B2F_CUDA(cudaGetDevice(&cur));
  B2F_CHECK_ARG(cur == ctx->device,
                "b2f_rescale_noalloc: the context's device %d must be current (is %d)",
                ctx->device, cur);
  if (!num_polys) return B2F_OK;
  NoAllocDevice *d = nullptr;
  int rc = noalloc_setup(ctx, &d);
  if (rc) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  uint64_t *last = d->scratch;
  noalloc_jobs_kernel<<<1, 64, 0, s>>>(d->jobs, l);
  B2F_LAUNCHED("noalloc_jobs_kernel");
  // the last limb back to coefficients, then lift, forward NTT and combine in
  // one launch, as b2f_rescale does
  rc = launch_ntt(ctx, in, (long long)l * kN, last, kN, d->jobs, 1, num_polys, 1,
                  nullptr, s);
  if (rc) return rc;
  return ntt_rescale_jobs(ctx, last, in, out, num_polys, l, d->jobs + 64, s);
}
