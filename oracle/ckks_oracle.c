/*
 * ckks_oracle.c -- CPU restatement of the CKKS evaluation ops (TEST ONLY).
 * The header (ckks_oracle.h) states the scope, the literature followed and the
 * parity status.  Every routine here is written for clarity first: exact
 * 128-bit modular arithmetic, one limb at a time, OpenMP only across
 * independent limbs.
 */
#include "ckks_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

typedef unsigned __int128 u128;

/* ------------------------------------------------------------------ */
/* modular arithmetic                                                  */
/* ------------------------------------------------------------------ */
static inline uint64_t mulmod(uint64_t a, uint64_t b, uint64_t q) {
  return (uint64_t)(((u128)a * b) % q);
}
static inline uint64_t addmod(uint64_t a, uint64_t b, uint64_t q) {
  uint64_t s = a + b;
  return s >= q ? s - q : s;
}
static inline uint64_t submod(uint64_t a, uint64_t b, uint64_t q) {
  return a >= b ? a - b : a + q - b;
}
static uint64_t powmod(uint64_t a, uint64_t e, uint64_t q) {
  uint64_t r = 1 % q;
  a %= q;
  while (e) {
    if (e & 1) r = mulmod(r, a, q);
    a = mulmod(a, a, q);
    e >>= 1;
  }
  return r;
}
static uint64_t invmod(uint64_t a, uint64_t q) { return powmod(a, q - 2, q); }
/* Shoup companion floor(w * 2^64 / q) for a constant w < q */
static inline uint64_t shoup(uint64_t w, uint64_t q) {
  return (uint64_t)(((u128)w << 64) / q);
}
static inline uint64_t mulmod_shoup(uint64_t x, uint64_t w, uint64_t ws,
                                    uint64_t q) {
  uint64_t qh = (uint64_t)(((u128)x * ws) >> 64);
  uint64_t r = x * w - qh * q;
  return r >= q ? r - q : r;
}

/* ------------------------------------------------------------------ */
/* primes and roots                                                    */
/* ------------------------------------------------------------------ */
int orc_is_prime(uint64_t n) {
  if (n < 2) return 0;
  static const uint64_t small[] = {2, 3, 5, 7, 11, 13, 17, 19, 23, 29, 31, 37};
  for (int i = 0; i < 12; i++) {
    if (n == small[i]) return 1;
    if (n % small[i] == 0) return 0;
  }
  uint64_t d = n - 1;
  int s = 0;
  while (!(d & 1)) {
    d >>= 1;
    s++;
  }
  /* these bases make Miller-Rabin deterministic for all n < 2^64 */
  static const uint64_t bases[] = {2, 325, 9375, 28178, 450775, 9780504,
                                   1795265022};
  for (int i = 0; i < 7; i++) {
    uint64_t a = bases[i] % n;
    if (a == 0) continue;
    uint64_t x = powmod(a, d, n);
    if (x == 1 || x == n - 1) continue;
    int comp = 1;
    for (int r = 1; r < s; r++) {
      x = mulmod(x, x, n);
      if (x == n - 1) {
        comp = 0;
        break;
      }
    }
    if (comp) return 0;
  }
  return 1;
}

static int in_list(uint64_t v, const uint64_t *l, int n) {
  for (int i = 0; i < n; i++)
    if (l[i] == v) return 1;
  return 0;
}

/* mode 0: largest primes below 2^bits with q = 1 mod 2N, descending.
 * mode 1: primes alternately just below and just above 2^bits (q = 1 mod 2N),
 *         below first, so the product of consecutive pairs stays near 2^2bits.
 * Primes in `exclude` (and ones already chosen) are skipped. */
int orc_gen_primes(int log_n, int bits, int count, int mode,
                   const uint64_t *exclude, int n_exclude, uint64_t *out) {
  const uint64_t m = 2ull << log_n;
  const uint64_t base = 1ull << bits;
  uint64_t below = base + 1 - m, above = base + 1 + m;
  int found = 0, side = 0;
  while (found < count) {
    uint64_t c;
    if (mode == 0 || side == 0) {
      c = below;
      if (below <= m) return -1;
      below -= m;
    } else {
      c = above;
      above += m;
    }
    int ok = orc_is_prime(c) && !in_list(c, exclude, n_exclude) &&
             !in_list(c, out, found);
    if (ok) {
      out[found++] = c;
      if (mode == 1) side ^= 1;
    }
  }
  return 0;
}

/* The smallest primitive 2N-th root of unity modulo q. */
uint64_t orc_find_psi(uint64_t q, int log_n) {
  const uint64_t n = 1ull << log_n, m = 2 * n;
  uint64_t psi0 = 0;
  for (uint64_t g = 2; g < q; g++) {
    uint64_t c = powmod(g, (q - 1) / m, q);
    if (powmod(c, n, q) == q - 1) {
      psi0 = c;
      break;
    }
  }
  /* all primitive 2N-th roots are psi0^(2k+1) */
  uint64_t best = psi0, sq = mulmod(psi0, psi0, q), cur = psi0;
  for (uint64_t k = 1; k < n; k++) {
    cur = mulmod(cur, sq, q);
    if (cur < best) best = cur;
  }
  return best;
}

static uint32_t bitrev(uint32_t x, int bits) {
  uint32_t r = 0;
  for (int i = 0; i < bits; i++) {
    r = (r << 1) | (x & 1);
    x >>= 1;
  }
  return r;
}

/* ------------------------------------------------------------------ */
/* ChaCha20 block function (Bernstein 2008), 64-bit counter + 64-bit nonce */
/* ------------------------------------------------------------------ */
#define ROTL32(v, c) (((v) << (c)) | ((v) >> (32 - (c))))
#define QR(a, b, c, d)                                                       \
  a += b; d ^= a; d = ROTL32(d, 16);                                         \
  c += d; b ^= c; b = ROTL32(b, 12);                                         \
  a += b; d ^= a; d = ROTL32(d, 8);                                          \
  c += d; b ^= c; b = ROTL32(b, 7);

void orc_chacha_block(uint64_t seed, uint64_t stream, uint64_t counter,
                      uint64_t out[8]) {
  uint32_t s[16] = {0x61707865u, 0x3320646eu, 0x79622d32u, 0x6b206574u,
                    (uint32_t)seed, (uint32_t)(seed >> 32), 0, 0, 0, 0, 0, 0,
                    (uint32_t)counter, (uint32_t)(counter >> 32),
                    (uint32_t)stream, (uint32_t)(stream >> 32)};
  uint32_t x[16];
  memcpy(x, s, sizeof x);
  for (int i = 0; i < 10; i++) {
    QR(x[0], x[4], x[8], x[12]);
    QR(x[1], x[5], x[9], x[13]);
    QR(x[2], x[6], x[10], x[14]);
    QR(x[3], x[7], x[11], x[15]);
    QR(x[0], x[5], x[10], x[15]);
    QR(x[1], x[6], x[11], x[12]);
    QR(x[2], x[7], x[8], x[13]);
    QR(x[3], x[4], x[9], x[14]);
  }
  for (int i = 0; i < 8; i++)
    out[i] = (uint64_t)(x[2 * i] + s[2 * i]) |
             ((uint64_t)(x[2 * i + 1] + s[2 * i + 1]) << 32);
}

static inline uint64_t stream_id(uint64_t tag, uint64_t a, uint64_t b,
                                 uint64_t c) {
  return (tag << 56) | ((a & 0xFFFFFFull) << 32) | ((b & 0xFFFFull) << 16) |
         (c & 0xFFFFull);
}
enum { TAG_SECRET = 1, TAG_KEY_A = 2, TAG_KEY_E = 3, TAG_ENC_A = 4,
       TAG_ENC_E = 5 };

/* uniform residue mod q for coefficient k of a stream */
static void sample_uniform(uint64_t seed, uint64_t stream, uint64_t q,
                           uint64_t n, uint64_t *out) {
  uint64_t blk[8];
  for (uint64_t k = 0; k < n; k += 4) {
    orc_chacha_block(seed, stream, k / 4, blk);
    for (int p = 0; p < 4; p++) {
      u128 v = ((u128)blk[2 * p] << 64) | blk[2 * p + 1];
      out[k + p] = (uint64_t)(v % q);
    }
  }
}
/* centred binomial, eta = 21: variance 10.5 */
static void sample_cbd(uint64_t seed, uint64_t stream, uint64_t n,
                       int64_t *out) {
  uint64_t blk[8];
  for (uint64_t k = 0; k < n; k += 8) {
    orc_chacha_block(seed, stream, k / 8, blk);
    for (int p = 0; p < 8; p++) {
      uint64_t w = blk[p];
      out[k + p] = (int64_t)__builtin_popcountll(w & 0x1FFFFFull) -
                   (int64_t)__builtin_popcountll((w >> 21) & 0x1FFFFFull);
    }
  }
}

/* ------------------------------------------------------------------ */
/* context                                                             */
/* ------------------------------------------------------------------ */
struct orc_ctx {
  int log_n, L, K, dnum, alpha, digits;
  uint64_t n;
  uint64_t *primes;     /* L + K */
  uint64_t **psi_rev;   /* per prime, N entries */
  uint64_t **psi_rev_s; /* Shoup companions */
  uint64_t **ipsi_rev;
  uint64_t **ipsi_rev_s;
  uint64_t *n_inv;
};

orc_ctx *orc_ctx_create(int log_n, const uint64_t *q, int L, const uint64_t *p,
                        int K, int dnum) {
  orc_ctx *c = (orc_ctx *)calloc(1, sizeof *c);
  c->log_n = log_n;
  c->n = 1ull << log_n;
  c->L = L;
  c->K = K;
  c->dnum = dnum;
  c->alpha = (L + dnum - 1) / dnum;
  c->digits = (L + c->alpha - 1) / c->alpha;
  int np = L + K;
  c->primes = (uint64_t *)malloc(sizeof(uint64_t) * np);
  memcpy(c->primes, q, sizeof(uint64_t) * L);
  if (K) memcpy(c->primes + L, p, sizeof(uint64_t) * K);
  c->psi_rev = (uint64_t **)calloc(np, sizeof(uint64_t *));
  c->psi_rev_s = (uint64_t **)calloc(np, sizeof(uint64_t *));
  c->ipsi_rev = (uint64_t **)calloc(np, sizeof(uint64_t *));
  c->ipsi_rev_s = (uint64_t **)calloc(np, sizeof(uint64_t *));
  c->n_inv = (uint64_t *)malloc(sizeof(uint64_t) * np);
#pragma omp parallel for schedule(dynamic)
  for (int i = 0; i < np; i++) {
    uint64_t qi = c->primes[i], n = c->n;
    uint64_t psi = orc_find_psi(qi, log_n), ipsi = invmod(psi, qi);
    uint64_t *pw = (uint64_t *)malloc(8 * n), *ipw = (uint64_t *)malloc(8 * n);
    uint64_t a = 1, b = 1;
    for (uint64_t k = 0; k < n; k++) {
      pw[k] = a;
      ipw[k] = b;
      a = mulmod(a, psi, qi);
      b = mulmod(b, ipsi, qi);
    }
    c->psi_rev[i] = (uint64_t *)malloc(8 * n);
    c->psi_rev_s[i] = (uint64_t *)malloc(8 * n);
    c->ipsi_rev[i] = (uint64_t *)malloc(8 * n);
    c->ipsi_rev_s[i] = (uint64_t *)malloc(8 * n);
    for (uint64_t k = 0; k < n; k++) {
      uint32_t r = bitrev((uint32_t)k, log_n);
      c->psi_rev[i][k] = pw[r];
      c->psi_rev_s[i][k] = shoup(pw[r], qi);
      c->ipsi_rev[i][k] = ipw[r];
      c->ipsi_rev_s[i][k] = shoup(ipw[r], qi);
    }
    free(pw);
    free(ipw);
    c->n_inv[i] = invmod(n % qi, qi);
  }
  return c;
}

void orc_ctx_free(orc_ctx *c) {
  if (!c) return;
  for (int i = 0; i < c->L + c->K; i++) {
    free(c->psi_rev[i]);
    free(c->psi_rev_s[i]);
    free(c->ipsi_rev[i]);
    free(c->ipsi_rev_s[i]);
  }
  free(c->psi_rev);
  free(c->psi_rev_s);
  free(c->ipsi_rev);
  free(c->ipsi_rev_s);
  free(c->n_inv);
  free(c->primes);
  free(c);
}
int orc_alpha(const orc_ctx *c) { return c->alpha; }
int orc_num_digits(const orc_ctx *c) { return c->digits; }

/* ------------------------------------------------------------------ */
/* NTT                                                                  */
/* ------------------------------------------------------------------ */
/* Forward: natural-order coefficients -> evaluations, position k holding
 * a(psi^(2*bitrev(k)+1)).  Cooley-Tukey, t halves each stage. */
void orc_ntt_forward(const orc_ctx *c, uint64_t *a, int pi) {
  const uint64_t q = c->primes[pi], n = c->n;
  const uint64_t *w = c->psi_rev[pi], *ws = c->psi_rev_s[pi];
  uint64_t t = n;
  for (uint64_t m = 1; m < n; m <<= 1) {
    t >>= 1;
    for (uint64_t i = 0; i < m; i++) {
      uint64_t j1 = 2 * i * t, W = w[m + i], WS = ws[m + i];
      for (uint64_t j = j1; j < j1 + t; j++) {
        uint64_t u = a[j], v = mulmod_shoup(a[j + t], W, WS, q);
        a[j] = addmod(u, v, q);
        a[j + t] = submod(u, v, q);
      }
    }
  }
}

/* Inverse: Gentleman-Sande with the inverse psi table, then times N^-1. */
void orc_ntt_inverse(const orc_ctx *c, uint64_t *a, int pi) {
  const uint64_t q = c->primes[pi], n = c->n;
  const uint64_t *w = c->ipsi_rev[pi], *ws = c->ipsi_rev_s[pi];
  uint64_t t = 1;
  for (uint64_t m = n; m > 1; m >>= 1) {
    uint64_t h = m >> 1, j1 = 0;
    for (uint64_t i = 0; i < h; i++) {
      uint64_t W = w[h + i], WS = ws[h + i];
      for (uint64_t j = j1; j < j1 + t; j++) {
        uint64_t u = a[j], v = a[j + t];
        a[j] = addmod(u, v, q);
        a[j + t] = mulmod_shoup(submod(u, v, q), W, WS, q);
      }
      j1 += 2 * t;
    }
    t <<= 1;
  }
  uint64_t ni = c->n_inv[pi], nis = shoup(ni, q);
  for (uint64_t j = 0; j < n; j++) a[j] = mulmod_shoup(a[j], ni, nis, q);
}

static inline int limb_prime(const orc_ctx *c, int q_limbs, int limb) {
  return limb < q_limbs ? limb : c->L + (limb - q_limbs);
}

void orc_poly_ntt(const orc_ctx *c, uint64_t *data, int num_polys, int q_limbs,
                  int p_limbs, int inverse) {
  int limbs = q_limbs + p_limbs;
#pragma omp parallel for schedule(dynamic)
  for (int x = 0; x < num_polys * limbs; x++) {
    int limb = x % limbs;
    uint64_t *a = data + (uint64_t)x * c->n;
    int pi = limb_prime(c, q_limbs, limb);
    if (inverse)
      orc_ntt_inverse(c, a, pi);
    else
      orc_ntt_forward(c, a, pi);
  }
}

/* ------------------------------------------------------------------ */
/* automorphisms                                                        */
/* ------------------------------------------------------------------ */
uint64_t orc_galois_element(int log_n, int64_t r) {
  const uint64_t m = 2ull << log_n, slots = 1ull << (log_n - 1);
  if ((uint64_t)r == m - 1) return m - 1; /* conjugation, index M-1 */
  int64_t rr = r % (int64_t)slots;
  if (rr < 0) rr += (int64_t)slots;
  uint64_t g = 1;
  for (int64_t i = 0; i < rr; i++) g = (g * 5) % m;
  return g;
}

/* evaluation k sits at exponent e_k = 2*bitrev(k)+1; sigma_g(a)(psi^e) =
 * a(psi^(e*g)), so out[k] = in[k'] with e_k' = e_k * g mod 2N. */
void orc_automorphism_perm(int log_n, uint64_t g, int32_t *perm) {
  const uint64_t n = 1ull << log_n, m = 2 * n;
  for (uint64_t k = 0; k < n; k++) {
    uint64_t e = 2 * (uint64_t)bitrev((uint32_t)k, log_n) + 1;
    uint64_t e2 = (e * g) % m;
    perm[k] = (int32_t)bitrev((uint32_t)((e2 - 1) / 2), log_n);
  }
}

static void apply_perm(const uint64_t *in, uint64_t *out, const int32_t *perm,
                       uint64_t n) {
  for (uint64_t k = 0; k < n; k++) out[k] = in[perm[k]];
}

/* ------------------------------------------------------------------ */
/* base conversion and key switching                                    */
/* ------------------------------------------------------------------ */
/* prime index of target limb t of an extended poly at level l */
static inline int ext_prime(const orc_ctx *c, int l, int t) {
  return t < l ? t : c->L + (t - l);
}

/* x_coeff: l limbs of the coefficient-domain c1.  For digit j (primes
 * [j*alpha, min((j+1)*alpha, l))) writes the fast base conversion
 *   y_t = sum_i [x_i * Qhat_i^-1]_{q_i} * (Qhat_i mod q_t)  mod q_t
 * into every target limb t of Q_l u P outside the digit, and copies the
 * digit's own limbs.  out_coeff has l+K limbs (coefficient domain). */
void orc_modup_digit(const orc_ctx *c, const uint64_t *x, int l, int j,
                     uint64_t *out) {
  const uint64_t n = c->n;
  int lo = j * c->alpha, hi = lo + c->alpha;
  if (hi > l) hi = l;
  int w = hi - lo;
  uint64_t *qhat_inv = (uint64_t *)malloc(8 * w);
  for (int i = lo; i < hi; i++) {
    uint64_t qi = c->primes[i], prod = 1;
    for (int i2 = lo; i2 < hi; i2++)
      if (i2 != i) prod = mulmod(prod, c->primes[i2] % qi, qi);
    qhat_inv[i - lo] = invmod(prod, qi);
  }
  uint64_t *xt = (uint64_t *)malloc(8 * n * w);
  for (int i = lo; i < hi; i++)
    for (uint64_t k = 0; k < n; k++)
      xt[(i - lo) * n + k] =
          mulmod(x[(uint64_t)i * n + k], qhat_inv[i - lo], c->primes[i]);
#pragma omp parallel for schedule(dynamic)
  for (int t = 0; t < l + c->K; t++) {
    uint64_t *o = out + (uint64_t)t * n;
    if (t >= lo && t < hi) {
      memcpy(o, x + (uint64_t)t * n, 8 * n);
      continue;
    }
    uint64_t pt = c->primes[ext_prime(c, l, t)];
    uint64_t qhat_mod[64];
    for (int i = lo; i < hi; i++) {
      uint64_t prod = 1;
      for (int i2 = lo; i2 < hi; i2++)
        if (i2 != i) prod = mulmod(prod, c->primes[i2] % pt, pt);
      qhat_mod[i - lo] = prod;
    }
    for (uint64_t k = 0; k < n; k++) {
      u128 s = 0;
      for (int i = 0; i < w; i++) s += (u128)xt[i * n + k] * qhat_mod[i];
      o[k] = (uint64_t)(s % pt);
    }
  }
  free(xt);
  free(qhat_inv);
}

/* Inner product of the extended digits with the key, accumulated over the
 * digits: acc_b[t] = sum_j ext_j[t] * key[j][b][prime(t)]. */
static void key_inner_product(const orc_ctx *c, const uint64_t *ext, int l,
                              int beta, const uint64_t *key, uint64_t *acc0,
                              uint64_t *acc1) {
  const uint64_t n = c->n;
  const int lk = l + c->K, np = c->L + c->K;
#pragma omp parallel for schedule(dynamic)
  for (int t = 0; t < lk; t++) {
    int pi = ext_prime(c, l, t);
    uint64_t q = c->primes[pi];
    for (uint64_t k = 0; k < n; k++) {
      uint64_t s0 = 0, s1 = 0;
      for (int j = 0; j < beta; j++) {
        uint64_t e = ext[((uint64_t)j * lk + t) * n + k];
        const uint64_t *kb = key + ((uint64_t)j * 2 * np) * n;
        s0 = addmod(s0, mulmod(e, kb[(uint64_t)pi * n + k], q), q);
        s1 = addmod(s1, mulmod(e, kb[((uint64_t)np + pi) * n + k], q), q);
      }
      acc0[(uint64_t)t * n + k] = s0;
      acc1[(uint64_t)t * n + k] = s1;
    }
  }
}

/* ModDown of one extended poly acc (l+K limbs, NTT) -> d (l limbs, NTT):
 * d_i = (acc_i - NTT(sum_k [z_k * Phat_k^-1]_{p_k} * Phat_k mod q_i)) * P^-1 */
static void moddown(const orc_ctx *c, const uint64_t *acc, int l,
                    uint64_t *d) {
  const uint64_t n = c->n;
  const int K = c->K;
  uint64_t *z = (uint64_t *)malloc(8 * n * (K ? K : 1));
  memcpy(z, acc + (uint64_t)l * n, 8 * n * K);
  for (int k = 0; k < K; k++) {
    int pi = c->L + k;
    uint64_t pk = c->primes[pi], prod = 1;
    orc_ntt_inverse(c, z + (uint64_t)k * n, pi);
    for (int k2 = 0; k2 < K; k2++)
      if (k2 != k) prod = mulmod(prod, c->primes[c->L + k2] % pk, pk);
    uint64_t inv = invmod(prod, pk);
    for (uint64_t x = 0; x < n; x++)
      z[k * n + x] = mulmod(z[k * n + x], inv, pk);
  }
#pragma omp parallel for schedule(dynamic)
  for (int i = 0; i < l; i++) {
    uint64_t qi = c->primes[i];
    uint64_t phat[64], pinv = 1;
    for (int k = 0; k < K; k++) {
      uint64_t prod = 1;
      for (int k2 = 0; k2 < K; k2++)
        if (k2 != k) prod = mulmod(prod, c->primes[c->L + k2] % qi, qi);
      phat[k] = prod;
      pinv = mulmod(pinv, c->primes[c->L + k] % qi, qi);
    }
    pinv = invmod(pinv, qi);
    uint64_t *conv = (uint64_t *)malloc(8 * n);
    for (uint64_t x = 0; x < n; x++) {
      u128 s = 0;
      for (int k = 0; k < K; k++) s += (u128)z[k * n + x] * phat[k];
      conv[x] = (uint64_t)(s % qi);
    }
    orc_ntt_forward(c, conv, i);
    for (uint64_t x = 0; x < n; x++)
      d[(uint64_t)i * n + x] =
          mulmod(submod(acc[(uint64_t)i * n + x], conv[x], qi), pinv, qi);
    free(conv);
  }
  free(z);
}

/* ModUp of c1 (NTT form, l limbs) into beta extended digits (NTT form,
 * l+K limbs each). */
static uint64_t *modup(const orc_ctx *c, const uint64_t *c1, int l,
                       int *beta_out) {
  const uint64_t n = c->n;
  const int beta = (l + c->alpha - 1) / c->alpha, lk = l + c->K;
  uint64_t *x = (uint64_t *)malloc(8 * n * l);
  memcpy(x, c1, 8 * n * l);
  orc_poly_ntt(c, x, 1, l, 0, 1);
  uint64_t *ext = (uint64_t *)malloc(8 * n * (uint64_t)lk * beta);
  for (int j = 0; j < beta; j++) {
    uint64_t *e = ext + (uint64_t)j * lk * n;
    orc_modup_digit(c, x, l, j, e);
    int lo = j * c->alpha, hi = lo + c->alpha;
    if (hi > l) hi = l;
#pragma omp parallel for schedule(dynamic)
    for (int t = 0; t < lk; t++) {
      if (t >= lo && t < hi)
        memcpy(e + (uint64_t)t * n, c1 + (uint64_t)t * n, 8 * n);
      else
        orc_ntt_forward(c, e + (uint64_t)t * n, ext_prime(c, l, t));
    }
  }
  free(x);
  *beta_out = beta;
  return ext;
}

static void keyswitch_ext(const orc_ctx *c, const uint64_t *ext, int l,
                          int beta, const uint64_t *key, uint64_t *d0,
                          uint64_t *d1) {
  const uint64_t n = c->n;
  const int lk = l + c->K;
  uint64_t *acc0 = (uint64_t *)malloc(8 * n * lk);
  uint64_t *acc1 = (uint64_t *)malloc(8 * n * lk);
  key_inner_product(c, ext, l, beta, key, acc0, acc1);
  moddown(c, acc0, l, d0);
  moddown(c, acc1, l, d1);
  free(acc0);
  free(acc1);
}

void orc_keyswitch(const orc_ctx *c, const uint64_t *c1, int l,
                   const uint64_t *key, uint64_t *d0, uint64_t *d1) {
  int beta;
  uint64_t *ext = modup(c, c1, l, &beta);
  keyswitch_ext(c, ext, l, beta, key, d0, d1);
  free(ext);
}

/* HRotate with the automorphism applied after the key switch:
 * (c0, c1) -> (pi_g(c0 + d0), pi_g(d1)), (d0, d1) = KS(c1) under a key that
 * switches s to sigma_g^-1(s). */
void orc_rotate(const orc_ctx *c, const uint64_t *ct, int l, uint64_t g,
                const uint64_t *key, uint64_t *out) {
  orc_rotate_hoisted(c, ct, l, 1, &g, &key, out);
}

void orc_rotate_hoisted(const orc_ctx *c, const uint64_t *ct, int l,
                        int count, const uint64_t *galois,
                        const uint64_t *const *keys, uint64_t *out) {
  const uint64_t n = c->n;
  int beta;
  uint64_t *ext = modup(c, ct + (uint64_t)l * n, l, &beta);
  uint64_t *d0 = (uint64_t *)malloc(8 * n * l), *d1 = (uint64_t *)malloc(8 * n * l);
  int32_t *perm = (int32_t *)malloc(4 * n);
  for (int r = 0; r < count; r++) {
    uint64_t *o = out + (uint64_t)r * 2 * l * n;
    keyswitch_ext(c, ext, l, beta, keys[r], d0, d1);
    for (int i = 0; i < l; i++) {
      uint64_t qi = c->primes[i];
      for (uint64_t x = 0; x < n; x++)
        d0[i * n + x] = addmod(d0[i * n + x], ct[i * n + x], qi);
    }
    orc_automorphism_perm(c->log_n, galois[r], perm);
    for (int i = 0; i < l; i++) {
      apply_perm(d0 + (uint64_t)i * n, o + (uint64_t)i * n, perm, n);
      apply_perm(d1 + (uint64_t)i * n, o + ((uint64_t)l + i) * n, perm, n);
    }
  }
  free(perm);
  free(d0);
  free(d1);
  free(ext);
}

/* Hoisted rotations left in the extended basis Q_l u P (double hoisting,
 * Bossuat et al. 2021): out[r] = (pi_g(P c0 + acc0), pi_g(acc1)) over l+K
 * limbs, i.e. P times the rotated ciphertext before ModDown.  A rotation with
 * galois element 1 is (P c0, P c1) with no key switch. */
void orc_rotate_hoisted_ext(const orc_ctx *c, const uint64_t *ct, int l,
                            int count, const uint64_t *galois,
                            const uint64_t *const *keys, uint64_t *out) {
  const uint64_t n = c->n;
  const int lk = l + c->K;
  int beta;
  uint64_t *ext = modup(c, ct + (uint64_t)l * n, l, &beta);
  uint64_t *acc0 = (uint64_t *)malloc(8 * n * lk), *acc1 = (uint64_t *)malloc(8 * n * lk);
  int32_t *perm = (int32_t *)malloc(4 * n);
  for (int r = 0; r < count; r++) {
    uint64_t *o0 = out + (uint64_t)r * 2 * lk * n, *o1 = o0 + (uint64_t)lk * n;
    if (galois[r] == 1) {
      for (int t = 0; t < lk; t++) {
        uint64_t q = c->primes[ext_prime(c, l, t)];
        uint64_t pm = 1;
        for (int k = 0; k < c->K; k++) pm = mulmod(pm, c->primes[c->L + k] % q, q);
        for (uint64_t x = 0; x < n; x++) {
          o0[t * n + x] = t < l ? mulmod(pm, ct[t * n + x], q) : 0;
          o1[t * n + x] = t < l ? mulmod(pm, ct[((uint64_t)l + t) * n + x], q) : 0;
        }
      }
      continue;
    }
    key_inner_product(c, ext, l, beta, keys[r], acc0, acc1);
    for (int t = 0; t < l; t++) {
      uint64_t q = c->primes[t];
      uint64_t pm = 1;
      for (int k = 0; k < c->K; k++) pm = mulmod(pm, c->primes[c->L + k] % q, q);
      for (uint64_t x = 0; x < n; x++)
        acc0[t * n + x] = addmod(acc0[t * n + x], mulmod(pm, ct[t * n + x], q), q);
    }
    orc_automorphism_perm(c->log_n, galois[r], perm);
    for (int t = 0; t < lk; t++) {
      apply_perm(acc0 + (uint64_t)t * n, o0 + (uint64_t)t * n, perm, n);
      apply_perm(acc1 + (uint64_t)t * n, o1 + (uint64_t)t * n, perm, n);
    }
  }
  free(perm);
  free(acc0);
  free(acc1);
  free(ext);
}

/* Relinearisation fused with the rescale that follows it
 * (homo_mul_relin_rescale_postop, llama3fhe/operators/nonlinear/polynomial.py:
 * 108-159): for ct3 = (d0, d1, d2) at l limbs, acc = IP(ModUp(d2), relin key)
 * over Q_l u P and Y_b = P d_b + acc_b (the P limbs of P d_b are zero); with
 * R = {q_{l-1}} u P and M = P q_{l-1},
 *   out_b = (Y_b - C(Y_b[R])) * M^-1   over Q_{l-1},
 * C(y) = sum_r y_r (M/r) - v M mod q_i,  y_r = [Y_r (M/r)^-1]_r,
 * v = floor(sum_r y_r / r + 1/2) in binary64 (products y_r * (1/r), then
 * sums in r order, no fused multiply-add): C(y) is the centred residue of Y
 * mod M (Halevi-Polyakov-Shoup 2019), so out is Y / M rounded to the
 * nearest integer.  One exact rounding division by P q_{l-1} in place of
 * ModDown by P followed by the rescale by q_{l-1}. */
void orc_relin_rescale(const orc_ctx *c, const uint64_t *ct3, int l,
                       const uint64_t *key, uint64_t *out) {
  const uint64_t n = c->n;
  const int K = c->K, lk = l + K, R = K + 1;
  int beta;
  uint64_t *ext = modup(c, ct3 + 2 * (uint64_t)l * n, l, &beta);
  uint64_t *acc[2];
  acc[0] = (uint64_t *)malloc(8 * n * lk);
  acc[1] = (uint64_t *)malloc(8 * n * lk);
  key_inner_product(c, ext, l, beta, key, acc[0], acc[1]);
  int rp[65];  /* prime index of removed limb r */
  rp[0] = l - 1;
  for (int k = 0; k < K; k++) rp[1 + k] = c->L + k;
  uint64_t *z = (uint64_t *)malloc(8 * n * R);
  double rinv[65];
  for (int r = 0; r < R; r++) rinv[r] = 1.0 / (double)c->primes[rp[r]];
  for (int b = 0; b < 2; b++) {
    const uint64_t *d = ct3 + (uint64_t)b * l * n, *Y = acc[b];
    /* removed limbs in NTT form, then coefficients times (M/r)^-1 mod r */
    for (int r = 0; r < R; r++) {
      const uint64_t pr = c->primes[rp[r]];
      uint64_t pm = 1, mr = 1; /* P mod pr, (M/r) mod pr */
      for (int k = 0; k < K; k++) pm = mulmod(pm, c->primes[c->L + k] % pr, pr);
      for (int r2 = 0; r2 < R; r2++)
        if (r2 != r) mr = mulmod(mr, c->primes[rp[r2]] % pr, pr);
      uint64_t *zr = z + (uint64_t)r * n;
      for (uint64_t x = 0; x < n; x++)
        zr[x] = r == 0 ? addmod(mulmod(pm, d[(uint64_t)(l - 1) * n + x], pr),
                                Y[(uint64_t)(l - 1) * n + x], pr)
                       : Y[((uint64_t)l + r - 1) * n + x];
      orc_ntt_inverse(c, zr, rp[r]);
      const uint64_t inv = invmod(mr, pr);
      for (uint64_t x = 0; x < n; x++) zr[x] = mulmod(zr[x], inv, pr);
    }
#pragma omp parallel for schedule(dynamic)
    for (int i = 0; i < l - 1; i++) {
      const uint64_t qi = c->primes[i];
      uint64_t mhat[65], pm = 1, minv = 1;
      for (int k = 0; k < K; k++) pm = mulmod(pm, c->primes[c->L + k] % qi, qi);
      for (int r = 0; r < R; r++) {
        uint64_t m = 1;
        for (int r2 = 0; r2 < R; r2++)
          if (r2 != r) m = mulmod(m, c->primes[rp[r2]] % qi, qi);
        mhat[r] = m;
      }
      const uint64_t mq = mulmod(pm, c->primes[l - 1] % qi, qi); /* M mod q_i */
      minv = invmod(mq, qi);
      uint64_t *conv = (uint64_t *)malloc(8 * n);
      for (uint64_t x = 0; x < n; x++) {
        u128 sum = 0;
        volatile double f = 0.0;
        for (int r = 0; r < R; r++) {
          const uint64_t y = z[(uint64_t)r * n + x];
          sum += (u128)y * mhat[r];
          volatile double t = (double)y * rinv[r];
          f = f + t;
        }
        volatile double h = f + 0.5;
        const uint64_t v = (uint64_t)h;
        conv[x] = submod((uint64_t)(sum % qi), mulmod(v % qi, mq, qi), qi);
      }
      orc_ntt_forward(c, conv, i);
      for (uint64_t x = 0; x < n; x++) {
        const uint64_t y = addmod(mulmod(pm, d[(uint64_t)i * n + x], qi),
                                  Y[(uint64_t)i * n + x], qi);
        out[((uint64_t)b * (l - 1) + i) * n + x] = mulmod(submod(y, conv[x], qi), minv, qi);
      }
      free(conv);
    }
  }
  free(z);
  free(acc[0]);
  free(acc[1]);
  free(ext);
}

/* ModDown of num_polys extended polys (l+K limbs each) to l limbs. */
void orc_moddown(const orc_ctx *c, const uint64_t *in, int num_polys, int l,
                 uint64_t *out) {
  const uint64_t n = c->n;
  for (int p = 0; p < num_polys; p++)
    moddown(c, in + (uint64_t)p * (l + c->K) * n, l, out + (uint64_t)p * l * n);
}

/* ------------------------------------------------------------------ */
/* rescale, multiply by i                                               */
/* ------------------------------------------------------------------ */
void orc_rescale(const orc_ctx *c, const uint64_t *in, int num_polys, int l,
                 uint64_t *out) {
  const uint64_t n = c->n;
  const uint64_t ql = c->primes[l - 1], half = (ql - 1) / 2;
  for (int p = 0; p < num_polys; p++) {
    const uint64_t *a = in + (uint64_t)p * l * n;
    uint64_t *o = out + (uint64_t)p * (l - 1) * n;
    uint64_t *last = (uint64_t *)malloc(8 * n);
    memcpy(last, a + (uint64_t)(l - 1) * n, 8 * n);
    orc_ntt_inverse(c, last, l - 1);
#pragma omp parallel for schedule(dynamic)
    for (int i = 0; i < l - 1; i++) {
      uint64_t qi = c->primes[i];
      uint64_t qlmod = ql % qi, inv = invmod(qlmod, qi);
      uint64_t *t = (uint64_t *)malloc(8 * n);
      for (uint64_t x = 0; x < n; x++) {
        uint64_t v = last[x] % qi;
        t[x] = last[x] <= half ? v : submod(v, qlmod, qi); /* centred lift */
      }
      orc_ntt_forward(c, t, i);
      for (uint64_t x = 0; x < n; x++)
        o[(uint64_t)i * n + x] =
            mulmod(submod(a[(uint64_t)i * n + x], t[x], qi), inv, qi);
      free(t);
    }
    free(last);
  }
}

/* ModRaise: polys at one limb (q_0, NTT form) -> l_out limbs, each limb the
 * centred lift of the q_0 coefficients (NTT form). */
void orc_modraise(const orc_ctx *c, const uint64_t *in, int num_polys, int l_out,
                  uint64_t *out) {
  const uint64_t n = c->n, q0 = c->primes[0];
  uint64_t *coef = (uint64_t *)malloc(8 * n);
  for (int p = 0; p < num_polys; p++) {
    memcpy(coef, in + (uint64_t)p * n, 8 * n);
    orc_ntt_inverse(c, coef, 0);
    uint64_t *o = out + (uint64_t)p * l_out * n;
    for (int t = 0; t < l_out; t++) {
      uint64_t qt = c->primes[t];
      for (uint64_t x = 0; x < n; x++) {
        uint64_t v = coef[x];
        o[(uint64_t)t * n + x] = v > (q0 - 1) / 2 ? (qt - (q0 - v) % qt) % qt : v % qt;
      }
    }
    orc_poly_ntt(c, o, 1, l_out, 0, 0);
  }
  free(coef);
}

/* times X^(N/2): evaluation at psi^e is multiplied by psi^(e*N/2) */
void orc_mul_i(const orc_ctx *c, uint64_t *data, int num_polys, int l,
               int negative) {
  const uint64_t n = c->n;
  for (int i = 0; i < l; i++) {
    uint64_t q = c->primes[i];
    uint64_t psi = orc_find_psi(q, c->log_n);
    uint64_t w = powmod(psi, n / 2, q); /* primitive 4th root */
    uint64_t w3 = q - w;
    if (negative) {
      uint64_t t = w;
      w = w3;
      w3 = t;
    }
    for (uint64_t k = 0; k < n; k++) {
      uint64_t e = 2 * (uint64_t)bitrev((uint32_t)k, c->log_n) + 1;
      uint64_t f = (e & 3) == 1 ? w : w3;
      for (int p = 0; p < num_polys; p++) {
        uint64_t *a = data + ((uint64_t)p * l + i) * n;
        a[k] = mulmod(a[k], f, q);
      }
    }
  }
}

/* ------------------------------------------------------------------ */
/* keys and encryption                                                  */
/* ------------------------------------------------------------------ */
/* hamming > 0: sparse ternary with that many +-1 entries (partial
 * Fisher-Yates over positions driven by the ChaCha stream); hamming == 0:
 * uniform ternary. */
void orc_sample_secret(int log_n, uint64_t seed, int hamming, int64_t *s) {
  const uint64_t n = 1ull << log_n;
  uint64_t blk[8];
  memset(s, 0, 8 * n);
  if (hamming <= 0) {
    uint64_t st = stream_id(TAG_SECRET, 1, 0, 0);
    for (uint64_t k = 0; k < n; k++) {
      if (k % 8 == 0) orc_chacha_block(seed, st, k / 8, blk);
      s[k] = (int64_t)(blk[k % 8] % 3) - 1;
    }
    return;
  }
  uint32_t *perm = (uint32_t *)malloc(4 * n);
  for (uint64_t k = 0; k < n; k++) perm[k] = (uint32_t)k;
  uint64_t st = stream_id(TAG_SECRET, 0, 0, 0);
  for (uint64_t i = 0; i < (uint64_t)hamming; i++) {
    if (i % 8 == 0) orc_chacha_block(seed, st, i / 8, blk);
    uint64_t w = blk[i % 8];
    uint64_t j = i + (w >> 1) % (n - i);
    uint32_t tmp = perm[i];
    perm[i] = perm[j];
    perm[j] = tmp;
    s[perm[i]] = (w & 1) ? -1 : 1;
  }
  free(perm);
}

static inline uint64_t signed_mod(int64_t v, uint64_t q) {
  return v >= 0 ? (uint64_t)v % q : (q - ((uint64_t)(-v) % q)) % q;
}

void orc_secret_to_ntt(const orc_ctx *c, const int64_t *s, uint64_t *out) {
  const uint64_t n = c->n;
  for (int t = 0; t < c->L + c->K; t++) {
    uint64_t q = c->primes[t];
    for (uint64_t k = 0; k < n; k++) out[(uint64_t)t * n + k] = signed_mod(s[k], q);
  }
  orc_poly_ntt(c, out, 1, c->L, c->K, 0);
}

/* Key switching key from s_from to s_to, all L+K limbs, NTT form:
 * key[j][0][t] = -a*s_to + e + [t in digit j] (P mod q_t) s_from,
 * key[j][1][t] = a, for the c->digits digits of the top level. */
void orc_keygen_switch(const orc_ctx *c, const uint64_t *s_from,
                       const uint64_t *s_to, uint64_t seed, uint32_t key_tag,
                       uint64_t *key) {
  const uint64_t n = c->n;
  const int np = c->L + c->K;
  int64_t *e = (int64_t *)malloc(8 * n);
  for (int j = 0; j < c->digits; j++) {
    int lo = j * c->alpha, hi = lo + c->alpha;
    if (hi > c->L) hi = c->L;
    sample_cbd(seed, stream_id(TAG_KEY_E, key_tag, j, 0), n, e);
    uint64_t *b = key + ((uint64_t)j * 2 * np) * n;
    uint64_t *a = b + (uint64_t)np * n;
#pragma omp parallel for schedule(dynamic)
    for (int t = 0; t < np; t++) {
      uint64_t q = c->primes[t];
      uint64_t *at = a + (uint64_t)t * n, *bt = b + (uint64_t)t * n;
      sample_uniform(seed, stream_id(TAG_KEY_A, key_tag, j, t), q, n, at);
      for (uint64_t k = 0; k < n; k++) bt[k] = signed_mod(e[k], q);
      orc_ntt_forward(c, bt, t);
      uint64_t pmod = 1;
      for (int k2 = 0; k2 < c->K; k2++)
        pmod = mulmod(pmod, c->primes[c->L + k2] % q, q);
      int gadget = (t >= lo && t < hi);
      for (uint64_t k = 0; k < n; k++) {
        uint64_t v = submod(bt[k], mulmod(at[k], s_to[(uint64_t)t * n + k], q), q);
        if (gadget)
          v = addmod(v, mulmod(pmod, s_from[(uint64_t)t * n + k], q), q);
        bt[k] = v;
      }
    }
  }
  free(e);
}

void orc_keygen_rotation(const orc_ctx *c, const uint64_t *s_ntt, uint64_t g,
                         uint64_t seed, uint64_t *key) {
  const uint64_t n = c->n, m = 2 * n;
  const int np = c->L + c->K;
  /* s_to = sigma_{g^-1}(s): inverse of g in (Z/2N)^* */
  uint64_t ginv = 1;
  for (uint64_t x = 1; x < m; x += 2)
    if ((x * g) % m == 1) {
      ginv = x;
      break;
    }
  int32_t *perm = (int32_t *)malloc(4 * n);
  orc_automorphism_perm(c->log_n, ginv, perm);
  uint64_t *s_to = (uint64_t *)malloc(8 * n * np);
  for (int t = 0; t < np; t++)
    apply_perm(s_ntt + (uint64_t)t * n, s_to + (uint64_t)t * n, perm, n);
  orc_keygen_switch(c, s_ntt, s_to, seed, (uint32_t)g, key);
  free(s_to);
  free(perm);
}

void orc_keygen_relin(const orc_ctx *c, const uint64_t *s_ntt, uint64_t seed,
                      uint64_t *key) {
  const uint64_t n = c->n;
  const int np = c->L + c->K;
  uint64_t *s2 = (uint64_t *)malloc(8 * n * np);
  for (int t = 0; t < np; t++) {
    uint64_t q = c->primes[t];
    for (uint64_t k = 0; k < n; k++)
      s2[(uint64_t)t * n + k] =
          mulmod(s_ntt[(uint64_t)t * n + k], s_ntt[(uint64_t)t * n + k], q);
  }
  orc_keygen_switch(c, s2, s_ntt, seed, 0u, key);
  free(s2);
}

/* symmetric encryption of m (l limbs, NTT form): (-a*s + e + m, a) */
void orc_encrypt(const orc_ctx *c, const uint64_t *m, int l,
                 const uint64_t *s_ntt, uint64_t seed, uint64_t nonce,
                 uint64_t *ct) {
  const uint64_t n = c->n;
  int64_t *e = (int64_t *)malloc(8 * n);
  sample_cbd(seed, stream_id(TAG_ENC_E, nonce, nonce >> 24, 0), n, e);
  for (int i = 0; i < l; i++) {
    uint64_t q = c->primes[i];
    uint64_t *c0 = ct + (uint64_t)i * n, *c1 = ct + ((uint64_t)l + i) * n;
    sample_uniform(seed, stream_id(TAG_ENC_A, nonce, nonce >> 24, i), q, n, c1);
    for (uint64_t k = 0; k < n; k++) c0[k] = signed_mod(e[k], q);
    orc_ntt_forward(c, c0, i);
    for (uint64_t k = 0; k < n; k++)
      c0[k] = addmod(submod(c0[k], mulmod(c1[k], s_ntt[(uint64_t)i * n + k], q), q),
                     m[(uint64_t)i * n + k], q);
  }
  free(e);
}

void orc_decrypt(const orc_ctx *c, const uint64_t *ct, int l,
                 const uint64_t *s_ntt, uint64_t *m) {
  const uint64_t n = c->n;
  for (int i = 0; i < l; i++) {
    uint64_t q = c->primes[i];
    for (uint64_t k = 0; k < n; k++)
      m[(uint64_t)i * n + k] =
          addmod(ct[(uint64_t)i * n + k],
                 mulmod(ct[((uint64_t)l + i) * n + k], s_ntt[(uint64_t)i * n + k], q), q);
  }
}

void orc_mul_plain(const orc_ctx *c, const uint64_t *ct, const uint64_t *pt,
                   int l, int unused, uint64_t *out) {
  (void)unused;
  const uint64_t n = c->n;
  for (int p = 0; p < 2; p++)
    for (int i = 0; i < l; i++) {
      uint64_t q = c->primes[i];
      for (uint64_t k = 0; k < n; k++)
        out[((uint64_t)p * l + i) * n + k] =
            mulmod(ct[((uint64_t)p * l + i) * n + k], pt[(uint64_t)i * n + k], q);
    }
}

/* ------------------------------------------------------------------ */
/* special FFT encode / decode (Cheon-Kim-Kim-Song 2017)               */
/* ------------------------------------------------------------------ */
/* Complex products are written out as (ac - bd, ad + bc) with no fused
 * multiply-add so the GPU kernels can reproduce them bit for bit. */
static void fft_tables(int log_n, uint64_t **rot, double **kre, double **kim) {
  const uint64_t n = 1ull << log_n, m = 2 * n, half = n / 2;
  *rot = (uint64_t *)malloc(8 * half);
  uint64_t g = 1;
  for (uint64_t j = 0; j < half; j++) {
    (*rot)[j] = g;
    g = (g * 5) % m;
  }
  *kre = (double *)malloc(8 * (m + 1));
  *kim = (double *)malloc(8 * (m + 1));
  for (uint64_t k = 0; k <= m; k++) {
    double ang = 2.0 * M_PI * (double)k / (double)m;
    (*kre)[k] = cos(ang);
    (*kim)[k] = sin(ang);
  }
}

static void bitrev_complex(double *re, double *im, int slots) {
  int bits = 0;
  while ((1 << bits) < slots) bits++;
  for (int i = 0; i < slots; i++) {
    int j = (int)bitrev((uint32_t)i, bits);
    if (i < j) {
      double t = re[i];
      re[i] = re[j];
      re[j] = t;
      t = im[i];
      im[i] = im[j];
      im[j] = t;
    }
  }
}

static inline double dmul(double a, double b) {
  volatile double r = a * b;
  return r;
}

void orc_special_fft(int log_n, double *re, double *im, int slots,
                     int inverse) {
  const uint64_t m = 2ull << log_n;
  uint64_t *rot;
  double *kre, *kim;
  fft_tables(log_n, &rot, &kre, &kim);
  if (!inverse) {
    bitrev_complex(re, im, slots);
    for (int len = 2; len <= slots; len <<= 1) {
      int lenh = len >> 1;
      uint64_t lenq = (uint64_t)len << 2, gap = m / lenq;
      for (int i = 0; i < slots; i += len)
        for (int j = 0; j < lenh; j++) {
          uint64_t idx = (rot[j] % lenq) * gap;
          double ur = re[i + j], ui = im[i + j];
          double xr = re[i + j + lenh], xi = im[i + j + lenh];
          double vr = dmul(xr, kre[idx]) - dmul(xi, kim[idx]);
          double vi = dmul(xr, kim[idx]) + dmul(xi, kre[idx]);
          re[i + j] = ur + vr;
          im[i + j] = ui + vi;
          re[i + j + lenh] = ur - vr;
          im[i + j + lenh] = ui - vi;
        }
    }
  } else {
    for (int len = slots; len >= 2; len >>= 1) {
      int lenh = len >> 1;
      uint64_t lenq = (uint64_t)len << 2, gap = m / lenq;
      for (int i = 0; i < slots; i += len)
        for (int j = 0; j < lenh; j++) {
          uint64_t idx = (lenq - (rot[j] % lenq)) * gap;
          double ar = re[i + j], ai = im[i + j];
          double br = re[i + j + lenh], bi = im[i + j + lenh];
          double dr = ar - br, di = ai - bi;
          re[i + j] = ar + br;
          im[i + j] = ai + bi;
          re[i + j + lenh] = dmul(dr, kre[idx]) - dmul(di, kim[idx]);
          im[i + j + lenh] = dmul(dr, kim[idx]) + dmul(di, kre[idx]);
        }
    }
    bitrev_complex(re, im, slots);
    double inv = 1.0 / (double)slots;
    for (int j = 0; j < slots; j++) {
      re[j] = dmul(re[j], inv);
      im[j] = dmul(im[j], inv);
    }
  }
  free(rot);
  free(kre);
  free(kim);
}

/* exact residue of an integral double: v = mant * 2^exp */
static uint64_t double_mod(double v, uint64_t q) {
  if (v == 0.0) return 0;
  int neg = v < 0;
  double a = neg ? -v : v;
  uint64_t r;
  if (a < 9223372036854775808.0) {
    r = (uint64_t)a % q;
  } else {
    int e;
    double f = frexp(a, &e); /* a = f * 2^e, f in [0.5,1) */
    uint64_t mant = (uint64_t)ldexp(f, 53);
    r = mulmod(mant % q, powmod(2, (uint64_t)(e - 53), q), q);
  }
  return neg ? (r ? q - r : 0) : r;
}

void orc_encode(const orc_ctx *c, const double *re_in, const double *im_in,
                int slots, double scale, int q_limbs, int p_limbs,
                uint64_t *out) {
  const uint64_t n = c->n, half = n / 2;
  double *re = (double *)malloc(8 * slots), *im = (double *)malloc(8 * slots);
  memcpy(re, re_in, 8 * slots);
  memcpy(im, im_in, 8 * slots);
  orc_special_fft(c->log_n, re, im, slots, 1);
  double *coef = (double *)calloc(n, 8);
  uint64_t gap = half / (uint64_t)slots;
  for (int j = 0; j < slots; j++) {
    coef[(uint64_t)j * gap] = nearbyint(dmul(re[j], scale));
    coef[(uint64_t)j * gap + half] = nearbyint(dmul(im[j], scale));
  }
  int limbs = q_limbs + p_limbs;
  for (int t = 0; t < limbs; t++) {
    uint64_t q = c->primes[limb_prime(c, q_limbs, t)];
    for (uint64_t k = 0; k < n; k++) out[(uint64_t)t * n + k] = double_mod(coef[k], q);
  }
  orc_poly_ntt(c, out, 1, q_limbs, p_limbs, 0);
  free(coef);
  free(re);
  free(im);
}

/* decode from the first min(l, 2) limbs by exact 128-bit CRT, centred */
void orc_decode(const orc_ctx *c, const uint64_t *in, int l, int slots,
                double scale, double *re, double *im) {
  const uint64_t n = c->n, half = n / 2;
  int use = l < 2 ? l : 2;
  uint64_t *a = (uint64_t *)malloc(8 * n * use);
  memcpy(a, in, 8 * n * use);
  orc_poly_ntt(c, a, 1, use, 0, 1);
  double *coef = (double *)malloc(8 * n);
  uint64_t q0 = c->primes[0];
  if (use == 1) {
    for (uint64_t k = 0; k < n; k++) {
      uint64_t v = a[k];
      coef[k] = v > q0 / 2 ? -(double)(q0 - v) : (double)v;
    }
  } else {
    uint64_t q1 = c->primes[1];
    u128 Q = (u128)q0 * q1;
    uint64_t q0inv = invmod(q0 % q1, q1);
    for (uint64_t k = 0; k < n; k++) {
      /* Garner: v = a0 + q0 * ((a1 - a0) * q0^-1 mod q1) */
      uint64_t a0 = a[k], a1 = a[n + k];
      uint64_t h = mulmod(submod(a1, a0 % q1, q1), q0inv, q1);
      u128 v = (u128)a0 + (u128)q0 * h;
      if (v > Q / 2)
        coef[k] = -(double)(Q - v);
      else
        coef[k] = (double)v;
    }
  }
  uint64_t gap = half / (uint64_t)slots;
  for (int j = 0; j < slots; j++) {
    re[j] = coef[(uint64_t)j * gap] / scale;
    im[j] = coef[(uint64_t)j * gap + half] / scale;
  }
  orc_special_fft(c->log_n, re, im, slots, 0);
  free(coef);
  free(a);
}

/* ------------------------------------------------------------------ */
/* BSGS inner multiply-accumulate (the pt x baby half of                */
/* hoisted_mac_sum, llama3fhe/operators/linear/operator.py:320-330):    */
/*   out[c][g] = sum_b pts[g B + b] * babies[c][b]   (mod q_i, limb-wise) */
/* babies [C][B][2][l][N], pts [G B][l][N], out [C][G][2][l][N].        */
/* ------------------------------------------------------------------ */
void orc_bsgs_mac(const orc_ctx *c, const uint64_t *babies, int num_cts,
                  int baby_count, const uint64_t *pts, int giant_count, int q_limbs,
                  int p_limbs, uint64_t *out) {
  const uint64_t n = c->n;
  const int l = q_limbs + p_limbs; /* limb t: prime t, or P prime t - q_limbs */
  const uint64_t limb = n, ct_words = 2 * (uint64_t)l * n;
#pragma omp parallel for schedule(dynamic) collapse(2)
  for (int g = 0; g < giant_count; g++)
    for (int i = 0; i < l; i++) {
      const uint64_t q = c->primes[i < q_limbs ? i : c->L + i - q_limbs];
      for (int ct = 0; ct < num_cts; ct++)
        for (int p = 0; p < 2; p++) {
          uint64_t *o = out + ((uint64_t)ct * giant_count + g) * ct_words +
                        ((uint64_t)p * l + i) * limb;
          for (uint64_t k = 0; k < n; k++) {
            u128 acc = 0;
            for (int b = 0; b < baby_count; b++) {
              const uint64_t *bb = babies + ((uint64_t)ct * baby_count + b) * ct_words +
                                   ((uint64_t)p * l + i) * limb;
              const uint64_t *pt = pts + ((uint64_t)g * baby_count + b) * l * n +
                                   (uint64_t)i * limb;
              acc += (u128)bb[k] * pt[k];
              if ((b & 7) == 7) acc %= q; /* keep the sum below 2^128 */
            }
            o[k] = (uint64_t)(acc % q);
          }
        }
    }
}
