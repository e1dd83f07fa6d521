#include <atomic>
// Context creation: RNS primes, NTT twiddle tables, key-switch constants.
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "b2f_internal.h"

using u128 = unsigned __int128;

namespace b2f {

static thread_local char g_err[1024];

void set_error(const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof g_err, fmt, ap);
  va_end(ap);
}

int cuda_status(cudaError_t e, const char *what) {
  set_error("%s: %s", what, cudaGetErrorString(e));
  return e == cudaErrorMemoryAllocation ? B2F_ERR_NOMEM : B2F_ERR_CUDA;
}

// ---- host number theory (independent of any oracle code) ----
static uint64_t h_mulmod(uint64_t a, uint64_t b, uint64_t q) {
  return (uint64_t)(((u128)a * b) % q);
}
static uint64_t h_pow(uint64_t a, uint64_t e, uint64_t q) {
  uint64_t r = 1 % q;
  a %= q;
  for (; e; e >>= 1) {
    if (e & 1) r = h_mulmod(r, a, q);
    a = h_mulmod(a, a, q);
  }
  return r;
}
static uint64_t h_inv(uint64_t a, uint64_t q) { return h_pow(a % q, q - 2, q); }
static uint64_t h_shoup(uint64_t w, uint64_t q) {
  return (uint64_t)(((u128)w << 64) / q);
}
static ulonglong2 shoup_pair(uint64_t w, uint64_t q) {
  return make_ulonglong2(w, h_shoup(w, q));
}

static bool h_is_prime(uint64_t n) {
  if (n < 2) return false;
  for (uint64_t p : {2ull, 3ull, 5ull, 7ull, 11ull, 13ull, 17ull, 19ull, 23ull,
                     29ull, 31ull, 37ull}) {
    if (n == p) return true;
    if (n % p == 0) return false;
  }
  uint64_t d = n - 1;
  int s = 0;
  while (!(d & 1)) d >>= 1, ++s;
  for (uint64_t a : {2ull, 325ull, 9375ull, 28178ull, 450775ull, 9780504ull,
                     1795265022ull}) {
    a %= n;
    if (!a) continue;
    uint64_t x = h_pow(a, d, n);
    if (x == 1 || x == n - 1) continue;
    bool composite = true;
    for (int r = 1; r < s && composite; ++r) {
      x = h_mulmod(x, x, n);
      if (x == n - 1) composite = false;
    }
    if (composite) return false;
  }
  return true;
}

static uint32_t h_bitrev(uint32_t x, int bits) {
  uint32_t r = 0;
  for (int i = 0; i < bits; ++i) r = (r << 1) | ((x >> i) & 1);
  return r;
}

// smallest primitive 2N-th root of unity mod q
static uint64_t h_min_psi(uint64_t q, int log_n) {
  const uint64_t n = 1ull << log_n, m = 2 * n;
  uint64_t psi0 = 0;
  for (uint64_t g = 2; g < q && !psi0; ++g) {
    uint64_t c = h_pow(g, (q - 1) / m, q);
    if (h_pow(c, n, q) == q - 1) psi0 = c;
  }
  uint64_t best = psi0, sq = h_mulmod(psi0, psi0, q), cur = psi0;
  for (uint64_t k = 1; k < n; ++k) {
    cur = h_mulmod(cur, sq, q);
    if (cur < best) best = cur;
  }
  return best;
}

static Mod make_mod(uint64_t q) {
  u128 m = (~(u128)0) / q;  // floor((2^128 - 1)/q) == floor(2^128/q), q odd
  Mod M;
  M.q = q;
  M.m_lo = (uint64_t)m;
  M.m_hi = (uint64_t)(m >> 64);
  const int k = 63 - __builtin_clzll(q);
  M.mu = (uint64_t)(((u128)1 << (64 + k)) / q);
  return M;
}

template <typename T>
static int upload(b2f_context *ctx, T **dst, const std::vector<T> &src) {
  void *p = nullptr;
  B2F_CUDA(cudaMalloc(&p, sizeof(T) * (src.size() ? src.size() : 1)));
  ctx->owned.push_back(p);
  if (!src.empty())
    B2F_CUDA(cudaMemcpy(p, src.data(), sizeof(T) * src.size(),
                        cudaMemcpyHostToDevice));
  *dst = static_cast<T *>(p);
  return B2F_OK;
}

static uint64_t prod_mod(const std::vector<uint64_t> &primes, int lo, int hi,
                         int skip, uint64_t m) {
  uint64_t r = 1 % m;
  for (int i = lo; i < hi; ++i)
    if (i != skip) r = h_mulmod(r, primes[i] % m, m);
  return r;
}

static int build_tables(b2f_context *ctx) {
  const int L = ctx->L, K = ctx->K, np = L + K, n = ctx->n;
  const auto &P = ctx->primes;
  std::vector<Mod> mods(np);
  std::vector<ulonglong2> twf((size_t)np * n), twi((size_t)np * n), ninv(np),
      ifac(np);
  ctx->psi.resize(np);
  std::vector<uint64_t> pw(n), ipw(n);
  for (int i = 0; i < np; ++i) {
    const uint64_t q = P[i];
    mods[i] = make_mod(q);
    const uint64_t psi = h_min_psi(q, ctx->log_n), ipsi = h_inv(psi, q);
    ctx->psi[i] = psi;
    uint64_t a = 1, b = 1;
    for (int k = 0; k < n; ++k) {
      pw[k] = a;
      ipw[k] = b;
      a = h_mulmod(a, psi, q);
      b = h_mulmod(b, ipsi, q);
    }
    for (int k = 0; k < n; ++k) {
      uint32_t r = h_bitrev((uint32_t)k, ctx->log_n);
      twf[(size_t)i * n + k] = shoup_pair(pw[r], q);
      twi[(size_t)i * n + k] = shoup_pair(ipw[r], q);
    }
    ninv[i] = shoup_pair(h_inv((uint64_t)n % q, q), q);
    ifac[i] = shoup_pair(pw[n / 2], q);
  }
  int rc;
  if ((rc = upload(ctx, &ctx->d_primes, P))) return rc;
  if ((rc = upload(ctx, &ctx->d_mod, mods))) return rc;
  {
    std::vector<Red79> red(P.size());
    for (size_t i = 0; i < P.size(); ++i) {
      const uint64_t q = P[i];
      const unsigned __int128 two64 = (unsigned __int128)1 << 64;
      const uint64_t r = (uint64_t)(two64 % q);
      red[i] = Red79{q, r, (uint64_t)(((unsigned __int128)r << 64) / q),
                     (uint64_t)(two64 / q)};
    }
    if ((rc = upload(ctx, &ctx->d_red79, red))) return rc;
  }
  if ((rc = upload(ctx, &ctx->d_tw_fwd, twf))) return rc;
  if ((rc = upload(ctx, &ctx->d_tw_inv, twi))) return rc;
  // binary64 arithmetic (every prime below 2^50): twiddles as doubles and 1/q
  ctx->fp64_ok = true;
  for (int i = 0; i < np; ++i) ctx->fp64_ok = ctx->fp64_ok && P[i] < (1ull << 50);
  if (ctx->fp64_ok) {
    std::vector<double> tdf((size_t)np * n), tdi((size_t)np * n), qinv(np);
    for (size_t k = 0; k < tdf.size(); ++k) {
      tdf[k] = (double)twf[k].x;
      tdi[k] = (double)twi[k].x;
    }
    for (int i = 0; i < np; ++i) qinv[i] = 1.0 / (double)P[i];
    if ((rc = upload(ctx, &ctx->d_twd_fwd, tdf))) return rc;
    if ((rc = upload(ctx, &ctx->d_twd_inv, tdi))) return rc;
    if ((rc = upload(ctx, &ctx->d_qinv, qinv))) return rc;
  }
  ctx->fp64 = ctx->fp64_ok;
  if ((rc = upload(ctx, &ctx->d_ninv, ninv))) return rc;
  if ((rc = upload(ctx, &ctx->d_i_factor, ifac))) return rc;

  // ModDown constants (level independent)
  std::vector<ulonglong2> md_scale(K ? K : 1), md_conv((size_t)L * (K ? K : 1)),
      md_pinv(L);
  std::vector<uint64_t> pmod(L);
  for (int k = 0; k < K; ++k) {
    uint64_t pk = P[L + k];
    uint64_t phat = prod_mod(P, L, L + K, L + k, pk);
    uint64_t s = h_mulmod(h_inv((uint64_t)n % pk, pk), h_inv(phat, pk), pk);
    md_scale[k] = shoup_pair(s, pk);
  }
  for (int i = 0; i < L; ++i) {
    uint64_t qi = P[i];
    for (int k = 0; k < K; ++k)
      md_conv[(size_t)i * K + k] =
          shoup_pair(prod_mod(P, L, L + K, L + k, qi), qi);
    uint64_t pm = prod_mod(P, L, L + K, -1, qi);
    pmod[i] = pm;
    md_pinv[i] = shoup_pair(h_inv(pm, qi), qi);
  }
  if ((rc = upload(ctx, &ctx->d_moddown_scale, md_scale))) return rc;
  if (K) {
    std::vector<uint8_t> mdb(conv_rows(L) * conv_kpad(K));
    conv_bytes(
        mdb.data(), L, K, conv_kpad(K),
        [&](int t, int k) { return md_conv[(size_t)t * K + k].x; },
        [&](int t) { return P[t]; });
    if ((rc = upload(ctx, &ctx->d_moddown_bytes, mdb))) return rc;
  }
  if ((rc = upload(ctx, &ctx->d_moddown_pinv, md_pinv))) return rc;
  if (ctx->fp64_ok && K >= 1 && K <= 4) {
    std::vector<double> mdd((size_t)L * K);
    for (size_t i = 0; i < mdd.size(); ++i) mdd[i] = (double)md_conv[i].x;
    if ((rc = upload(ctx, &ctx->d_md_conv_f64, mdd))) return rc;
  }
  if ((rc = upload(ctx, &ctx->d_pmod, pmod))) return rc;

  // per-level ModUp and rescale constants
  const int alpha = ctx->alpha;
  ctx->levels.assign(L + 1, LevelTables{});
  for (int l = 1; l <= L; ++l) {
    LevelTables &T = ctx->levels[l];
    T.l = l;
    T.beta = (l + alpha - 1) / alpha;
    std::vector<ulonglong2> scale(l), conv((size_t)T.beta * (l + K) * alpha);
    for (int j = 0; j < T.beta; ++j) {
      int lo = j * alpha, hi = std::min(lo + alpha, l);
      for (int i = lo; i < hi; ++i) {
        uint64_t qi = P[i];
        uint64_t qhat = prod_mod(P, lo, hi, i, qi);
        scale[i] = shoup_pair(
            h_mulmod(h_inv((uint64_t)n % qi, qi), h_inv(qhat, qi), qi), qi);
      }
      for (int t = 0; t < l + K; ++t) {
        int pt_idx = t < l ? t : L + (t - l);
        uint64_t pt = P[pt_idx];
        for (int i = lo; i < lo + alpha; ++i) {
          ulonglong2 v = make_ulonglong2(0, 0);
          if (i < hi) v = shoup_pair(prod_mod(P, lo, hi, i, pt), pt);
          conv[((size_t)j * (l + K) + t) * alpha + (i - lo)] = v;
        }
      }
    }
    if ((rc = upload(ctx, &T.modup_scale, scale))) return rc;
    {
      // targets of digit j: limbs t < l+K outside [lo, hi), in order
      const int lk = l + K;
      T.modup_bytes_stride = conv_rows(lk) * conv_kpad(alpha);
      std::vector<uint8_t> mb(T.modup_bytes_stride * T.beta);
      for (int j = 0; j < T.beta; ++j) {
        const int lo = j * alpha, hi = std::min(lo + alpha, l), w = hi - lo;
        auto tgt = [&](int tau) { return tau < lo ? tau : tau + w; };
        conv_bytes(
            mb.data() + (size_t)j * T.modup_bytes_stride, lk - w, w,
            conv_kpad(alpha),
            [&](int tau, int i) {
              return conv[((size_t)j * lk + tgt(tau)) * alpha + i].x;
            },
            [&](int tau) {
              const int t = tgt(tau);
              return P[t < l ? t : L + (t - l)];
            });
      }
      if ((rc = upload(ctx, &T.modup_bytes, mb))) return rc;
    }
    std::vector<ulonglong2> rinv(l > 1 ? l - 1 : 1);
    std::vector<uint64_t> rq(l > 1 ? l - 1 : 1);
    for (int i = 0; i + 1 < l; ++i) {
      uint64_t qi = P[i], ql = P[l - 1] % qi;
      rq[i] = ql;
      rinv[i] = shoup_pair(h_inv(ql, qi), qi);
    }
    if ((rc = upload(ctx, &T.rescale_inv, rinv))) return rc;
    if ((rc = upload(ctx, &T.rescale_qlast, rq))) return rc;
    if (l >= 2 && K >= 1) {
      // removed limbs of the fused relinearise + rescale
      const int R = K + 1;
      std::vector<uint64_t> rp(R);
      rp[0] = P[l - 1];
      for (int k = 0; k < K; ++k) rp[1 + k] = P[L + k];
      auto mhat = [&](int r, uint64_t m) {  // (M / r) mod m
        uint64_t v = 1 % m;
        for (int r2 = 0; r2 < R; ++r2)
          if (r2 != r) v = h_mulmod(v, rp[r2] % m, m);
        return v;
      };
      std::vector<ulonglong2> msc(R);
      std::vector<double> mri(R);
      for (int r = 0; r < R; ++r) {
        const uint64_t pr = rp[r];
        msc[r] = shoup_pair(
            h_mulmod(h_inv((uint64_t)n % pr, pr), h_inv(mhat(r, pr), pr), pr), pr);
        mri[r] = 1.0 / (double)pr;
      }
      const int kp = conv_kpad(R + 1);
      std::vector<uint8_t> mb(conv_rows(l - 1) * kp);
      conv_bytes(
          mb.data(), l - 1, R + 1, kp,
          [&](int t, int r) -> uint64_t {
            const uint64_t qt = P[t];
            if (r < R) return mhat(r, qt);
            const uint64_t m = h_mulmod(mhat(0, qt), rp[0] % qt, qt);  // M mod q_t
            return m ? qt - m : 0;
          },
          [&](int t) { return P[t]; });
      if ((rc = upload(ctx, &T.mdr_scale, msc))) return rc;
      if ((rc = upload(ctx, &T.mdr_rinv, mri))) return rc;
      if ((rc = upload(ctx, &T.mdr_bytes, mb))) return rc;
    }
  }

  // FFT tables: ksi_k = exp(2 pi i k / M), rotation group 5^j mod M
  const uint64_t M = 2ull * n;
  std::vector<double2> ksi(M + 1);
  for (uint64_t k = 0; k <= M; ++k) {
    double ang = 2.0 * M_PI * (double)k / (double)M;
    ksi[k] = make_double2(cos(ang), sin(ang));
  }
  std::vector<uint32_t> rot(n / 2);
  uint64_t g = 1;
  for (int j = 0; j < n / 2; ++j) {
    rot[j] = (uint32_t)g;
    g = (g * 5) % M;
  }
  if ((rc = upload(ctx, &ctx->d_ksi, ksi))) return rc;
  if ((rc = upload(ctx, &ctx->d_rot_group, rot))) return rc;
  return B2F_OK;
}

std::atomic<unsigned long long> g_launch_count{0};
void note_launch() { g_launch_count.fetch_add(1, std::memory_order_relaxed); }

const LimbJob *job_table(b2f_context *ctx, const std::vector<int> &key,
                         const std::vector<LimbJob> &jobs) {
  std::lock_guard<std::mutex> g(ctx->mu);
  auto it = ctx->jobs.find(key);
  if (it != ctx->jobs.end()) return it->second;
  void *p = nullptr;
  cudaError_t e = cudaMalloc(&p, sizeof(LimbJob) * jobs.size());
  if (e == cudaSuccess)
    e = cudaMemcpy(p, jobs.data(), sizeof(LimbJob) * jobs.size(),
                   cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    if (p) cudaFree(p);
    cuda_status(e, "job table upload");
    return nullptr;
  }
  ctx->owned.push_back(p);
  ctx->jobs[key] = static_cast<LimbJob *>(p);
  return static_cast<LimbJob *>(p);
}

}  // namespace b2f

using namespace b2f;

extern "C" {

const char *b2f_last_error(void) { return g_err; }
unsigned long long b2f_launch_count(void) {
  return g_launch_count.load(std::memory_order_relaxed);
}
int b2f_abi_version(void) { return 1; }

int b2f_generate_primes(int log_n, int bits, int count, int mode,
                        const uint64_t *exclude, int n_exclude, uint64_t *out) {
  B2F_CHECK_ARG(log_n >= 1 && log_n <= 20 && bits > log_n + 1 && bits <= 61 &&
                    count >= 0 && out,
                "b2f_generate_primes: bad arguments");
  const uint64_t m = 2ull << log_n, base = 1ull << bits;
  uint64_t below = base + 1 - m, above = base + 1 + m;
  int found = 0, side = 0;
  auto taken = [&](uint64_t c) {
    for (int i = 0; i < n_exclude; ++i)
      if (exclude[i] == c) return true;
    for (int i = 0; i < found; ++i)
      if (out[i] == c) return true;
    return false;
  };
  while (found < count) {
    uint64_t c;
    if (mode == 0 || side == 0) {
      if (below <= m) {
        set_error("b2f_generate_primes: ran out of %d-bit primes", bits);
        return B2F_ERR_ARG;
      }
      c = below;
      below -= m;
    } else {
      c = above;
      above += m;
    }
    if (h_is_prime(c) && !taken(c)) {
      out[found++] = c;
      if (mode == 1) side ^= 1;
    }
  }
  return B2F_OK;
}

int b2f_context_create(int log_n, const uint64_t *q, int L, const uint64_t *p,
                       int K, int dnum, int device, b2f_context **out) {
  if (out) *out = nullptr;
  B2F_CHECK_ARG(out && q && L >= 1 && K >= 0 && (K == 0 || p) && dnum >= 1,
                "b2f_context_create: bad arguments");
  if (log_n != kLogN) {
    set_error("b2f_context_create: log_n=%d unsupported (kernels are built "
              "for N=2^16)", log_n);
    return B2F_ERR_UNSUPPORTED;
  }
  B2F_CHECK_ARG(L + K <= 64, "b2f_context_create: at most 64 primes");
  for (int i = 0; i < L + K; ++i) {
    uint64_t v = i < L ? q[i] : p[i - L];
    B2F_CHECK_ARG(v < (1ull << 61) && v > (1ull << 33) &&
                      v % (2ull << log_n) == 1 && h_is_prime(v),
                  "b2f_context_create: prime %d (%llu) is not an NTT prime "
                  "in (2^33, 2^61)", i, (unsigned long long)v);
  }
  B2F_CUDA(cudaSetDevice(device));
  auto *ctx = new b2f_context();
  ctx->device = device;
  ctx->L = L;
  ctx->K = K;
  ctx->dnum = dnum;
  ctx->alpha = (L + dnum - 1) / dnum;
  ctx->digits = (L + ctx->alpha - 1) / ctx->alpha;
  ctx->primes.assign(q, q + L);
  for (int k = 0; k < K; ++k) ctx->primes.push_back(p[k]);
  int rc = build_tables(ctx);
  if (rc) {
    b2f_context_destroy(ctx);
    return rc;
  }
  *out = ctx;
  return B2F_OK;
}

int b2f_context_destroy(b2f_context *ctx) {
  if (!ctx) return B2F_OK;
  cudaSetDevice(ctx->device);
  for (void *p : ctx->owned) cudaFree(p);
  delete ctx;
  return B2F_OK;
}

int b2f_context_set_arith(b2f_context *ctx, int mode) {
  B2F_CHECK_ARG(ctx, "b2f_context_set_arith: null context");
  B2F_CHECK_ARG(mode >= 0 && mode <= 2, "b2f_context_set_arith: mode %d not in 0..2",
                mode);
  if (mode == 2 && !ctx->fp64_ok) {
    set_error("b2f_context_set_arith: binary64 arithmetic needs every prime "
              "below 2^50");
    return B2F_ERR_UNSUPPORTED;
  }
  ctx->fp64 = mode == 1 ? false : ctx->fp64_ok;
  return B2F_OK;
}

int b2f_context_arith(const b2f_context *ctx) {
  return ctx && ctx->fp64 ? 2 : 1;
}

int b2f_context_info(const b2f_context *ctx, int *info) {
  B2F_CHECK_ARG(ctx && info, "b2f_context_info: null argument");
  info[0] = ctx->log_n;
  info[1] = ctx->L;
  info[2] = ctx->K;
  info[3] = ctx->dnum;
  info[4] = ctx->alpha;
  info[5] = ctx->digits;
  return B2F_OK;
}

uint64_t b2f_galois_element(int log_n, int64_t rotation) {
  const uint64_t m = 2ull << log_n, slots = 1ull << (log_n - 1);
  if ((uint64_t)rotation == m - 1) return m - 1;
  int64_t r = rotation % (int64_t)slots;
  if (r < 0) r += (int64_t)slots;
  return h_pow(5, (uint64_t)r, m);
}

}  // extern "C"
