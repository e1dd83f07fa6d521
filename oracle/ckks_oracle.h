/*
 * ckks_oracle.h -- CPU restatement of the CKKS evaluation ops on the hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (the easyfhe package and
 * libb200fhe.so) links, loads or calls this code.  Only tests/, the smoke()
 * check in __graft_entry__.py and bench.py's cpu_baseline / reference arm use
 * it, and there only as the checker or as the timed CPU baseline.
 *
 * What it restates.  The reference (Azathoth13/easyfhe-llama3-8b) delegates all
 * CKKS arithmetic to the external EasyFHE package (NOTICE:10, docs/SETUP.md:34),
 * which is not vendored, not installed and has no pinned version.  Its residue
 * conventions are therefore unknown; this oracle restates the published
 * algorithms instead:
 *   - negacyclic NTT, Cooley-Tukey forward / Gentleman-Sande inverse with
 *     bit-reversed psi tables (Longa-Naehrig 2016);
 *   - RNS-CKKS encode/decode through the special FFT of Cheon-Kim-Kim-Song
 *     (2017) and the RNS variant of Cheon-Han-Kim-Kim-Song (2018);
 *   - hybrid key switching with dnum digits and K special primes, fast base
 *     conversion for ModUp and ModDown (Han-Ki 2020);
 *   - rescale by the last prime with a centred lift;
 *   - Galois automorphisms X -> X^g, g = 5^r mod 2N, conjugation g = 2N-1.
 * The call semantics it has to honour come from the reference's callers:
 * rotations (llama3fhe/operators/linear/operator.py:320-339), conjugation
 * index M-1 (llama3fhe/operators/linear/complex.py:47-51), rescale after the
 * BSGS MAC (operator.py:380-392), level drop by align_to
 * (llama3fhe/operators/primitives.py:100-155), multiply by i
 * (complex.py:10-37).
 *
 * Parity status: residue parity against EasyFHE is UNPINNED (the library is
 * absent).  The oracle itself is pinned by known-answer properties computed
 * independently in the tests (schoolbook negacyclic products, the DFT
 * definition of the NTT ordering, exact CRT base conversion with Python
 * integers, the canonical-embedding definition of encode) and by golden
 * vectors generated from the reference's own NumPy code (tests/golden/).
 */
#ifndef CKKS_ORACLE_H
#define CKKS_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct orc_ctx orc_ctx;

/* number theory */
int      orc_is_prime(uint64_t n);
uint64_t orc_find_psi(uint64_t q, int log_n);
int      orc_gen_primes(int log_n, int bits, int count, int mode,
                        const uint64_t *exclude, int n_exclude, uint64_t *out);
void     orc_chacha_block(uint64_t seed, uint64_t stream, uint64_t counter,
                          uint64_t out[8]);

/* context: Q primes q[0..L), special primes p[0..K), dnum key-switch digits */
orc_ctx *orc_ctx_create(int log_n, const uint64_t *q, int L, const uint64_t *p,
                        int K, int dnum);
void     orc_ctx_free(orc_ctx *ctx);
int      orc_alpha(const orc_ctx *ctx);
int      orc_num_digits(const orc_ctx *ctx);

/* limb-level transforms.  prime_idx indexes [q_0..q_{L-1}, p_0..p_{K-1}] */
void orc_ntt_forward(const orc_ctx *ctx, uint64_t *a, int prime_idx);
void orc_ntt_inverse(const orc_ctx *ctx, uint64_t *a, int prime_idx);
/* polys of q_limbs Q limbs followed by p_limbs P limbs, num_polys polys */
void orc_poly_ntt(const orc_ctx *ctx, uint64_t *data, int num_polys,
                  int q_limbs, int p_limbs, int inverse);

/* NTT-domain automorphism permutation: out[k] = in[perm[k]] */
void orc_automorphism_perm(int log_n, uint64_t g, int32_t *perm);
uint64_t orc_galois_element(int log_n, int64_t rotation);

/* fast base conversion of one digit (coefficient domain) */
void orc_modup_digit(const orc_ctx *ctx, const uint64_t *x_coeff, int l,
                     int digit, uint64_t *out_coeff /* (l+K) limbs */);

/* hybrid key switching of c1 (NTT form, l limbs) with key
 * [digits][2][L+K][N] (NTT form); d0,d1: l limbs each (NTT form) */
void orc_keyswitch(const orc_ctx *ctx, const uint64_t *c1, int l,
                   const uint64_t *key, uint64_t *d0, uint64_t *d1);
/* HRotate: ct (2 polys x l limbs) -> out; key generated for galois g */
void orc_rotate(const orc_ctx *ctx, const uint64_t *ct, int l, uint64_t g,
                const uint64_t *key, uint64_t *out);
/* hoisted rotations: one ModUp, then one inner product + ModDown per key */
void orc_rotate_hoisted(const orc_ctx *ctx, const uint64_t *ct, int l,
                        int count, const uint64_t *galois,
                        const uint64_t *const *keys, uint64_t *out);
void orc_rotate_hoisted_ext(const orc_ctx *ctx, const uint64_t *ct, int l,
                            int count, const uint64_t *galois,
                            const uint64_t *const *keys, uint64_t *out);
/* relinearisation fused with the following rescale: ct3 (3 x l limbs) ->
 * out (2 x (l-1) limbs), one division by P q_{l-1} */
void orc_relin_rescale(const orc_ctx *c, const uint64_t *ct3, int l,
                       const uint64_t *key, uint64_t *out);
void orc_moddown(const orc_ctx *ctx, const uint64_t *in, int num_polys, int l,
                 uint64_t *out);
void orc_rescale(const orc_ctx *ctx, const uint64_t *in, int num_polys, int l,
                 uint64_t *out);
void orc_modraise(const orc_ctx *ctx, const uint64_t *in, int num_polys,
                  int l_out, uint64_t *out);
void orc_mul_i(const orc_ctx *ctx, uint64_t *data, int num_polys, int l,
               int negative);

/* keys and encryption */
void orc_sample_secret(int log_n, uint64_t seed, int hamming, int64_t *s);
void orc_secret_to_ntt(const orc_ctx *ctx, const int64_t *s,
                       uint64_t *s_ntt /* (L+K) limbs */);
void orc_keygen_switch(const orc_ctx *ctx, const uint64_t *s_from_ntt,
                       const uint64_t *s_to_ntt, uint64_t seed,
                       uint32_t key_tag, uint64_t *key);
void orc_keygen_rotation(const orc_ctx *ctx, const uint64_t *s_ntt, uint64_t g,
                         uint64_t seed, uint64_t *key);
void orc_keygen_relin(const orc_ctx *ctx, const uint64_t *s_ntt, uint64_t seed,
                      uint64_t *key);
void orc_encrypt(const orc_ctx *ctx, const uint64_t *m_ntt, int l,
                 const uint64_t *s_ntt, uint64_t seed, uint64_t nonce,
                 uint64_t *ct);
void orc_decrypt(const orc_ctx *ctx, const uint64_t *ct, int l,
                 const uint64_t *s_ntt, uint64_t *m_ntt);

/* encoding */
void orc_encode(const orc_ctx *ctx, const double *re, const double *im,
                int slots, double scale, int q_limbs, int p_limbs,
                uint64_t *out_ntt);
void orc_decode(const orc_ctx *ctx, const uint64_t *in_ntt, int l, int slots,
                double scale, double *re, double *im);
void orc_special_fft(int log_n, double *re, double *im, int slots, int inverse);

/* elementwise helpers (NTT form, same limb layout on both operands) */
/* out[c][g] = sum_b pts[g B + b] * babies[c][b] (the inner multiply-accumulate
 * of a BSGS linear, llama3fhe/operators/linear/operator.py:320-330). */
void orc_bsgs_mac(const orc_ctx *ctx, const uint64_t *babies, int num_cts,
                  int baby_count, const uint64_t *pts, int giant_count, int q_limbs,
                  int p_limbs, uint64_t *out);
void orc_mul_plain(const orc_ctx *ctx, const uint64_t *ct, const uint64_t *pt,
                   int l, int q_limbs_pt_stride, uint64_t *out);

#ifdef __cplusplus
}
#endif
#endif
