/*
 * b200fhe.h -- C ABI of libb200fhe, the B200 (sm_100a) CKKS evaluation
 * backend that replaces the external EasyFHE runtime behind the reference's
 * `easyfhe.fhe` Python surface.
 *
 * Conventions
 *  - Every pointer named *data / *in / *out / *key / *ws is a DEVICE pointer
 *    on the context's device; sizes are element counts unless named *_bytes.
 *  - A polynomial at l limbs is l contiguous limbs of N = 2^16 uint64
 *    residues (limb i modulo prime i).  An extended polynomial holds l Q-limbs
 *    followed by K P-limbs.  A ciphertext is two polynomials back to back
 *    (c0 then c1); a batch of ciphertexts is contiguous.
 *  - Polynomials are in the evaluation (NTT) form unless a function says
 *    otherwise; evaluation k is a(psi^(2*bitrev(k)+1)), psi the smallest
 *    primitive 2N-th root of unity modulo the limb's prime.
 *  - Residues are fully reduced ([0, q)) on input and output.
 *  - Device buffers start on a 32-byte boundary (every cudaMalloc'd or
 *    torch-allocated buffer, and any limb offset into one, does); the kernels
 *    move whole 32-byte sectors.
 *  - `stream` is a cudaStream_t (NULL = legacy default stream); every call is
 *    asynchronous on it.  Scratch memory is passed in as `ws`/`ws_bytes`
 *    (size from the matching *_workspace query, 256-byte aligned); ws == NULL
 *    makes the call allocate and free its scratch stream-ordered
 *    (cudaMallocAsync).  A misaligned buffer is refused with B2F_ERR_ARG
 *    where a transform or a workspace receives it.
 *  - Every function returns 0 (B2F_OK) or a b2f_status; the message of the
 *    last failure on the calling thread is b2f_last_error().
 *
 * Reference citations are to Azathoth13/easyfhe-llama3-8b; the Python names
 * are the `easyfhe.fhe` calls the reference makes at those lines.
 */
#ifndef B200FHE_H
#define B200FHE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct b2f_context b2f_context;

typedef enum {
  B2F_OK = 0,
  B2F_ERR_ARG = 1,         /* bad argument: shape, level, pointer, size */
  B2F_ERR_CUDA = 2,        /* a CUDA runtime call failed */
  B2F_ERR_NOMEM = 3,       /* device allocation failed */
  B2F_ERR_UNSUPPORTED = 4  /* parameters outside what the kernels implement */
} b2f_status;

/* Message of the last failure on the calling thread ("" if none). */
const char *b2f_last_error(void);
/* Kernel launches the library has issued in this process (all contexts,
 * all threads; a relaxed counter).  No counterpart in the reference:
 * instrumentation, so a caller can count the launches inside a timed region. */
unsigned long long b2f_launch_count(void);
int b2f_abi_version(void);

/* NTT-friendly primes q = 1 mod 2N: mode 0 descending below 2^bits, mode 1
 * alternating just below / just above 2^bits.  Serves the modulus chain of
 * fhe.CKKSContextSpec(depth, log_n, dnum, dcrt_bits, first_mod)
 * (llama3fhe/application/session.py:31-45, llama3fhe/backend.py:457-471). */
int b2f_generate_primes(int log_n, int bits, int count, int mode,
                        const uint64_t *exclude, int n_exclude, uint64_t *out);

/* Context over Q = q[0..L) and special primes P = p[0..K), dnum digits.
 * Replaces the native context of fhe.generate_client_context
 * (llama3fhe/application/session.py:31-45).  log_n must be 16. */
int b2f_context_create(int log_n, const uint64_t *q, int L, const uint64_t *p,
                       int K, int dnum, int device, b2f_context **out);
int b2f_context_destroy(b2f_context *ctx);
/* log_n, L, K, dnum, alpha (limbs per digit), digits (top level) */
int b2f_context_info(const b2f_context *ctx, int *info6);

/* Arithmetic of the NTT butterflies and the key-switch inner product: mode 0 =
 * automatic (binary64 when every prime of the context is below 2^50, else
 * 64-bit integer; the default), 1 = 64-bit integer (Shoup products, 128-bit
 * accumulation), 2 = binary64 (exact products of residues below 2^52;
 * B2F_ERR_UNSUPPORTED when a prime is 2^50 or more).  Both give the same
 * fully reduced residues.  b2f_context_arith returns 1 or 2, the arithmetic
 * in use. */
int b2f_context_set_arith(b2f_context *ctx, int mode);
int b2f_context_arith(const b2f_context *ctx);

/* ---- number-theoretic transform (inside every op; no direct Python site) ----
 * data: num_polys polynomials of q_limbs + p_limbs limbs, 32-byte aligned
 * (B2F_ERR_ARG otherwise). */
int b2f_ntt(b2f_context *ctx, uint64_t *data, int num_polys, int q_limbs,
            int p_limbs, int inverse, void *stream);

/* ---- automorphism X -> X^g in evaluation form: out[k] = in[perm_g(k)] ----
 * Part of fhe.homo_rotate (llama3fhe/operators/linear/operator.py:333-337). */
int b2f_automorphism(b2f_context *ctx, const uint64_t *in, uint64_t *out,
                     int num_polys, int limbs, uint64_t galois, void *stream);
/* Galois element of a slot rotation r (5^r mod 2N); r == 2N-1 is complex
 * conjugation (index context.M - 1, llama3fhe/operators/linear/complex.py:47-51). */
uint64_t b2f_galois_element(int log_n, int64_t rotation);

/* ---- hybrid key switching ----
 * Key layout: [digits][2][L+K][N], NTT form, generated for the top level and
 * used truncated at any level l (limbs 0..l-1 and L..L+K-1).  At l limbs only
 * digits j < ceil(l / alpha) are read, so a key kept for levels <= l may be
 * stored as its first ceil(l / alpha) digits (fhe.Context.truncate_rotation_keys). */
/* fhe.homo_rotate(ct, r, ctx) (34 call sites, e.g.
 * llama3fhe/operators/linear/operator.py:333-337, qkv_kernel.py:829-834):
 * out = (pi_g(c0 + d0), pi_g(d1)), (d0, d1) = KeySwitch(c1).  num_cts
 * ciphertexts at l limbs share one key. */
size_t b2f_rotate_workspace(const b2f_context *ctx, int num_cts, int l);
int b2f_rotate(b2f_context *ctx, const uint64_t *ct_in, uint64_t *ct_out,
               int num_cts, int l, uint64_t galois, const uint64_t *key,
               void *ws, size_t ws_bytes, void *stream);

/* Relinearisation of degree-2 ciphertexts (d0, d1, d2) -> (d0 + ks0(d2),
 * d1 + ks1(d2)): fhe.homo_relinearize / the relin inside fhe.homo_mul_relin
 * (llama3fhe/operators/primitives.py:25, attention/kernel_helpers.py:155). */
size_t b2f_relinearize_workspace(const b2f_context *ctx, int num_cts, int l);
int b2f_relinearize(b2f_context *ctx, const uint64_t *ct3_in, uint64_t *ct_out,
                    int num_cts, int l, const uint64_t *relin_key, void *ws,
                    size_t ws_bytes, void *stream);

/* Relinearisation and the rescale after it in one pass: the rescale of
 * homo_mul_relin_rescale_postop (llama3fhe/operators/nonlinear/polynomial.py:
 * 108-159) merged into the ModDown as one rounding division by P q_{l-1}.
 * ct3_in [num_cts][3][l][N] -> ct_out [num_cts][2][l-1][N] (l >= 2): each
 * coefficient is round(Y / (P q_{l-1})) for Y = P (d0, d1) + KeySwitch
 * accumulator, the same ciphertext as b2f_relinearize then b2f_rescale except
 * where a rounding tie moves (probability about K / q per coefficient). */
size_t b2f_relinearize_rescale_workspace(const b2f_context *ctx, int num_cts,
                                         int l);
int b2f_relinearize_rescale(b2f_context *ctx, const uint64_t *ct3_in,
                            uint64_t *ct_out, int num_cts, int l,
                            const uint64_t *relin_key, void *ws,
                            size_t ws_bytes, void *stream);
/* b2f_relinearize_rescale with the post-operation of
 * fhe.homo_mul_relin_rescale_postop (llama3fhe/operators/nonlinear/
 * polynomial.py:108-159: the Chebyshev basis step T_{a+b} = 2 T_a T_b -
 * T_{a-b}) folded into the same final transform's epilogue:
 *   out = r * (apply_double ? 2 : 1) - sub + scalar
 * with r the relinearised, rescaled product (l-1 limbs).  sub (optional):
 * num_cts ciphertexts of sub_limbs >= l-1 limbs, of which the first l-1 are
 * read (no alignment copy); scalar_residues (optional): l-1 residues in
 * HOST memory, passed to the kernel by value (no copy, no synchronisation),
 * added to poly 0.  Same launches as without the post-op. */
int b2f_relinearize_rescale_postop(b2f_context *ctx, const uint64_t *ct3_in,
                                   uint64_t *ct_out, int num_cts, int l,
                                   const uint64_t *relin_key, int apply_double,
                                   const uint64_t *sub, int sub_limbs,
                                   const uint64_t *scalar_residues, void *ws,
                                   size_t ws_bytes, void *stream);

/* Hoisting: ModUp of c1 once into the extended digits
 * ext[digit][l+K][N] (NTT form) ...
 * fhe.prepare_hoisted_baby_rotations (llama3fhe/operators/linear/operator.py:105-111) */
size_t b2f_modup_workspace(const b2f_context *ctx, int l);
int b2f_modup(b2f_context *ctx, const uint64_t *ct, int l, uint64_t *ext,
              void *ws, size_t ws_bytes, void *stream);
/* ... then the inner product + ModDown + automorphism of every rotation:
 * out[r] = rotation galois[r] of ct using keys[r] (an array of `count` device
 * key pointers, host array); galois 1 copies ct and needs no key (ext may be
 * null when every item is galois 1).  Rotations run in groups of up to 64
 * per launch sequence.  fhe.prepare_hoisted_baby_rotations / fast_rotate
 * (llama3fhe/operators/attention/input.py:792-797, 1143-1148). */
size_t b2f_rotate_hoisted_workspace(const b2f_context *ctx, int count, int l);
int b2f_rotate_hoisted(b2f_context *ctx, const uint64_t *ct, int l,
                       const uint64_t *ext, int count, const uint64_t *galois,
                       const uint64_t *const *keys, uint64_t *out, void *ws,
                       size_t ws_bytes, void *stream);

/* The same for a batch of num_cts ciphertexts (ct [num_cts][2][l][N]): the
 * ModUp digits are ext [num_cts][beta][l+K][N] and the rotations out
 * [num_cts][count][2][l][N]; all ciphertexts x keyed rotations run in launch
 * groups of up to 64, so a batch fills the GPU with one ModUp, one inner
 * product and one ModDown per group.  Serves prepare_hoisted_baby_rotations /
 * hoisted_mac_sum on a ciphertext batch (fhe.pack_cipher_batch) and the
 * bootstrapping transforms of several ciphertexts. */
size_t b2f_modup_batch_workspace(const b2f_context *ctx, int num_cts, int l);
int b2f_modup_batch(b2f_context *ctx, const uint64_t *ct, int num_cts, int l,
                    uint64_t *ext, void *ws, size_t ws_bytes, void *stream);
size_t b2f_rotate_hoisted_batch_workspace(const b2f_context *ctx, int num_cts,
                                          int count, int l);
int b2f_rotate_hoisted_batch(b2f_context *ctx, const uint64_t *ct, int num_cts,
                             int l, const uint64_t *ext, int count,
                             const uint64_t *galois, const uint64_t *const *keys,
                             uint64_t *out, void *ws, size_t ws_bytes,
                             void *stream);

/* Hoisted rotations left in the extended basis (double hoisting): out[r]
 * (2 polys x (l+K) limbs, Q limbs then P limbs) = (pi_g(P c0 + acc0),
 * pi_g(acc1)), P times the rotation before ModDown; galois 1 gives (P c0,
 * P c1) and needs no key.  fhe.fast_rotate(ct, offsets, ctx, output_ext=True)
 * (llama3fhe/operators/attention/input.py:792-797, 1143-1148). */
size_t b2f_rotate_hoisted_ext_workspace(const b2f_context *ctx, int count, int l);
int b2f_rotate_hoisted_ext(b2f_context *ctx, const uint64_t *ct, int l,
                           const uint64_t *ext, int count, const uint64_t *galois,
                           const uint64_t *const *keys, uint64_t *out, void *ws,
                           size_t ws_bytes, void *stream);
/* ModDown of num_cts extended ciphertexts (2 x (l+K) limbs) to l limbs:
 * fhe.moddown_from_ext (llama3fhe/operators/attention/input.py:821-826). */
size_t b2f_moddown_ext_workspace(const b2f_context *ctx, int num_cts, int l);
int b2f_moddown_ext(b2f_context *ctx, const uint64_t *in, int num_cts, int l,
                    uint64_t *out, void *ws, size_t ws_bytes, void *stream);

/* ---- level management ----
 * fhe.rescale (llama3fhe/operators/linear/operator.py:386-388): divide by the
 * last prime with a centred lift; in (num_polys x l limbs) -> out
 * (num_polys x (l-1) limbs). */
size_t b2f_rescale_workspace(const b2f_context *ctx, int num_polys, int l);
int b2f_rescale(b2f_context *ctx, const uint64_t *in, uint64_t *out,
                int num_polys, int l, void *ws, size_t ws_bytes, void *stream);
/* Same result as b2f_rescale, bit for bit, with no device allocation: for
 * callers that cannot allocate device memory (their HBM is owned by another
 * allocator, or the step runs under a fixed memory budget).  No counterpart
 * in the reference.  Scratch is a fixed 16 MiB array in device memory that
 * every GPU loading this library holds until exit: it keeps the last limb of
 * each poly, so num_polys must be <= 32 (16 ciphertexts, at any level);
 * larger requests fail with B2F_ERR_ARG.  The context's device must be the
 * current device (else B2F_ERR_ARG).  The first call on a device looks up
 * that device's array address; make it before any stream capture.  All calls
 * share the array: calls that overlap on the GPU (other streams, other
 * threads) race. */
int b2f_rescale_noalloc(b2f_context *ctx, const uint64_t *in, uint64_t *out,
                        int num_polys, int l, void *stream);
/* ModRaise of bootstrapping: num_polys polys at one limb (q_0, NTT form)
 * -> l_out limbs: the coefficients' centred lift modulo every prime, NTT
 * form (bs.bootstrap, mode "modraise_first": llama3fhe/model.py:45,
 * llama3fhe/operators/nonlinear/bootstrap.py:370). */
int b2f_modraise(b2f_context *ctx, const uint64_t *in, int num_polys, int l_out,
                 uint64_t *out, void *stream);
/* fhe.align_to to fewer limbs (llama3fhe/operators/primitives.py:100-155):
 * keep limbs 0..l_out-1 of each poly. */
int b2f_drop_limbs(b2f_context *ctx, const uint64_t *in, uint64_t *out,
                   int num_polys, int l_in, int l_out, void *stream);

/* ---- elementwise (limb-wise, NTT form) ----
 * op: 0 add, 1 sub, 2 mul.  fhe.homo_add / homo_sub (28 / 9 sites),
 * fhe.homo_mul_pt (llama3fhe/operators/primitives.py:43), homo_add_pt.
 * a, b and out hold num_polys polys of l limbs; b_polys is 1 (plaintext
 * broadcast over the polys) or num_polys. */
int b2f_elementwise(b2f_context *ctx, int op, const uint64_t *a,
                    const uint64_t *b, uint64_t *out, int num_polys, int l,
                    int b_polys, void *stream);
/* The same limb-wise op (b with num_polys polys) over the extended basis
 * Q_{q_limbs} u P: polys of q_limbs + p_limbs limbs, limb t prime t below
 * q_limbs and prime L + t - q_limbs after it.  Sums of extended ciphertexts
 * before one ModDown (hoisted_mac_sum, strategy="ext_double_hoist",
 * llama3fhe/operators/linear/config.py:295-300). */
int b2f_elementwise_ext(b2f_context *ctx, int op, const uint64_t *a,
                        const uint64_t *b, uint64_t *out, int num_polys, int q_limbs,
                        int p_limbs, void *stream);
/* out = a * X^(N/2) (multiply every slot by i, or -i when negative):
 * fhe.homo_mul_i (llama3fhe/operators/linear/complex.py:22). */
int b2f_mul_i(b2f_context *ctx, const uint64_t *a, uint64_t *out,
              int num_polys, int l, int negative, void *stream);
/* Tensor product of num_cts ciphertext pairs at l limbs (NTT form): out[c]
 * (3 polys) = (a0 b0, a0 b1 + a1 b0, a1 b1).  fhe.homo_mul_no_relin
 * (llama3fhe/operators/attention/qk.py:399, primitives.py:21-31). */
int b2f_tensor(b2f_context *ctx, const uint64_t *a, const uint64_t *b,
               uint64_t *out, int num_cts, int l, void *stream);
/* out = sum_k weights[k][i] * terms[k] (mod q_i) over num_cts ciphertexts of
 * `polys` polynomials at l limbs; term k (device pointer) has term_limbs[k]
 * >= l limbs per polynomial (its limbs beyond l are skipped, so no modulus
 * drop is needed first); weights is a host array [num_terms][l] of
 * residues.  At most 8 terms of 40 limbs (B2F_ERR_UNSUPPORTED beyond).  No
 * reference counterpart: one pass for the scalar-weighted sums of the
 * bootstrapping polynomial (homo_mul_scalar + homo_add per term,
 * llama3fhe/operators/nonlinear/polynomial.py:41-88). */
int b2f_linear_combination(b2f_context *ctx, int num_terms,
                           const uint64_t *const *terms, const int *term_limbs,
                           const uint64_t *weights, int num_cts, int polys, int l,
                           uint64_t *out, void *stream);
/* out = a * c (+ add) with per-limb integer constants c[l], add[l]
 * (residues, NULL = none); add goes to poly add_poly, to every poly (-1) or
 * to c0 of every ciphertext of a batch of 2-poly ciphertexts (-2):
 * fhe.homo_mul_scalar / homo_add_scalar on fhe.encode_scalar constants
 * (llama3fhe/operators/nonlinear/bootstrap.py:331-349). */
int b2f_scalar_op(b2f_context *ctx, const uint64_t *a, uint64_t *out,
                  int num_polys, int l, const uint64_t *mul_residues,
                  const uint64_t *add_residues, int add_poly, void *stream);

/* ---- baby-step / giant-step plaintext x ciphertext MAC ----
 * fhe.hoisted_mac_sum (llama3fhe/operators/linear/operator.py:320-330,
 * llama3fhe/operators/transform.py:108-116): for each giant g < giant_count,
 * inner_g = sum_b pt[g*B + b] * babies[b]; out = Horner over the giants with
 * the rotation by giant_offset (key giant_key):
 *   acc = inner_{G-1}; acc = rot(acc) + inner_g for g = G-2..0.
 * babies: B ciphertexts at l limbs; pts: G*B plaintexts at l limbs.
 * The chain runs as b2f_set_giant_chain selects (by default in Q_l u P,
 * one ModDown per chain). */
size_t b2f_bsgs_mac_workspace(const b2f_context *ctx, int l);
int b2f_bsgs_mac(b2f_context *ctx, const uint64_t *babies, int baby_count,
                 const uint64_t *pts, int giant_count, int l,
                 uint64_t giant_galois, const uint64_t *giant_key,
                 uint64_t *out, void *ws, size_t ws_bytes, void *stream);
/* b2f_bsgs_mac for num_cts ciphertexts sharing the plaintext rows: babies
 * [num_cts][baby_count][2][l][N] -> out [num_cts][2][l][N]; every plaintext
 * row streams from HBM once per batch and each giant rotation of the Horner
 * chain is one batched HRotate. */
size_t b2f_bsgs_mac_batch_workspace(const b2f_context *ctx, int num_cts,
                                    int giant_count, int l);
int b2f_bsgs_mac_batch(b2f_context *ctx, const uint64_t *babies, int num_cts,
                       int baby_count, const uint64_t *pts, int giant_count,
                       int l, uint64_t giant_galois, const uint64_t *giant_key,
                       uint64_t *out, void *ws, size_t ws_bytes, void *stream);
/* out[g] = sum_{i in group g} ct[i] * pt[i] over q_limbs Q limbs and p_limbs
 * P limbs (extended ciphertexts and plaintexts), count pairs split into
 * `groups` consecutive groups; plaintext rows are pt_limb_stride limbs apart.
 * fhe.grouped_pairwise_mac(batch, plaintexts, groups, ctx)
 * (llama3fhe/operators/attention/input.py:814-819, 1274-1279). */
int b2f_pairwise_mac(b2f_context *ctx, const uint64_t *cts, const uint64_t *pts,
                     int count, int groups, int q_limbs, int p_limbs,
                     int pt_limb_stride, uint64_t *out, void *stream);
/* Only the MAC: out[g] = sum_b pt[g*B+b] * babies[b] for g < giant_count
 * (num_cts independent baby sets, each with its own output block). */
int b2f_mac(b2f_context *ctx, const uint64_t *babies, int baby_count,
            const uint64_t *pts, int giant_count, int l, uint64_t *out,
            int num_cts, void *stream);
/* The same over the extended basis Q_{q_limbs} u P: babies [num_cts][B][2]
 * [q_limbs + p_limbs][N] and plaintext rows [G*B][q_limbs + p_limbs][N]
 * (limb t is prime t below q_limbs, prime L + t - q_limbs after), out
 * [num_cts][G][2][q_limbs + p_limbs][N].  The multiply-accumulate of
 * fhe.hoisted_mac_sum(..., strategy="ext_normal" | "ext_double_hoist")
 * (llama3fhe/operators/transform.py:108-116, operators/linear/config.py:9,
 * 286-305): babies left in Q u P by the key switch, one ModDown per giant. */
int b2f_mac_ext(b2f_context *ctx, const uint64_t *babies, int baby_count,
                const uint64_t *pts, int giant_count, int q_limbs, int p_limbs,
                uint64_t *out, int num_cts, void *stream);
/* Which units run the multiply-accumulate of b2f_mac, b2f_mac_ext and
 * b2f_bsgs_mac(_batch): path 0 (the default) the u8 tensor cores on the byte
 * split of the residues for launches of 4-8 giants over 16-1024 babies and
 * two or more ciphertexts wherever the sum is exact (baby_count * q^2 <
 * 2^128 for every prime of the call), the CUDA cores otherwise; path 1 the
 * CUDA cores always.  Both give the same residues.  Inputs are canonical
 * residues (below their prime). */
int b2f_set_mac_path(b2f_context *ctx, int path);
/* 1 when a MAC of num_cts ciphertexts x baby_count babies x giant_count
 * giants over Q_{q_limbs} u P_{p_limbs} runs (its first launch of up to 8
 * giants) on the tensor cores under the context's current path, else 0. */
int b2f_mac_uses_tensor_cores(const b2f_context *ctx, int baby_count, int giant_count,
                              int q_limbs, int p_limbs, int num_cts);
/* Stages the tensor-core MAC gave up waiting for (its bounded waits on the
 * TMA loads timed out; the block ended and its outputs are not written) since
 * the library loaded, on the current device; 0 on a healthy run, -1 when the
 * counter cannot be read. */
int b2f_mac_wait_errors(void);
/* Which tensor-core kernels run the fast base conversions of the key switch
 * (ModUp step 2, ModDown's P-to-Q step): tcgen05.mma kind::i8 with the
 * accumulators in tensor memory (up to 64 targets, else mma.sync) or the
 * warp-level mma.sync kernel.  Path 0 (the default): the faster of the two,
 * measured on B200 (the ModDown conversion of 16 or more ciphertexts on
 * tcgen05, everything else on mma.sync); path 1: mma.sync always; path 2:
 * tcgen05 for both conversions.  All give the same residues. */
int b2f_set_conv_path(b2f_context *ctx, int path);
/* Tiles the tcgen05 conversion gave up waiting for (its bounded wait on the
 * MMAs' completion timed out; the block's outputs are not written) since the
 * library loaded, on the current device; 0 on a healthy run, -1 when the
 * counter cannot be read. */
int b2f_conv_wait_errors(void);
/* How b2f_bsgs_mac(_batch) runs its Horner chain over the giants (the one
 * giant key, as llama3fhe/operators/linear/config.py:292-305 plans it for
 * the `normal` strategy).  Mode 0 (the default): the chain stays in Q_l u P;
 * each rotation's key switch leaves P times its result there, the next
 * rotation ModDowns only the second poly (the one it key-switches), and one
 * ModDown of both polys ends the chain.  Mode 1: each giant rotation is a
 * full HRotate (ModDown of both polys) followed by the addition.  The
 * results decrypt to the same values; mode 0 rounds once per step where
 * mode 1 rounds twice, so residues differ. */
int b2f_set_giant_chain(b2f_context *ctx, int mode);
/* The Horner chain over the giants of fhe.hoisted_mac_sum by itself, kept in
 * Q_l u P as b2f_set_giant_chain's mode 0 describes: sums [num_cts]
 * [giant_count][2][limbs][N] as b2f_mac leaves them (limbs = l, extended =
 * 0) or as b2f_mac_ext does (limbs = l + K, extended = 1: P times the giant
 * sums, which then need no ModDown of their own) -> out [num_cts][2][l][N]
 * = acc, acc = sum_{G-1}; acc = rot(acc) + sum_g for g = G-2..0 with the
 * rotation by the giant offset (giant_galois, giant_key).  The `ext_normal`
 * strategy's chain (llama3fhe/operators/transform.py:108-116,
 * operators/linear/config.py:292-305): one ModDown per chain instead of one
 * per giant sum and one per rotation.  giant_count 1: the ModDown of the
 * extended sum, or a copy. */
size_t b2f_giant_chain_workspace(const b2f_context *ctx, int num_cts, int l);
int b2f_giant_chain(b2f_context *ctx, const uint64_t *sums, int extended, int num_cts,
                    int giant_count, int l, uint64_t giant_galois, const uint64_t *giant_key,
                    uint64_t *out, void *ws, size_t ws_bytes, void *stream);

/* ---- calibration (no reference counterpart) ----
 * Rate of the NTT's lazy Shoup butterfly from registers alone (every SM
 * full, `iters` rounds of 8 butterflies per thread), per second: the
 * integer-multiply roofline the NTT kernels are measured against, since
 * their 64-bit products on CUDA cores bound them before HBM does. */
int b2f_butterfly_peak(b2f_context *ctx, int iters, double *per_second,
                       void *stream);
/* Rate of mac_kernel's inner step from registers alone (2 babies x 8 giants
 * x 2 polys of 128-bit multiply-adds per step, each accumulator reduced every
 * 32 babies, every SM full), in multiply-adds per second: the integer-multiply
 * roofline the BSGS multiply-accumulate is measured against.  No reference
 * counterpart (calibration). */
int b2f_mac_peak(b2f_context *ctx, int iters, double *per_second, void *stream);
/* Byte multiply-adds per second of mma.sync m16n8k32 u8 from registers alone
 * (mac_mma_kernel's tensor-core step: 32 independent tiles per warp, every SM
 * full): the compute roofline of the tensor-core MAC. */
int b2f_mma_u8_peak(b2f_context *ctx, int iters, double *per_second, void *stream);

/* ---- encoding ----
 * Slot vectors (complex128 interleaved re/im, device) -> plaintexts at
 * q_limbs (+ p_limbs) in NTT form: special inverse FFT, times scale, round
 * to nearest, reduce per limb, NTT.  fhe.ConstantBundle.plaintext
 * (llama3fhe/backend.py:231-297, llama3fhe/operators/linear/weight.py:344-357),
 * client.encrypt's encoding (llama3fhe/application/session.py:71-77). */
int b2f_encode(b2f_context *ctx, const double *values, int num_rows, int slots,
               double scale, int q_limbs, int p_limbs, uint64_t *out, void *ws,
               size_t ws_bytes, void *stream);
size_t b2f_encode_workspace(const b2f_context *ctx, int num_rows, int slots);
/* Plaintext (l limbs, NTT) -> complex slots, decoded from the first
 * min(l, 2) limbs (client.decrypt, llama3fhe/backend.py:305-313). */
int b2f_decode(b2f_context *ctx, const uint64_t *pt, int l, int slots,
               double scale, double *values, void *ws, size_t ws_bytes,
               void *stream);
size_t b2f_decode_workspace(const b2f_context *ctx, int slots);

/* Diagonal packer of a feature-major BSGS chunk (replaces the reference's
 * Triton kernels, llama3fhe/operators/linear/gpu_packer.py:144-184 and
 * 317-424, formula weight.py:18-47):
 *   row(g,b)[s] = W[(f(s) - g*B) mod D, (f(s) + b) mod D], f(s) = s / lanes,
 * g = giant_base + row / B.  weight: D x D, dtype 0 float64, 1 float32,
 * 2 complex128 (interleaved).  out: rows x slots complex128 interleaved. */
int b2f_pack_diagonals(b2f_context *ctx, const void *weight, int dtype,
                       int dimension, int token_lanes, int baby_steps,
                       int giant_base, int giant_count, int slots,
                       double *out, void *stream);
/* Structured variant: W_phys[o,i] = column_scale[i] * (real_scale[o] *
 * src[real_source[o]][real_row[o], column[i]] + 1j * imag_scale[o] *
 * src[imag_source[o]][imag_row[o], column[i]]), -1 = zero
 * (llama3fhe/operators/linear/structured_weight.py:1-20). maps: int64 x D,
 * scales: float64 x D; sources: up to 3 device matrices with (row, col)
 * strides in elements, dtype 0 float64 / 1 float32. */
int b2f_pack_structured(b2f_context *ctx, const void *const *sources,
                        const int64_t *strides, int source_count, int dtype,
                        const int64_t *real_source, const int64_t *real_row,
                        const double *real_scale, const int64_t *imag_source,
                        const int64_t *imag_row, const double *imag_scale,
                        const int64_t *column, const double *column_scale,
                        int dimension, int token_lanes, int baby_steps,
                        int giant_base, int giant_count, int slots, double *out,
                        void *stream);

/* ---- keys and (de)cryption (client side of fhe.generate_client_context,
 * client.encrypt / client.decrypt, session.py:31-77, backend.py:305-313) ----
 * Randomness: ChaCha20 keyed by `seed`.  s_* are secrets in NTT form over all
 * L+K primes.  Not a hot path. */
int b2f_secret_to_ntt(b2f_context *ctx, const int8_t *s_coeff /* host, N */,
                      uint64_t *s_ntt, void *stream);
int b2f_keygen_switch(b2f_context *ctx, const uint64_t *s_from_ntt,
                      const uint64_t *s_to_ntt, uint64_t seed, uint32_t tag,
                      uint64_t *key, void *stream);
int b2f_keygen_rotation(b2f_context *ctx, const uint64_t *s_ntt,
                        uint64_t galois, uint64_t seed, uint64_t *key,
                        void *stream);
int b2f_keygen_relin(b2f_context *ctx, const uint64_t *s_ntt, uint64_t seed,
                     uint64_t *key, void *stream);
int b2f_encrypt(b2f_context *ctx, const uint64_t *m_ntt, int l,
                const uint64_t *s_ntt, uint64_t seed, uint64_t nonce,
                uint64_t *ct, void *stream);
int b2f_decrypt(b2f_context *ctx, const uint64_t *ct, int l,
                const uint64_t *s_ntt, uint64_t *m_ntt, void *stream);
/* sparse ternary (hamming > 0) or uniform ternary (hamming == 0) secret,
 * host output, same ChaCha20 stream definition as the keys. */
int b2f_sample_secret(int log_n, uint64_t seed, int hamming, int8_t *s_out);

#ifdef __cplusplus
}
#endif
#endif /* B200FHE_H */
