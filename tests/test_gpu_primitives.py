"""GPU parity of the CKKS primitives against the CPU oracle, bit-exact in RNS
residues (rotation, rescale, elementwise ops, NTT, keys).  Inputs are seeded uniform
residues at N = 2^16 with 50-bit NTT primes (q = 1 mod 2^17), the primitive
microbench parameters, plus one small parameter set whose special primes
cover a digit so that decrypted values are meaningful."""

from __future__ import annotations

import contextlib

import numpy as np
import pytest

from _ckks import N, pair, rand_residues, to_dev, to_host

pytestmark = pytest.mark.gpu


def test_generated_primes_match_oracle(oracle_mod):
    from easyfhe import core

    for log_n, bits, count, mode in ((16, 50, 12, 0), (16, 59, 9, 1), (16, 60, 5, 0)):
        assert core.gen_primes(log_n, bits, count, mode) == oracle_mod.gen_primes(
            log_n, bits, count, mode)


@contextlib.contextmanager
def use_arith(ctx, mode):
    ctx.set_arith(mode)
    try:
        yield
    finally:
        ctx.set_arith("auto")


def test_arith_selection():
    """50-bit primes take the binary64 butterflies by default; a context
    with a prime of 2^50 or more keeps the integer ones and refuses f64."""

    from easyfhe import core

    ctx, _ = pair(8, 2, 4)
    assert ctx.arith == "f64"
    with use_arith(ctx, "int64"):
        assert ctx.arith == "int64"
    assert ctx.arith == "f64"
    wide = core.NativeContext(core.Params.uniform(4, 1, 2, bits=59), "cuda:0")
    assert wide.arith == "int64"
    with pytest.raises(NotImplementedError):
        wide.set_arith("f64")
    with pytest.raises(ValueError):
        ctx.set_arith("f32")


@pytest.mark.parametrize("arith", ["f64", "int64"])
def test_ntt_extreme_residues(arith):
    """All-(q-1), all-zero and alternating limbs: the largest products the
    butterflies see."""

    ctx, orc = pair(8, 2, 4)
    q = np.array(ctx.primes[:8], dtype=np.uint64)[:, None]
    ones = np.ones((8, N), dtype=np.uint64)
    x = np.stack([ones * (q - 1), ones * 0, np.where(np.arange(N) % 2 == 0, q - 1, 0) * ones,
                  ones * (q - 1) // 2])
    with use_arith(ctx, arith):
        d = to_dev(x)
        ctx.ntt(d, 8, 0, inverse=False)
        assert np.array_equal(to_host(d), orc.ntt(x, 8, 0, inverse=False).reshape(x.shape))
        d = to_dev(x)
        ctx.ntt(d, 8, 0, inverse=True)
        assert np.array_equal(to_host(d), orc.ntt(x, 8, 0, inverse=True).reshape(x.shape))


@pytest.mark.parametrize("arith", ["f64", "int64"])
@pytest.mark.parametrize("L", [8, 16, 24, 32])
def test_ntt_forward_inverse_bit_exact(L, arith):
    ctx, orc = pair(L, 2, 4)
    with use_arith(ctx, arith):
        _ntt_round_trip(ctx, orc, L)


def _ntt_round_trip(ctx, orc, L):
    rng = np.random.default_rng(1000 + L)
    x = rand_residues(rng, ctx.primes[:L], 3)
    d = to_dev(x)
    ctx.ntt(d, L, 0, inverse=False)
    got = to_host(d)
    want = orc.ntt(x, L, 0, inverse=False).reshape(x.shape)
    assert np.array_equal(got, want)
    ctx.ntt(d, L, 0, inverse=True)
    assert np.array_equal(to_host(d), x)
    # inverse on fresh data, against the oracle
    y = rand_residues(rng, ctx.primes[:L], 2)
    dy = to_dev(y)
    ctx.ntt(dy, L, 0, inverse=True)
    assert np.array_equal(to_host(dy), orc.ntt(y, L, 0, inverse=True).reshape(y.shape))


def test_ntt_extended_limbs():
    ctx, orc = pair(8, 2, 4)
    rng = np.random.default_rng(7)
    x = rand_residues(rng, ctx.primes[:5] + ctx.primes[8:10], 2)
    d = to_dev(x)
    ctx.ntt(d, 5, 2)
    assert np.array_equal(to_host(d), orc.ntt(x, 5, 2).reshape(x.shape))


def test_secret_and_keys_match_oracle(oracle_mod):
    from easyfhe import core

    ctx, orc = pair(8, 2, 3)
    s = core.sample_secret(1234, 192)
    assert np.array_equal(s.astype(np.int64), oracle_mod.sample_secret(16, 1234, 192))
    assert int(np.count_nonzero(s)) == 192
    su = core.sample_secret(99, 0)
    assert np.array_equal(su.astype(np.int64), oracle_mod.sample_secret(16, 99, 0))
    s_ntt = ctx.secret_to_ntt(s)
    want = orc.secret_to_ntt(s.astype(np.int64))
    assert np.array_equal(to_host(s_ntt), want)
    g = core.galois_element(5)
    key = ctx.keygen_rotation(s_ntt, g, seed=77)
    assert np.array_equal(to_host(key), orc.keygen_rotation(want, g, 77))
    rk = ctx.keygen_relin(s_ntt, seed=78)
    assert np.array_equal(to_host(rk), orc.keygen_relin(want, 78))


@pytest.mark.parametrize("rotation,arith", [(1, "f64"), (3, "f64"), (1024, "f64"),
                                             (131071, "f64"), (3, "int64")])
def test_rotate_bit_exact(rotation, arith):
    from easyfhe import core

    L, l = 8, 7
    ctx, orc = pair(L, 2, 3)
    s = core.sample_secret(5, 192)
    s_ntt = ctx.secret_to_ntt(s)
    g = core.galois_element(rotation)
    key = ctx.keygen_rotation(s_ntt, g, seed=11)
    rng = np.random.default_rng(rotation)
    cts = rand_residues(rng, ctx.primes[:l], 6).reshape(3, 2, l, N)
    with use_arith(ctx, arith):
        out = to_host(ctx.rotate(to_dev(cts), l, g, key))
    hkey = to_host(key)
    for c in range(3):
        assert np.array_equal(out[c], orc.rotate(cts[c], l, g, hkey)), f"ct {c}"


@pytest.mark.parametrize("arith", ["f64", "int64"])
def test_hoisted_rotations_bit_exact(arith):
    from easyfhe import core

    L, l = 8, 8
    ctx, orc = pair(L, 2, 3)
    s_ntt = ctx.secret_to_ntt(core.sample_secret(6, 192))
    gs = [core.galois_element(r) for r in (1, 2, 8)]
    keys = [ctx.keygen_rotation(s_ntt, g, seed=20 + i) for i, g in enumerate(gs)]
    rng = np.random.default_rng(3)
    ct = rand_residues(rng, ctx.primes[:l], 2)
    dct = to_dev(ct)
    with use_arith(ctx, arith):
        ext = ctx.modup(dct, l)
        got = to_host(ctx.rotate_hoisted(dct, l, ext, gs, keys))
        plain = to_host(ctx.rotate(dct, l, gs[1], keys[1]))
    want = orc.rotate_hoisted(ct, l, gs, [to_host(k) for k in keys])
    assert np.array_equal(got, want)
    # one hoisted rotation equals the plain HRotate
    assert np.array_equal(got[1], plain)


@pytest.mark.parametrize("L,K,dnum", [(9, 3, 3), (12, 4, 3), (12, 6, 4)])
def test_rotate_special_prime_counts(L, K, dnum):
    """HRotate with K = 3, 4 (the ModDown conversion computed inside its NTT,
    binary64) and K = 6 (the tensor-core conversion) against the oracle."""

    from easyfhe import core

    ctx, orc = pair(L, K, dnum)
    l = L - 1
    s_ntt = ctx.secret_to_ntt(core.sample_secret(K, 192))
    g = core.galois_element(7)
    key = ctx.keygen_rotation(s_ntt, g, seed=30 + K)
    rng = np.random.default_rng(K)
    cts = rand_residues(rng, ctx.primes[:l], 4).reshape(2, 2, l, N)
    hkey = to_host(key)
    for arith in ("f64", "int64"):
        with use_arith(ctx, arith):
            out = to_host(ctx.rotate(to_dev(cts), l, g, key))
        for c in range(2):
            assert np.array_equal(out[c], orc.rotate(cts[c], l, g, hkey)), (arith, c)


@pytest.mark.parametrize("K,batch", [(1, 16), (2, 64)])
def test_rotate_dnum4_small_special_batches(K, batch):
    """HRotate at dnum 4 with 1 or 2 special primes on batches of 16 and 64
    ciphertexts sharing one key (the primitive microbench's grid): the first
    and last ciphertext against the oracle, every ciphertext of the batch
    against its own single-ciphertext rotation, under both arithmetics."""

    from easyfhe import core

    L, l = 16, 16
    ctx, orc = pair(L, K, 4)
    s_ntt = ctx.secret_to_ntt(core.sample_secret(40 + K, 192))
    g = core.galois_element(5)
    key = ctx.keygen_rotation(s_ntt, g, seed=90 + K)
    rng = np.random.default_rng(batch)
    cts = rand_residues(rng, ctx.primes[:l], 2 * batch).reshape(batch, 2, l, N)
    dcts = to_dev(cts)
    hkey = to_host(key)
    for arith in ("f64", "int64"):
        with use_arith(ctx, arith):
            out = to_host(ctx.rotate(dcts, l, g, key))
            for c in range(0, batch, 7):
                one = to_host(ctx.rotate(dcts[c:c + 1].contiguous(), l, g, key))
                assert np.array_equal(out[c], one[0]), (arith, c)
        for c in (0, batch - 1):
            assert np.array_equal(out[c], orc.rotate(cts[c], l, g, hkey)), (arith, c)


def test_hoisted_rotations_identity_items_and_groups():
    """Identity items (galois 1, no key) anywhere in the list are copies, and
    more than 64 rotations run as several launch groups."""

    from easyfhe import core

    L, l = 4, 4
    ctx, orc = pair(L, 1, 2)
    s_ntt = ctx.secret_to_ntt(core.sample_secret(12, 192))
    base = [core.galois_element(r) for r in (1, 3, 5)]
    keys3 = [ctx.keygen_rotation(s_ntt, g, seed=40 + i) for i, g in enumerate(base)]
    rng = np.random.default_rng(13)
    ct = rand_residues(rng, ctx.primes[:l], 2)
    dct = to_dev(ct)
    ext = ctx.modup(dct, l)
    gs, keys = [], []
    for r in range(70):
        if r in (0, 33, 64):
            gs.append(1)
            keys.append(None)
        else:
            gs.append(base[r % 3])
            keys.append(keys3[r % 3])
    got = to_host(ctx.rotate_hoisted(dct, l, ext, gs, keys))
    hk = [to_host(k) for k in keys3]
    want3 = orc.rotate_hoisted(ct, l, base, hk)
    for r in range(70):
        want = ct if gs[r] == 1 else want3[r % 3]
        assert np.array_equal(got[r], want), f"item {r}"


def test_tensor_product_bit_exact():
    ctx, _ = pair(8, 2, 3)
    l, cts = 3, 2
    rng = np.random.default_rng(14)
    a = rand_residues(rng, ctx.primes[:l], 2 * cts).reshape(cts, 2, l, N)
    b = rand_residues(rng, ctx.primes[:l], 2 * cts).reshape(cts, 2, l, N)
    got = to_host(ctx.tensor(to_dev(a), to_dev(b), cts, l)).reshape(cts, 3, l, N)
    q = np.array(ctx.primes[:l], dtype=object)[:, None]
    A, B = a.astype(object), b.astype(object)
    for c in range(cts):
        want = [(A[c, 0] * B[c, 0]) % q, (A[c, 0] * B[c, 1] + A[c, 1] * B[c, 0]) % q,
                (A[c, 1] * B[c, 1]) % q]
        for p in range(3):
            assert np.array_equal(got[c, p], want[p].astype(np.uint64)), (c, p)


def test_relinearize_bit_exact():
    from easyfhe import core

    L, l = 8, 6
    ctx, orc = pair(L, 2, 3)
    s_ntt = ctx.secret_to_ntt(core.sample_secret(8, 192))
    rk = ctx.keygen_relin(s_ntt, seed=5)
    rng = np.random.default_rng(4)
    ct3 = rand_residues(rng, ctx.primes[:l], 3)
    got = to_host(ctx.relinearize(to_dev(ct3), l, rk))
    d0, d1 = orc.keyswitch(ct3[2], l, to_host(rk))
    q = np.array(ctx.primes[:l], dtype=object)[:, None]
    w0 = (ct3[0].astype(object) + d0.astype(object)) % q
    w1 = (ct3[1].astype(object) + d1.astype(object)) % q
    assert np.array_equal(got[0], w0.astype(np.uint64))
    assert np.array_equal(got[1], w1.astype(np.uint64))


@pytest.mark.parametrize("L,K,dnum,l,cts,arith", [(8, 2, 3, 6, 1, "f64"), (8, 2, 3, 2, 2, "f64"),
                                                   (10, 4, 5, 10, 1, "f64"),
                                                   (12, 8, 3, 7, 2, "f64"),
                                                   (8, 2, 3, 6, 2, "int64")])
def test_relinearize_rescale_bit_exact(L, K, dnum, l, cts, arith):
    """The fused relinearise + rescale against the oracle's rounding division
    by P q_{l-1}, and against the GPU's own relinearise then rescale (equal but
    for rounding ties, probability about K / q per coefficient).  K = 2, 4, 8
    reach the three widths of the tensor-core conversion (K + 2 words)."""

    from easyfhe import core

    ctx, orc = pair(L, K, dnum)
    s_ntt = ctx.secret_to_ntt(core.sample_secret(9, 192))
    rk = ctx.keygen_relin(s_ntt, seed=6)
    rng = np.random.default_rng(100 + l + K)
    ct3 = np.stack([rand_residues(rng, ctx.primes[:l], 3) for _ in range(cts)])
    with use_arith(ctx, arith):
        got = to_host(ctx.relinearize_rescale(to_dev(ct3), l, rk))
        two = to_host(ctx.rescale(ctx.relinearize(to_dev(ct3), l, rk), 2 * cts, l))
    assert got.shape == (cts, 2, l - 1, N)
    rk_h = to_host(rk)
    for c in range(cts):
        assert np.array_equal(got[c], orc.relin_rescale(ct3[c], l, rk_h)), c
    assert np.array_equal(got.reshape(two.shape), two)


@pytest.mark.parametrize("l,polys,arith", [(2, 2, "f64"), (9, 2, "f64"), (16, 3, "f64"),
                                           (2, 2, "int64"), (16, 3, "int64")])
def test_rescale_bit_exact(l, polys, arith):
    ctx, orc = pair(16, 2, 4)
    rng = np.random.default_rng(l)
    x = rand_residues(rng, ctx.primes[:l], polys)
    with use_arith(ctx, arith):
        got = to_host(ctx.rescale(to_dev(x), polys, l))
    assert np.array_equal(got, orc.rescale(x, polys, l))


@pytest.mark.parametrize("negative", [False, True])
def test_mul_i_bit_exact(negative):
    ctx, orc = pair(8, 2, 3)
    rng = np.random.default_rng(17)
    x = rand_residues(rng, ctx.primes[:5], 2)
    got = to_host(ctx.mul_i(to_dev(x), 2, 5, negative))
    assert np.array_equal(got, orc.mul_i(x, 2, 5, negative).reshape(x.shape))


def test_elementwise_bit_exact():
    ctx, _ = pair(8, 2, 3)
    rng = np.random.default_rng(2)
    l = 6
    a = rand_residues(rng, ctx.primes[:l], 2)
    b = rand_residues(rng, ctx.primes[:l], 1)
    q = np.array(ctx.primes[:l], dtype=object)[None, :, None]
    A, B = a.astype(object), b.astype(object)
    for op, ref in ((0, (A + B) % q), (1, (A - B) % q), (2, (A * B) % q)):
        got = to_host(ctx.elementwise(op, to_dev(a), to_dev(b), 2, l, b_polys=1))
        assert np.array_equal(got, ref.astype(np.uint64)), op


def test_encode_bit_exact_and_decode():
    ctx, orc = pair(8, 2, 3)
    import torch

    rng = np.random.default_rng(21)
    z = rng.uniform(-1, 1, 32768) + 1j * rng.uniform(-1, 1, 32768)
    scale = 2.0 ** 40
    got = to_host(ctx.encode(torch.from_numpy(z).to("cuda:0"), scale, 6, 2))
    want = orc.encode(z, scale, 6, 2)
    assert np.array_equal(got, want)
    dec = ctx.decode(to_dev(want), 6, 32768, scale)
    assert np.max(np.abs(dec - z)) < 1e-9
    # sparse slots
    z2 = z[:1024]
    got2 = to_host(ctx.encode(torch.from_numpy(z2).to("cuda:0"), scale, 3, 0))
    assert np.array_equal(got2, orc.encode(z2, scale, 3, 0))


def test_encrypt_rotate_decrypt_values():
    """Functional check where noise is meaningful (alpha = K): slots rotate
    left, conjugation conjugates, rescale divides the scale."""

    import torch

    from easyfhe import core

    ctx, orc = pair(4, 2, 2, bits=50)
    s_ntt = ctx.secret_to_ntt(core.sample_secret(31, 192))
    scale = 2.0 ** 40
    rng = np.random.default_rng(8)
    z = rng.uniform(-1, 1, 32768) + 1j * rng.uniform(-1, 1, 32768)
    m = ctx.encode(torch.from_numpy(z).to("cuda:0"), scale, 4)
    ct = ctx.encrypt(m, 4, s_ntt, seed=3, nonce=1)
    # encryption matches the oracle bit for bit
    want = orc.encrypt(to_host(m), 4, to_host(s_ntt), 3, 1)
    assert np.array_equal(to_host(ct), want)
    for r in (1, 7, 131071):
        g = core.galois_element(r)
        key = ctx.keygen_rotation(s_ntt, g, seed=40 + r)
        rot = ctx.rotate(ct, 4, g, key)
        dec = ctx.decode(ctx.decrypt(rot, 4, s_ntt), 4, 32768, scale)
        ref = np.conj(z) if r == 131071 else np.roll(z, -r)
        assert np.max(np.abs(dec - ref)) < 1e-4, r


def test_linear_combination_matches_scalar_ops():
    """homo_linear_combination equals align_to + homo_mul_scalar + homo_add,
    bit for bit, for a batch whose terms sit at different levels."""

    from easyfhe import fhe

    client, ctx = fhe.generate_client_context(
        fhe.CKKSContextSpec(depth=6, log_n=16, dnum=2, dcrt_bits=45, first_mod=55,
                            rotations=(1,)), "cuda:0")
    rng = np.random.default_rng(72)
    n = ctx.max_slots
    terms, scalars = [], []
    for k, limbs in enumerate((7, 5, 6, 5)):
        cts = [client.encrypt(rng.uniform(-1, 1, n), slots=n, cur_limbs=limbs,
                              scaling_factor=ctx.scale_at(limbs)) for _ in range(3)]
        terms.append(fhe.pack_cipher_batch(cts))
        scalars.append(fhe.encode_scalar(0.37 * (k + 1) - 0.8, cur_limbs=5, scale_degree=1,
                                         scaling_factor=ctx.scale_at(5), context=ctx))
    got = fhe.homo_linear_combination(terms, scalars, ctx)
    acc = None
    for t, e in zip(terms, scalars):
        p = fhe.homo_mul_scalar(fhe.align_to(t, t.state.replace(cur_limbs=5), ctx), e, ctx)
        acc = p if acc is None else fhe.homo_add(acc, p, ctx)
    assert got.state.cur_limbs == 5 and got.batch_size == 3
    assert np.array_equal(to_host(got.data), to_host(acc.data))
