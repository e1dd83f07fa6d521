"""Pins the CPU oracle (test infrastructure) to independent known answers:
definitions evaluated with Python integers, a published ChaCha20 keystream and
functional decryption checks.  Runs on CPU."""

from __future__ import annotations

import numpy as np
import pytest


def brv(x: int, bits: int) -> int:
    return int(format(x, f"0{bits}b")[::-1], 2)


@pytest.mark.parametrize("log_n,bits", [(4, 30), (5, 50), (6, 59), (4, 60)])
def test_ntt_matches_definitions(oracle_mod, log_n, bits):
    O = oracle_mod
    n = 1 << log_n
    q = O.gen_primes(log_n, bits, 1)[0]
    assert O.is_prime(q) and q % (2 * n) == 1
    o = O.Oracle(log_n, [q], [], 1)
    rng = np.random.default_rng(bits)
    a = [int(v) for v in rng.integers(0, min(q, 2**62), n, dtype=np.uint64)]
    b = [int(v) for v in rng.integers(0, min(q, 2**62), n, dtype=np.uint64)]
    a = [v % q for v in a]
    b = [v % q for v in b]
    psi = O.find_psi(q, log_n)
    assert pow(psi, n, q) == q - 1
    assert all(pow(psi, 2 * k + 1, q) >= psi for k in range(n))  # smallest root
    A = o.ntt(np.array(a, dtype=np.uint64), 1)
    ev = [sum(a[j] * pow(psi, (2 * brv(k, log_n) + 1) * j, q) for j in range(n)) % q
          for k in range(n)]
    assert [int(v) for v in A] == ev
    B = o.ntt(np.array(b, dtype=np.uint64), 1)
    C = np.array([(int(x) * int(y)) % q for x, y in zip(A, B)], dtype=np.uint64)
    c = o.ntt(C, 1, inverse=True)
    ref = [0] * n
    for i in range(n):
        for j in range(n):
            if i + j < n:
                ref[i + j] += a[i] * b[j]
            else:
                ref[i + j - n] -= a[i] * b[j]
    assert [int(v) for v in c] == [v % q for v in ref]


def test_chacha20_known_answer(oracle_mod):
    # ChaCha20, all-zero key and nonce, block 0 (Bernstein's reference keystream)
    ks = bytes.fromhex(
        "76b8e0ada0f13d90405d6ae55386bd28bdd219b8a08ded1aa836efcc8b770dc7"
        "da41597c5157488d7724e03fb8d84a376a43b8f41518a11cc387b669b2ee6586")
    words = oracle_mod.chacha_block(0, 0, 0)
    assert words.astype("<u8").tobytes() == ks


def test_automorphism_perm_matches_coefficient_definition(oracle_mod):
    O = oracle_mod
    log_n = 5
    n = 1 << log_n
    q = O.gen_primes(log_n, 40, 1)[0]
    o = O.Oracle(log_n, [q], [], 1)
    rng = np.random.default_rng(2)
    a = rng.integers(0, q, n, dtype=np.uint64)
    for g in (5, 25, 2 * n - 1, O.galois_element(log_n, 3)):
        # sigma_g(a)(X) = a(X^g) in R_q[X]/(X^N + 1)
        sa = [0] * n
        for i in range(n):
            e = (i * g) % (2 * n)
            if e < n:
                sa[e] = (sa[e] + int(a[i])) % q
            else:
                sa[e - n] = (sa[e - n] - int(a[i])) % q
        want = o.ntt(np.array(sa, dtype=np.uint64), 1)
        perm = O.automorphism_perm(log_n, g)
        got = o.ntt(a, 1)[perm]
        assert np.array_equal(got, want), g


def test_galois_elements(oracle_mod):
    assert oracle_mod.galois_element(16, 0) == 1
    assert oracle_mod.galois_element(16, 1) == 5
    assert oracle_mod.galois_element(16, 131071) == 131071
    assert oracle_mod.galois_element(16, -1) == pow(5, 32767, 1 << 17)


def test_modup_is_exact_crt_plus_multiple(oracle_mod):
    O = oracle_mod
    log_n = 4
    n = 1 << log_n
    primes = O.gen_primes(log_n, 45, 7)
    q, p = primes[:5], primes[5:]
    o = O.Oracle(log_n, q, p, 2)  # alpha = 3: digits [0,3), [3,5)
    rng = np.random.default_rng(1)
    l = 5
    x = np.array([rng.integers(0, qi, n, dtype=np.uint64) for qi in q])
    for j, (lo, hi) in enumerate(((0, 3), (3, 5))):
        out = o.modup_digit(x, l, j)
        Qj = 1
        for qi in q[lo:hi]:
            Qj *= qi
        targets = q + p
        for k in range(n):
            # exact CRT value of the digit
            v = 0
            for i in range(lo, hi):
                qh = Qj // q[i]
                v += int(x[i][k]) * pow(qh, -1, q[i]) % q[i] * qh
            exact = v % Qj
            for t, pt in enumerate(targets):
                if lo <= t < hi:
                    assert int(out[t][k]) == int(x[t][k])
                    continue
                # fast conversion = exact + e * Qj with 0 <= e < digit width
                diff = (int(out[t][k]) - exact) % pt
                assert any(diff == (e * Qj) % pt for e in range(hi - lo))


def _small_setup(O, log_n=8, L=4, K=2, dnum=2, bits=50):
    primes = O.gen_primes(log_n, bits, L + K)
    o = O.Oracle(log_n, primes[:L], primes[L:], dnum)
    s = O.sample_secret(log_n, 9, 32)
    return o, s, o.secret_to_ntt(s)


def test_encode_matches_canonical_embedding(oracle_mod):
    O = oracle_mod
    log_n = 5
    n = 1 << log_n
    o, _, _ = _small_setup(O, log_n=log_n)
    rng = np.random.default_rng(4)
    slots = n // 2
    z = rng.uniform(-1, 1, slots) + 1j * rng.uniform(-1, 1, slots)
    scale = 2.0 ** 30
    pt = o.encode(z, scale, 1)
    coef = o.ntt(pt, 1, inverse=True)[0].astype(np.float64)
    q0 = o.q[0]
    coef = np.where(coef > q0 / 2, coef - q0, coef)
    zeta = np.exp(1j * np.pi / n)
    for j in range(slots):
        root = zeta ** pow(5, j, 2 * n)
        val = sum(coef[k] * root ** k for k in range(n)) / scale
        assert abs(val - z[j]) < 1e-6
    assert np.max(np.abs(o.decode(pt, 1, slots, scale) - z)) < 1e-6


def test_rotation_conjugation_rescale_decrypt(oracle_mod):
    O = oracle_mod
    log_n = 8
    o, s, s_ntt = _small_setup(O, log_n=log_n)
    n, slots = 1 << log_n, 1 << (log_n - 1)
    rng = np.random.default_rng(5)
    z = rng.uniform(-1, 1, slots) + 1j * rng.uniform(-1, 1, slots)
    scale = 2.0 ** 40
    l = 4
    ct = o.encrypt(o.encode(z, scale, l), l, s_ntt, 1, 1)
    for r in (1, 5, 2 * n - 1):
        g = O.galois_element(log_n, r)
        key = o.keygen_rotation(s_ntt, g, 3)
        out = o.rotate(ct, l, g, key)
        dec = o.decode(o.decrypt(out, l, s_ntt), l, slots, scale)
        ref = np.conj(z) if r == 2 * n - 1 else np.roll(z, -r)
        assert np.max(np.abs(dec - ref)) < 1e-5, r
    # multiply by i
    mi = o.mul_i(ct, 2, l)
    assert np.max(np.abs(o.decode(o.decrypt(mi, l, s_ntt), l, slots, scale) - 1j * z)) < 1e-6
    # rescale: a message at scale q_{l-1} * 2^30 decrypts at scale 2^30
    big = float(o.q[l - 1]) * 2.0 ** 30
    ct2 = o.encrypt(o.encode(z, big, l), l, s_ntt, 1, 2)
    rs = o.rescale(ct2.reshape(2 * l, n), 2, l)
    dec = o.decode(o.decrypt(rs, l - 1, s_ntt), l - 1, slots, 2.0 ** 30)
    assert np.max(np.abs(dec - z)) < 1e-5


def test_relinearisation_decrypts(oracle_mod):
    O = oracle_mod
    log_n = 8
    o, s, s_ntt = _small_setup(O, log_n=log_n)
    slots = 1 << (log_n - 1)
    rng = np.random.default_rng(6)
    x = rng.uniform(-1, 1, slots)
    y = rng.uniform(-1, 1, slots)
    scale = 2.0 ** 40
    l = 4
    a = o.encrypt(o.encode(x, scale, l), l, s_ntt, 1, 1)
    b = o.encrypt(o.encode(y, scale, l), l, s_ntt, 1, 2)
    q = np.array(o.q[:l], dtype=object)[:, None]
    A, B = a.astype(object), b.astype(object)
    d0 = (A[0] * B[0]) % q
    d1 = (A[0] * B[1] + A[1] * B[0]) % q
    d2 = (A[1] * B[1]) % q
    rk = o.keygen_relin(s_ntt, 4)
    k0, k1 = o.keyswitch(d2.astype(np.uint64), l, rk)
    c0 = ((d0 + k0.astype(object)) % q).astype(np.uint64)
    c1 = ((d1 + k1.astype(object)) % q).astype(np.uint64)
    prod = np.stack([c0, c1])
    rs = o.rescale(prod.reshape(2 * l, -1), 2, l)
    dec = o.decode(o.decrypt(rs, l - 1, s_ntt), l - 1, slots, scale * scale / o.q[l - 1])
    assert np.max(np.abs(dec.real - x * y)) < 1e-3
    # relinearise + rescale as one rounding division by P q_{l-1}: the same
    # ciphertext as the two steps (they differ only at rounding ties, with
    # probability about K / q per coefficient)
    ct3 = np.stack([d0, d1, d2]).astype(np.uint64)
    fused = o.relin_rescale(ct3, l, rk)
    assert np.array_equal(fused.reshape(rs.shape), rs)


def test_secret_sampler(oracle_mod):
    s = oracle_mod.sample_secret(16, 3, 192)
    assert int(np.count_nonzero(s)) == 192 and set(np.unique(s)) <= {-1, 0, 1}
    u = oracle_mod.sample_secret(16, 3, 0)
    assert set(np.unique(u)) == {-1, 0, 1}


def test_oracle_bsgs_mac_equals_exact_sum(oracle_mod):
    """orc_bsgs_mac (the CPU baseline of the linear block) against exact
    integer sums: out[c][g] = sum_b pts[g B + b] * babies[c][b] mod q."""

    O = oracle_mod
    primes = O.gen_primes(10, 60, 3)
    o = O.Oracle(10, primes[:2], primes[2:], 1)
    n, l, C, B, G = 1 << 10, 2, 2, 9, 3
    rng = np.random.default_rng(17)
    qs = np.array(primes[:l], dtype=object)
    babies = np.stack([rng.integers(0, q, (C, B, 2, n), dtype=np.uint64) for q in primes[:l]],
                      axis=3)
    pts = np.stack([rng.integers(0, q, (G * B, n), dtype=np.uint64) for q in primes[:l]],
                   axis=1)
    got = o.bsgs_mac(babies, C, B, pts, G, l)
    for c in range(C):
        for g in range(G):
            want = sum(babies[c, b].astype(object) * pts[g * B + b].astype(object)[None]
                       for b in range(B)) % qs[None, :, None]
            assert np.array_equal(got[c, g], want.astype(np.uint64))


def test_giant_chain_ext_decrypts_like_rotations(oracle_mod):
    """The oracle's Horner chain kept in Q_l u P (one poly ModDown'ed per
    step, both at the end; what the library's bsgs_mac runs by default), the
    same chain from extended sums, and the chain of full HRotates decrypt to
    the same giant sum, the exact sum_j rot_{j G}(m_j) of the messages."""

    O = oracle_mod
    log_n = 8
    o, s, s_ntt = _small_setup(O, log_n=log_n, L=5, K=2, dnum=3)
    slots = 1 << (log_n - 1)
    rng = np.random.default_rng(8)
    scale, l, G, step = 2.0 ** 40, 4, 4, 3
    msgs = [rng.uniform(-1, 1, slots) + 1j * rng.uniform(-1, 1, slots) for _ in range(G)]
    inner = np.stack([o.encrypt(o.encode(m, scale, l), l, s_ntt, 1, 10 + j)
                      for j, m in enumerate(msgs)])
    g = O.galois_element(log_n, step)
    key = o.keygen_rotation(s_ntt, g, 5)
    q = np.array(o.q[:l], dtype=object)[:, None]
    acc = inner[G - 1]
    for j in range(G - 2, -1, -1):
        acc = ((o.rotate(acc, l, g, key).astype(object) + inner[j].astype(object)) % q)
        acc = acc.astype(np.uint64)
    ext = o.giant_chain_ext(inner, G, l, g, key)
    # extended sums (P times each ciphertext in Q_l u P, as the ext_normal
    # MAC leaves them) through the same chain
    ext_sums = np.stack([o.rotate_hoisted_ext(c, l, [1], [None])[0] for c in inner])
    ext2 = o.giant_chain_ext(ext_sums, G, l, g, key, extended=True)
    want = sum(np.roll(m, -j * step) for j, m in enumerate(msgs))
    for ct in (acc, ext, ext2):
        dec = o.decode(o.decrypt(ct, l, s_ntt), l, slots, scale)
        assert np.max(np.abs(dec - want)) < 1e-5
    assert not np.array_equal(acc, ext)  # different roundings, same message
