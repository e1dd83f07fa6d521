"""GPU parity of the extended-basis batch ops: hoisted
rotations left in Q_l u P, the grouped pairwise MAC and ModDown, bit-exact
against the oracle, and the attention input call sequence
(llama3fhe/operators/attention/input.py:792-827) decrypted."""

from __future__ import annotations

import numpy as np
import pytest

from _ckks import N, pair, rand_residues, to_dev, to_host

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("arith,l", [("f64", 7), ("int64", 7), ("int64", 1)])
def test_ext_rotations_and_moddown_bit_exact(arith, l):
    """Hoisted rotations left in Q_l u P, an identity among them (the integer
    kernels store the keyed ones from the key inner product, the automorphism
    folded in; l = 1 has fewer Q limbs than special primes), and ModDown."""

    from easyfhe import core

    ctx, orc = pair(8, 2, 3)
    ctx.set_arith(arith)
    try:
        _ext_rotations_and_moddown(ctx, orc, core, l)
    finally:
        ctx.set_arith("auto")


def _ext_rotations_and_moddown(ctx, orc, core, l):
    s_ntt = ctx.secret_to_ntt(core.sample_secret(41, 192))
    gs = [1, core.galois_element(5), core.galois_element(131071)]
    keys = [None] + [ctx.keygen_rotation(s_ntt, g, seed=50 + i) for i, g in enumerate(gs[1:])]
    rng = np.random.default_rng(44)
    ct = rand_residues(rng, ctx.primes[:l], 2)
    dct = to_dev(ct)
    ext = ctx.modup(dct, l)
    got = to_host(ctx.rotate_hoisted_ext(dct, l, ext, gs, keys))
    want = orc.rotate_hoisted_ext(ct, l, gs, [None] + [to_host(k) for k in keys[1:]])
    assert np.array_equal(got, want)
    md = to_host(ctx.moddown_ext(to_dev(want), 3, l))
    assert np.array_equal(md, orc.moddown(want.reshape(6 * (l + 2), N), 6, l).reshape(3, 2, l, N))


def test_pairwise_mac_ext_bit_exact():
    ctx, _ = pair(8, 2, 3)
    l = 5
    primes = ctx.primes[:l] + ctx.primes[8:10]
    rng = np.random.default_rng(45)
    cts = rand_residues(rng, primes, 12).reshape(6, 2, l + 2, N)
    pts = rand_residues(rng, primes, 6)
    got = to_host(ctx.pairwise_mac(to_dev(cts), to_dev(pts), 6, 2, l, 2, l + 2))
    q = np.array(primes, dtype=object)[None, :, None]
    for g in range(2):
        acc = np.zeros((2, l + 2, N), dtype=object)
        for i in range(3 * g, 3 * g + 3):
            acc = (acc + cts[i].astype(object) * pts[i].astype(object)[None]) % q
        assert np.array_equal(got[g], acc.astype(np.uint64))


def test_attention_input_double_hoisting_sequence_decrypts():
    """fast_rotate(output_ext=True) -> unpack -> pack four -> grouped_pairwise_mac
    with extended masks -> moddown_from_ext, then rescale, as
    llama3fhe/operators/attention/input.py:792-827 runs it."""

    from easyfhe import fhe

    offsets = (0, 3, 1024, -7)
    spec = fhe.CKKSContextSpec(depth=3, log_n=16, dnum=2, dcrt_bits=40, first_mod=55,
                               rotations=offsets)
    client, ctx = fhe.generate_client_context(spec, "cuda:0")
    slots = ctx.max_slots
    rng = np.random.default_rng(46)
    x = rng.uniform(-1, 1, slots)
    l = ctx.L
    ct = client.encrypt(x, slots=slots, cur_limbs=l, scaling_factor=ctx.scale_at(l))
    rotations = fhe.fast_rotate(ct, offsets, ctx, output_ext=True)
    items = fhe.unpack_cipher_batch(rotations)
    batch = fhe.pack_cipher_batch(items[h] for h in range(4))
    masks = rng.uniform(-1, 1, (4, slots))
    bundle = fhe.ConstantBundle(vectors={"rows": fhe.PackedRaw(masks)})
    pts = bundle.plaintext("rows", state=fhe.CipherState(l, 1, ctx.scale_at(l)), slots=slots,
                           context=ctx, is_ext=True)
    product = fhe.grouped_pairwise_mac(batch, pts, 1, ctx)
    assert product.is_ext
    out = fhe.rescale(fhe.moddown_from_ext(product, ctx), ctx)
    got = client.decrypt(out)
    want = sum(masks[h] * np.roll(x, -offsets[h]) for h in range(4))
    assert np.max(np.abs(got - want)) < 1e-4
    # a plaintext batch slice (llama3fhe/operators/attention/input.py:1108-1115)
    part = pts.cipher_like([c[1:3] for c in pts.cv], batch_size=2)
    sub = fhe.pack_cipher_batch(items[1:3])
    p2 = fhe.rescale(fhe.moddown_from_ext(fhe.grouped_pairwise_mac(sub, part, 1, ctx), ctx), ctx)
    want2 = masks[1] * np.roll(x, -offsets[1]) + masks[2] * np.roll(x, -offsets[2])
    assert np.max(np.abs(client.decrypt(p2) - want2)) < 1e-4
