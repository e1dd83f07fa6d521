"""hoisted_mac_sum's hoist strategies and baby anchors (GPU).

The reference selects one of three strategies (llama3fhe/operators/linear/
config.py:9, 286-305; operators/transform.py:108-116 always passes
"ext_normal"):

* ext_normal: babies left in Q_l u P by their key switch, plaintexts encoded
  there, the multiply-accumulate over Q_l u P, then the Horner chain with the
  one giant key (by default straight from the extended sums and kept in
  Q_l u P; with set_giant_chain("rotations") one ModDown per giant and full
  rotations);
* ext_double_hoist: the same sums, each giant's ModDown'ed and rotated with
  its own key back into Q_l u P, summed there, one ModDown at the end.

Both are compared bit for bit with the oracle's restatement of exactly those
steps, and by decryption with the normal strategy.  baby_anchor_step
(config.py:50-57, 207-233) builds the babies in blocks from anchors reached by
the one anchor key; it decrypts to the unanchored result.
"""

from __future__ import annotations

import numpy as np
import pytest

from _ckks import to_host

pytestmark = pytest.mark.gpu

STEP, B, G = 8, 4, 3
OFFSETS = tuple(b * STEP for b in range(B))
GIANT = B * STEP


def _setup():
    from easyfhe import fhe
    from oracle.oracle import Oracle

    rots = set(OFFSETS[1:]) | {g * GIANT for g in range(1, G)}
    # 59/60-bit primes: the integer arithmetic of the layer parameters
    spec = fhe.CKKSContextSpec(depth=5, log_n=16, dnum=3, dcrt_bits=59, first_mod=60,
                               rotations=tuple(sorted(rots)), seed=31)
    client, ctx = fhe.generate_client_context(spec, "cuda:0")
    orc = Oracle(16, ctx.params.q, ctx.params.p, ctx.params.dnum)
    return fhe, client, ctx, orc


def _encode(fhe, ctx, values, l, ext):
    import torch

    scale = ctx.scale_at(l)
    data = ctx.native.encode(torch.from_numpy(values).to(ctx.device), scale, l,
                             ctx.K if ext else 0)
    return fhe.Plaintext(data, fhe.CipherState(l, 1, scale), values.shape[-1], ext)


def _add(a, b, primes):
    q = np.array(primes, dtype=np.uint64)[None, :, None]
    s = a + b
    return np.where(s >= q, s - q, s)


def test_hoisted_mac_sum_extended_strategies_bit_exact():
    fhe, client, ctx, orc = _setup()
    l, K, L = 4, ctx.K, ctx.L
    rng = np.random.default_rng(41)
    z = rng.uniform(-1, 1, ctx.max_slots)
    ct = client.encrypt(z, slots=ctx.max_slots, cur_limbs=l, scaling_factor=ctx.scale_at(l))
    rows = (rng.uniform(-1, 1, (G * B, ctx.max_slots))
            + 1j * rng.uniform(-1, 1, (G * B, ctx.max_slots)))
    pt_q = _encode(fhe, ctx, rows, l, False)
    pt_x = _encode(fhe, ctx, rows, l, True)
    normal = fhe.hoisted_mac_sum(ct, OFFSETS, pt_q, GIANT, G, ctx, strategy="normal")
    ext = fhe.hoisted_mac_sum(ct, OFFSETS, pt_x, GIANT, G, ctx, strategy="ext_normal")
    dh = fhe.hoisted_mac_sum(ct, OFFSETS, pt_x, GIANT, G, ctx, strategy="ext_double_hoist")
    ctx.native.set_giant_chain("rotations")
    ext_rot = fhe.hoisted_mac_sum(ct, OFFSETS, pt_x, GIANT, G, ctx, strategy="ext_normal")
    ctx.native.set_giant_chain("extended")

    # the oracle's restatement of the two extended strategies
    ct_h = to_host(ct.data)
    gal = [fhe.galois_element(o, 16) for o in OFFSETS]
    keys = [None if g == 1 else to_host(ctx.rotation_key(o, l)[1]) for o, g in zip(OFFSETS, gal)]
    babies = orc.rotate_hoisted_ext(ct_h, l, gal, keys)            # [B, 2, l+K, N]
    inner = orc.bsgs_mac(babies[None], 1, B, to_host(pt_x.data), G, l, K)[0]
    giants = orc.moddown(inner.reshape(2 * G, l + K, -1), 2 * G, l).reshape(G, 2, l, -1)
    qs = ctx.params.q[:l]
    ext_primes = list(ctx.params.q[:l]) + list(ctx.params.p)
    gg = fhe.galois_element(GIANT, 16)
    gkey = to_host(ctx.rotation_key(GIANT, l)[1])
    acc = giants[G - 1]
    for g in range(G - 2, -1, -1):
        acc = _add(orc.rotate(acc, l, gg, gkey), giants[g], qs)
    assert np.array_equal(to_host(ext_rot.data), acc)  # a ModDown per giant and rotation
    # the default: the chain straight from the extended sums, one ModDown
    assert np.array_equal(to_host(ext.data),
                          orc.giant_chain_ext(inner, G, l, gg, gkey, extended=True))
    acc_x = inner[0]
    for g in range(1, G):
        gk = fhe.galois_element(g * GIANT, 16)
        r = orc.rotate_hoisted_ext(giants[g], l, [gk],
                                   [to_host(ctx.rotation_key(g * GIANT, l)[1])])[0]
        acc_x = _add(acc_x, r, ext_primes)
    assert np.array_equal(to_host(dh.data), orc.moddown(acc_x, 2, l))

    # the same linear map: every strategy decrypts to the normal result
    want = client.decrypt_complex(fhe.rescale(normal, ctx))
    for r in (ext, ext_rot, dh):
        got = client.decrypt_complex(fhe.rescale(r, ctx))
        assert np.max(np.abs(got - want)) < 1e-6 * max(1.0, np.max(np.abs(want)))


def test_baby_anchor_blocks_and_strategy_errors():
    fhe, client, ctx, _ = _setup()
    l = 4
    rng = np.random.default_rng(43)
    z = rng.uniform(-1, 1, ctx.max_slots)
    ct = client.encrypt(z, slots=ctx.max_slots, cur_limbs=l, scaling_factor=ctx.scale_at(l))
    rows = rng.uniform(-1, 1, (G * B, ctx.max_slots)).astype(np.complex128)
    pt = _encode(fhe, ctx, rows, l, False)
    plain = fhe.hoisted_mac_sum(ct, OFFSETS, pt, GIANT, G, ctx)
    # anchor 2: babies 0,1 hoisted from ct, babies 2,3 from rot_16(ct)
    anchored = fhe.hoisted_mac_sum(ct, OFFSETS, pt, GIANT, G, ctx, baby_anchor_step=2)
    want = client.decrypt_complex(fhe.rescale(plain, ctx))
    got = client.decrypt_complex(fhe.rescale(anchored, ctx))
    assert np.max(np.abs(got - want)) < 1e-6 * max(1.0, np.max(np.abs(want)))
    with pytest.raises(ValueError, match="hoist strategy"):
        fhe.hoisted_mac_sum(ct, OFFSETS, pt, GIANT, G, ctx, strategy="ext_triple")
    with pytest.raises(ValueError, match="extended basis"):
        fhe.hoisted_mac_sum(ct, OFFSETS, pt, GIANT, G, ctx, strategy="ext_normal")
    babies = fhe.prepare_hoisted_baby_rotations(ct, OFFSETS, ctx)
    with pytest.raises(ValueError, match="strategy"):
        fhe.hoisted_mac_sum(ct, OFFSETS, _encode(fhe, ctx, rows, l, True), GIANT, G, ctx,
                            strategy="ext_normal", baby_rotations=babies)


def test_normal_strategy_giant_chains_decrypt_alike():
    """The normal strategy's Horner chain, kept in Q_l u P (the default) or
    run as full HRotates: the same linear map after the rescale, within the
    key-switch noise, and the default is the chain the library takes."""

    fhe, client, ctx, _ = _setup()
    l = 4
    rng = np.random.default_rng(44)
    z = rng.uniform(-1, 1, ctx.max_slots)
    ct = client.encrypt(z, slots=ctx.max_slots, cur_limbs=l, scaling_factor=ctx.scale_at(l))
    rows = rng.uniform(-1, 1, (G * B, ctx.max_slots)).astype(np.complex128)
    pt = _encode(fhe, ctx, rows, l, False)
    outs = {}
    for chain in ("rotations", "extended"):
        ctx.native.set_giant_chain(chain)
        outs[chain] = fhe.hoisted_mac_sum(ct, OFFSETS, pt, GIANT, G, ctx)
    default = fhe.hoisted_mac_sum(ct, OFFSETS, pt, GIANT, G, ctx)
    assert np.array_equal(to_host(default.data), to_host(outs["extended"].data))
    assert not np.array_equal(to_host(outs["rotations"].data), to_host(outs["extended"].data))
    want = client.decrypt_complex(fhe.rescale(outs["rotations"], ctx))
    got = client.decrypt_complex(fhe.rescale(outs["extended"], ctx))
    assert np.max(np.abs(got - want)) < 1e-6 * max(1.0, np.max(np.abs(want)))
    with pytest.raises(ValueError):
        ctx.native.set_giant_chain("ext")
