"""GPU parity of the feature-major linear path: the
plaintext x ciphertext MAC and its Horner over giant rotations against the CPU
oracle (bit-exact), the CUDA diagonal packers against the reference formula
pinned by the golden fixtures, and the whole LinearOperator.apply call sequence
(llama3fhe/operators/linear/operator.py:195-405) through easyfhe.fhe,
decrypted against the direct matrix-vector product."""

from __future__ import annotations

import numpy as np
import pytest

from _ckks import N, pair, rand_residues, to_dev, to_host
from _packer import bsgs_left, pack_dense, pack_structured

pytestmark = pytest.mark.gpu


def _mac_ref(babies, pts, G, B, primes):
    q = np.array(primes, dtype=object)[None, :, None]
    out = []
    for g in range(G):
        acc = np.zeros(babies.shape[1:], dtype=object)
        for b in range(B):
            acc = (acc + babies[b].astype(object) * pts[g * B + b].astype(object)[None]) % q
        out.append(acc.astype(np.uint64))
    return np.array(out)


def test_mac_bit_exact():
    ctx, _ = pair(8, 2, 3)
    l, B, G = 4, 5, 3
    rng = np.random.default_rng(31)
    babies = rand_residues(rng, ctx.primes[:l], 2 * B).reshape(B, 2, l, N)
    pts = rand_residues(rng, ctx.primes[:l], G * B)
    got = to_host(ctx.mac(to_dev(babies), B, to_dev(pts), G, l))
    assert np.array_equal(got[0], _mac_ref(babies, pts, G, B, ctx.primes[:l]))


@pytest.mark.parametrize("C,B,G", [(5, 64, 8), (9, 24, 3), (2, 33, 11)])
def test_batched_mac_bit_exact(C, B, G):
    """A batch through one MAC launch sequence: every ciphertext of the
    batch, every giant (more than 8 split over launches) equals the modular
    sum of products."""

    ctx, orc = pair(8, 2, 3)
    l = 2
    rng = np.random.default_rng(34 + C)
    babies = rand_residues(rng, ctx.primes[:l], C * B * 2).reshape(C, B, 2, l, N)
    pts = rand_residues(rng, ctx.primes[:l], G * B)
    got = to_host(ctx.mac(to_dev(babies.reshape(C * B, 2, l, N)), B, to_dev(pts), G, l,
                          num_cts=C))
    q = np.array(ctx.primes[:l], dtype=np.uint64)[None, :, None]
    for c in (0, C - 1):  # the first and the last ciphertext of the batch
        for g in range(G):
            want = np.zeros((2, l, N), dtype=np.uint64)
            for b in range(B):  # modular products from the oracle, sums mod q
                want = want + orc.mul_plain(babies[c, b], pts[g * B + b], l)
                want = np.where(want >= q, want - q, want)
            assert np.array_equal(got[c, g], want), (c, g)


@pytest.mark.parametrize("chain", ["extended", "rotations"])
def test_bsgs_mac_horner_bit_exact(chain):
    """The Horner chain over the giants, both ways the library runs it: kept
    in Q_l u P (the default) against the oracle's giant_chain_ext, a full
    HRotate per giant against the oracle's rotations."""

    from easyfhe import core

    ctx, orc = pair(8, 2, 3)
    l, B, G = 4, 3, 3
    s_ntt = ctx.secret_to_ntt(core.sample_secret(12, 192))
    gg = core.galois_element(24)
    key = ctx.keygen_rotation(s_ntt, gg, seed=4)
    rng = np.random.default_rng(32)
    babies = rand_residues(rng, ctx.primes[:l], 2 * B).reshape(B, 2, l, N)
    pts = rand_residues(rng, ctx.primes[:l], G * B)
    ctx.set_giant_chain(chain)
    try:
        got = to_host(ctx.bsgs_mac(to_dev(babies), B, to_dev(pts), G, l, gg, key))
    finally:
        ctx.set_giant_chain("extended")
    inner = _mac_ref(babies, pts, G, B, ctx.primes[:l])
    hkey = to_host(key)
    if chain == "extended":
        assert np.array_equal(got, orc.giant_chain_ext(inner, G, l, gg, hkey))
        return
    q = np.array(ctx.primes[:l], dtype=object)[None, :, None]
    acc = inner[G - 1]
    for g in range(G - 2, -1, -1):
        acc = ((orc.rotate(acc, l, gg, hkey).astype(object) + inner[g].astype(object)) % q)
        acc = acc.astype(np.uint64)
    assert np.array_equal(got, acc)


@pytest.mark.parametrize("conv,l", [("auto", 5), ("tcgen05", 5), ("auto", 1)])
def test_giant_chain_layer_primes_batch(conv, l):
    """The extended-basis chain at the layer's prime sizes (59/60-bit: the
    integer kernels, the chain's steps stored by the key inner product) on a
    batch of 3 ciphertexts with 8 giants, both base conversion kernels
    (tcgen05 takes the one-poly ModDown conversions too), and one Q limb
    under three special primes: every ciphertext bit-exact against the
    oracle's chain."""

    from easyfhe import core

    ctx, orc = pair(6, 3, 3, 60)
    B, G, C = 2, 8, 3
    s_ntt = ctx.secret_to_ntt(core.sample_secret(13, 192))
    gg = core.galois_element(40)
    key = ctx.keygen_rotation(s_ntt, gg, seed=6)
    rng = np.random.default_rng(36)
    babies = rand_residues(rng, ctx.primes[:l], C * B * 2).reshape(C, B, 2, l, N)
    pts = rand_residues(rng, ctx.primes[:l], G * B)
    ctx.set_conv_path(conv)
    try:
        got = to_host(ctx.bsgs_mac(to_dev(babies.reshape(C * B, 2, l, N)), B, to_dev(pts), G,
                                   l, gg, key, num_cts=C))
    finally:
        ctx.set_conv_path("auto")
    hkey = to_host(key)
    for c in range(C):
        inner = _mac_ref(babies[c], pts, G, B, ctx.primes[:l])
        assert np.array_equal(got[c], orc.giant_chain_ext(inner, G, l, gg, hkey)), c


def test_batched_hoisting_and_bsgs_match_single_ciphertext():
    """A batch of ciphertexts through ModUp, hoisted rotations (an identity
    item included) and the BSGS MAC equals the ciphertexts one at a time,
    bit for bit; the single-ciphertext path is pinned to the oracle above."""

    from easyfhe import core

    ctx, _ = pair(8, 2, 3)
    l, B, G, C = 6, 4, 3, 3
    s_ntt = ctx.secret_to_ntt(core.sample_secret(15, 192))
    offsets = [0, 2, 4, 6]
    gal = [core.galois_element(o) for o in offsets]
    keys = [None] + [ctx.keygen_rotation(s_ntt, g, seed=50 + i) for i, g in enumerate(gal[1:])]
    gg = core.galois_element(8)
    gkey = ctx.keygen_rotation(s_ntt, gg, seed=60)
    rng = np.random.default_rng(33)
    cts = rand_residues(rng, ctx.primes[:l], 2 * C).reshape(C, 2, l, N)
    pts = to_dev(rand_residues(rng, ctx.primes[:l], G * B))
    dcts = to_dev(cts)
    ext = ctx.modup(dcts, l, C)
    babies = ctx.rotate_hoisted(dcts, l, ext, gal, keys, num_cts=C)
    out = to_host(ctx.bsgs_mac(babies.reshape(C * B, 2, l, N), B, pts, G, l, gg, gkey,
                               num_cts=C))
    for c in range(C):
        one = to_dev(cts[c])
        e1 = ctx.modup(one, l)
        b1 = ctx.rotate_hoisted(one, l, e1, gal, keys)
        assert np.array_equal(to_host(babies[c]), to_host(b1)), f"babies of ct {c}"
        o1 = to_host(ctx.bsgs_mac(b1, B, pts, G, l, gg, gkey))
        assert np.array_equal(out[c], o1), f"bsgs of ct {c}"


def test_hoisted_rotation_groups_match_single_ciphertext():
    """20 keyed rotations of 5 ciphertexts: the batch runs in launch groups
    of 5 ciphertexts x 12 rotations (each key read once per group), a single
    ciphertext in one group of all 20; every rotation of every ciphertext
    bit-exact between the two, the first against the oracle."""

    from easyfhe import core

    ctx, orc = pair(8, 2, 3)
    l, C = 3, 5
    s_ntt = ctx.secret_to_ntt(core.sample_secret(16, 192))
    offsets = list(range(1, 21))
    gal = [core.galois_element(o) for o in offsets]
    keys = [ctx.keygen_rotation(s_ntt, g, seed=70 + i) for i, g in enumerate(gal)]
    rng = np.random.default_rng(35)
    cts = rand_residues(rng, ctx.primes[:l], 2 * C).reshape(C, 2, l, N)
    dcts = to_dev(cts)
    ext = ctx.modup(dcts, l, C)
    out = to_host(ctx.rotate_hoisted(dcts, l, ext, gal, keys, num_cts=C))
    for c in range(C):
        one = to_dev(cts[c])
        single = to_host(ctx.rotate_hoisted(one, l, ctx.modup(one, l), gal, keys))
        assert np.array_equal(out[c], single), c
    want = orc.rotate_hoisted(cts[0], l, gal[:2], [to_host(k) for k in keys[:2]])
    assert np.array_equal(out[0][:2], want)


def test_dense_packer_matches_reference_formula():
    import torch

    ctx, _ = pair(8, 2, 3)
    rng = np.random.default_rng(33)
    D, lanes, B = 1024, 32, 64
    for dtype in (np.float64, np.float32, np.complex128):
        W = rng.normal(0, 1, (D, D))
        if dtype == np.complex128:
            W = W + 1j * rng.normal(0, 1, (D, D))
        W = W.astype(dtype)
        got = ctx.pack_diagonals(torch.from_numpy(W).to("cuda:0"), D, lanes, B, 8, 4, 32768)
        want = pack_dense(W.astype(np.complex128) if dtype != np.float32 else W.astype(np.float64),
                          dimension=D, token_lanes=lanes, baby_steps=B, giant_base=8,
                          giant_count=4, slots=32768)
        assert np.array_equal(got.cpu().numpy(), want.astype(np.complex128)), dtype


def test_structured_packer_matches_reference_formula():
    import ctypes

    import torch

    from easyfhe import _native

    ctx, _ = pair(8, 2, 3)
    rng = np.random.default_rng(34)
    D, lanes, B = 512, 64, 32
    src = [rng.normal(0, 1, (300, 600)), rng.normal(0, 1, (200, 600)), rng.normal(0, 1, (100, 600))]
    maps = {
        "real_source": rng.integers(-1, 3, D), "imag_source": rng.integers(-1, 3, D),
        "real_scale": rng.normal(0, 1, D), "imag_scale": rng.normal(0, 1, D),
        "column_scale": rng.normal(0, 1, D),
    }
    for side in ("real", "imag"):
        sid = maps[f"{side}_source"]
        maps[f"{side}_row"] = np.where(sid >= 0, rng.integers(0, 100, D), -1)
    col = rng.permutation(600)[:D]
    col[::17] = -1
    maps["column"] = col
    dev = {k: torch.from_numpy(np.ascontiguousarray(v)).to("cuda:0") for k, v in maps.items()}
    dsrc = [torch.from_numpy(s).to("cuda:0") for s in src]
    ptrs = (ctypes.c_void_p * 3)(*[s.data_ptr() for s in dsrc])
    strides = (ctypes.c_int64 * 6)(*[v for s in dsrc for v in s.stride()])
    out = torch.empty(2 * B, 32768, dtype=torch.complex128, device="cuda:0")
    _native.call("b2f_pack_structured", ctx.handle, ptrs, strides, 3, 0,
                 dev["real_source"].data_ptr(), dev["real_row"].data_ptr(),
                 dev["real_scale"].data_ptr(), dev["imag_source"].data_ptr(),
                 dev["imag_row"].data_ptr(), dev["imag_scale"].data_ptr(),
                 dev["column"].data_ptr(), dev["column_scale"].data_ptr(), D, lanes, B, 3, 2,
                 32768, out.data_ptr(), int(torch.cuda.current_stream().cuda_stream))
    want = pack_structured(src, maps, dimension=D, token_lanes=lanes, baby_steps=B,
                           giant_base=3, giant_count=2, slots=32768)
    assert np.array_equal(out.cpu().numpy(), want)


def test_linear_operator_call_sequence_decrypts_to_matvec():
    """The call sequence of LinearOperator.apply with the production plan shape
    scaled down (D = 64, token_lanes = 512, B = 8, 32 rows per chunk):
    prepare_hoisted_baby_rotations, per chunk ConstantBundle(UnpackedRaw).plaintext
    + hoisted_mac_sum + chunk-alignment homo_rotate + homo_add, then rescale."""

    import torch

    from easyfhe import core, fhe

    D, lanes, B, rows = 64, 512, 8, 32
    slots = 32768
    G = D // B
    chunk_giants = rows // B
    chunks = [(i, base, min(chunk_giants, G - base))
              for i, base in enumerate(range(0, G, chunk_giants))]
    giant_offset = B * lanes
    offsets = [b * lanes for b in range(B)]
    rotations = set(offsets[1:]) | {giant_offset} | {base * giant_offset for _, base, _ in chunks if base}
    spec = fhe.CKKSContextSpec(depth=4, log_n=16, dnum=2, dcrt_bits=40, first_mod=55,
                               rotations=tuple(sorted(rotations)), special_bits=60)
    client, ctx = fhe.generate_client_context(spec, "cuda:0")
    rng = np.random.default_rng(35)
    W = rng.normal(0, 1 / np.sqrt(D), (D, D))
    tokens = rng.normal(0, 1, (lanes, D))
    x = np.zeros(slots)
    for f in range(D):
        x[f * lanes:(f + 1) * lanes] = tokens[:, f]
    level_limbs = ctx.L
    ct = client.encrypt(x, slots=slots, cur_limbs=level_limbs,
                        scaling_factor=ctx.scale_at(level_limbs))
    babies = fhe.prepare_hoisted_baby_rotations(ct, offsets, ctx)
    wdev = torch.from_numpy(W).to("cuda:0")
    acc = None
    for _, base, count in chunks:
        def packer(source, req_slots, context, base=base, count=count):
            return ctx.native.pack_diagonals(source, D, lanes, B, base, count, req_slots)

        bundle = fhe.ConstantBundle(vectors={"chunk": fhe.UnpackedRaw(wdev, packer)})
        pts = bundle.plaintext("chunk", state=fhe.CipherState(level_limbs, 1,
                                                              ctx.scale_at(level_limbs)),
                               slots=slots, context=ctx, is_ext=False)
        r = fhe.hoisted_mac_sum(ct, offsets, pts, giant_offset, count, ctx,
                                baby_rotations=babies)
        if base:
            r = fhe.homo_rotate(r, base * giant_offset, ctx)
        acc = r if acc is None else fhe.homo_add(acc, r, ctx)
    out = fhe.rescale(acc, ctx)
    assert out.state.cur_limbs == level_limbs - 1
    got = client.decrypt(out)
    y = tokens @ W.T
    want = np.zeros(slots)
    for f in range(D):
        want[f * lanes:(f + 1) * lanes] = y[:, f]
    # same answer as the reference's BSGS restatement on the clear values
    rows_all = np.concatenate([
        pack_dense(W, dimension=D, token_lanes=lanes, baby_steps=B, giant_base=base,
                   giant_count=count, slots=slots) for _, base, count in chunks])
    clear = bsgs_left(x, rows_all, offsets, giant_offset, chunks).real
    assert np.max(np.abs(clear - want)) < 1e-9
    assert np.max(np.abs(got - want)) < 1e-4
