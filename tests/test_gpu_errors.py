"""Failure paths on the GPU (failure detection): argument
and level errors surface as Python exceptions from the C-ABI status codes,
before any kernel runs, and leave the context usable; ciphertexts survive a
save / load round trip at a stage boundary."""

from __future__ import annotations

import numpy as np
import pytest

from _ckks import N, pair, rand_residues, to_dev, to_host

pytestmark = pytest.mark.gpu


def _rotation_setup():
    from easyfhe import core

    ctx, orc = pair(8, 2, 3)
    s_ntt = ctx.secret_to_ntt(core.sample_secret(21, 192))
    g = core.galois_element(3)
    key = ctx.keygen_rotation(s_ntt, g, seed=5)
    rng = np.random.default_rng(70)
    ct = rand_residues(rng, ctx.primes[:6], 2)
    return ctx, orc, g, key, ct


def test_bad_level_galois_and_workspace_raise_then_context_still_works():
    from easyfhe import _native, core

    ctx, orc, g, key, ct = _rotation_setup()
    dct = to_dev(ct)
    with pytest.raises(ValueError, match="level limbs"):
        ctx.rotate(dct, 99, g, key)
    with pytest.raises(ValueError, match="galois"):
        ctx.rotate(dct, 6, 4, key)  # even: not an automorphism of Z[X]/(X^N + 1)
    out = dct.clone()
    with pytest.raises(ValueError, match="workspace too small"):
        _native.call("b2f_rotate", ctx.handle, dct.data_ptr(), out.data_ptr(), 1, 6, g,
                     key.data_ptr(), out.data_ptr(), 8, None)
    with pytest.raises(ValueError, match="in-place"):
        _native.call("b2f_rotate", ctx.handle, dct.data_ptr(), dct.data_ptr(), 1, 6, g,
                     key.data_ptr(), None, 0, None)
    # nothing was launched: the context still rotates bit-exactly
    got = to_host(ctx.rotate(dct, 6, g, key))
    assert np.array_equal(got, orc.rotate(ct, 6, g, to_host(key)))
    assert core.lib.b2f_last_error()


def test_misaligned_limbs_raise_before_any_launch():
    """The transforms move 32-byte sectors: a buffer that is only 16-byte
    aligned is refused on the host and the context keeps working."""
    import torch

    from easyfhe import _native

    ctx, orc = pair(8, 2, 3)
    rng = np.random.default_rng(72)
    x = rand_residues(rng, ctx.primes[:2], 1)
    buf = torch.zeros(2 * N + 4, dtype=torch.int64, device="cuda:0")
    with pytest.raises(ValueError, match="32-byte aligned"):
        _native.call("b2f_ntt", ctx.handle, buf.data_ptr() + 16, 1, 2, 0, 0, None)
    from easyfhe import core

    g = core.galois_element(1)
    s_ntt = ctx.secret_to_ntt(core.sample_secret(22, 192))
    key = ctx.keygen_rotation(s_ntt, g, seed=6)
    ct = to_dev(rand_residues(rng, ctx.primes[:6], 2))
    out = ct.clone()
    need = core.lib.b2f_rotate_workspace(ctx.handle, 1, 6)
    ws = torch.empty(need + 512, dtype=torch.uint8, device="cuda:0")
    with pytest.raises(ValueError, match="256-byte aligned"):
        _native.call("b2f_rotate", ctx.handle, ct.data_ptr(), out.data_ptr(), 1, 6, g,
                     key.data_ptr(), ws.data_ptr() + 128, need, None)
    d = to_dev(x)
    ctx.ntt(d, 2, 0, inverse=False)
    assert np.array_equal(to_host(d), orc.ntt(x, 2, 0, inverse=False).reshape(x.shape))


def test_fhe_level_errors_are_value_errors():
    from easyfhe import fhe

    client, ctx = fhe.generate_client_context(
        fhe.CKKSContextSpec(depth=3, log_n=16, dnum=2, dcrt_bits=40, first_mod=55,
                            rotations=(1,)), "cuda:0")
    ct = client.encrypt(np.ones(ctx.max_slots), slots=ctx.max_slots, cur_limbs=2,
                        scaling_factor=ctx.scale_at(2))
    one = fhe.rescale(ct, ctx)
    with pytest.raises(ValueError):
        fhe.rescale(one, ctx)  # a single limb cannot be rescaled
    with pytest.raises(ValueError):
        fhe.align_to(one, one.state.replace(cur_limbs=2), ctx)  # no raising
    with pytest.raises(ValueError):
        fhe.homo_mul_relin(ct, fhe.homo_mul_no_relin(ct, ct, ctx), ctx)


def test_ciphertext_save_load_round_trip(tmp_path):
    from easyfhe import fhe

    client, ctx = fhe.generate_client_context(
        fhe.CKKSContextSpec(depth=3, log_n=16, dnum=2, dcrt_bits=40, first_mod=55,
                            rotations=(1,)), "cuda:0")
    rng = np.random.default_rng(71)
    z = rng.uniform(-1, 1, ctx.max_slots)
    cts = [client.encrypt(z * (i + 1), slots=ctx.max_slots, cur_limbs=3,
                          scaling_factor=ctx.scale_at(3)) for i in range(2)]
    batch = fhe.pack_cipher_batch(cts)
    path = tmp_path / "state.npz"
    fhe.save_ciphertext(batch, path)
    back = fhe.load_ciphertext(path, ctx)
    assert back.state == batch.state and back.slots == batch.slots
    assert np.array_equal(to_host(back.data), to_host(batch.data))
    for i, c in enumerate(fhe.unpack_cipher_batch(back)):
        assert np.max(np.abs(client.decrypt(c) - z * (i + 1))) < 1e-6
    np.savez(path, **{**dict(np.load(path)), "cur_limbs": 2})
    with pytest.raises(ValueError):
        fhe.load_ciphertext(path, ctx)
