"""CKKS bootstrapping on the GPU (bs.bootstrap): ModRaise bit-exact against
the oracle, then bs.bootstrap at the reference's layer parameters
(assets/feature_major.json: logN 16, depth 37, dnum 5, dcrtBits 59, firstMod
60; BootstrapSpec(15, (4, 4), output_levels = depth - 18), llama3fhe/model.py:
26-59, settings.py:100-108) checked by decryption, and the two-pass Meta-BTS
correction of llama3fhe/operators/nonlinear/bootstrap.py:352-437 run through
the same fhe calls."""

from __future__ import annotations

import functools
import time

import numpy as np
import pytest

from _ckks import N, pair, rand_residues, to_dev, to_host

pytestmark = pytest.mark.gpu


def test_modraise_bit_exact():
    ctx, orc = pair(8, 2, 3)
    rng = np.random.default_rng(60)
    x = rand_residues(rng, ctx.primes[:1], 2)
    got = to_host(ctx.modraise(to_dev(x), 2, 8))
    assert np.array_equal(got, orc.modraise(x, 2, 8))


@functools.lru_cache(maxsize=None)
def _layer_context():
    from easyfhe import fhe
    from easyfhe.bs import openfhe as bs

    spec = bs.BootstrapSpec(log_slots=15, level_budget=(4, 4), output_levels=19)
    rots = bs.requirements((spec,), 16).rotations
    client, ctx = fhe.generate_client_context(
        fhe.CKKSContextSpec(depth=37, log_n=16, dnum=5, dcrt_bits=59, first_mod=60,
                            rotations=rots), "cuda:0")
    program = bs.generate(ctx, spec)
    return client, ctx, program


def _encrypt(client, ctx, z, limbs):
    return client.encrypt(np.asarray(z), slots=ctx.max_slots, cur_limbs=limbs,
                          scaling_factor=ctx.scale_at(limbs))


def test_bootstrap_layer_parameters():
    import torch

    from easyfhe.bs import openfhe as bs

    client, ctx, program = _layer_context()
    assert ctx.L == 38 and ctx.K == 8
    rng = np.random.default_rng(61)
    z = rng.uniform(-1, 1, ctx.max_slots) + 1j * rng.uniform(-1, 1, ctx.max_slots)
    ct = _encrypt(client, ctx, z, 2)
    out = bs.bootstrap(ct, ctx, program)  # warm-up
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    out = bs.bootstrap(ct, ctx, program)
    torch.cuda.synchronize()
    seconds = time.perf_counter() - t0
    assert out.state.cur_limbs == 20  # output_levels 19 = depth - 18
    assert out.state.scaling_factor == ct.state.scaling_factor
    err = np.max(np.abs(client.decrypt_complex(out) - z))
    print(f"bootstrap: {seconds * 1e3:.1f} ms, max error 2^{np.log2(err):.1f}")
    assert err < 2.0 ** -17  # 2^-19.3 measured on B200


def test_bootstrap_output_is_at_the_nominal_scale():
    """An input whose tracked scale is off 2^dcrt_bits (the Paterson-Stockmeyer
    evaluator's outputs are: every product squares the ratio) comes out with
    the same message at the nominal scale scale_at(L), so the ratio does not
    compound over a layer's polynomial-and-refresh cycles."""

    from easyfhe.bs import openfhe as bs

    client, ctx, program = _layer_context()
    rng = np.random.default_rng(62)
    z = rng.uniform(-1, 1, ctx.max_slots) + 1j * rng.uniform(-1, 1, ctx.max_slots)
    ct = client.encrypt(np.asarray(z), slots=ctx.max_slots, cur_limbs=3,
                        scaling_factor=ctx.scale_at(3) * 1.37)
    out = bs.bootstrap(ct, ctx, program)
    assert out.state.scaling_factor == ctx.scale_at(ctx.L)
    err = np.max(np.abs(client.decrypt_complex(out) - z))
    assert err < 2.0 ** -17, np.log2(err)


def test_meta_bts_two_pass_correction():
    """The reference's two-pass correction (bootstrap.py:398-431) with
    precision_bits = 16 on top of bs.bootstrap."""

    from easyfhe import fhe
    from easyfhe.bs import openfhe as bs

    client, ctx, program = _layer_context()
    rng = np.random.default_rng(62)
    z = rng.uniform(-1, 1, ctx.max_slots) + 1j * rng.uniform(-1, 1, ctx.max_slots)
    original = _encrypt(client, ctx, z, 3)
    first = bs.bootstrap(original, ctx, program)
    factor = 1 << 16

    def mul_int(c, v):
        enc = fhe.encode_scalar(int(v), cur_limbs=int(c.state.cur_limbs), scale_degree=0,
                                mode="integer", context=ctx)
        return fhe.homo_mul_scalar(c, enc, ctx)

    first_scaled = mul_int(first, factor)
    first_down = fhe.align_to(first_scaled, original.state, ctx)
    original_scaled = fhe.align_to(mul_int(original, factor), first_down.state, ctx)
    error = bs.bootstrap(fhe.homo_sub(first_down, original_scaled, ctx), ctx, program)
    first_aligned = fhe.align_to(first_scaled, error.state, ctx)
    error_aligned = fhe.align_to(error, first_aligned.state, ctx)
    corrected = fhe.homo_sub(first_aligned, error_aligned, ctx)
    enc = fhe.encode_scalar(1.0 / factor, cur_limbs=int(corrected.state.cur_limbs),
                            scale_degree=1, scaling_factor=corrected.state.scaling_factor,
                            context=ctx)
    result = fhe.homo_mul_scalar_rescale(corrected, enc, ctx)
    e1 = np.max(np.abs(client.decrypt_complex(first) - z))
    e2 = np.max(np.abs(client.decrypt_complex(result) - z))
    print(f"Meta-BTS: one pass 2^{np.log2(e1):.1f}, two passes 2^{np.log2(e2):.1f}")
    assert e1 < 2.0 ** -17
    assert e2 < 2.0 ** -28  # 2^-35 measured on B200: the correction adds ~16 bits


@functools.lru_cache(maxsize=None)
def _program_context():
    """One context with the keys of a deep (3, 3) full-slot program and a
    sparse (slim, 2^7 slots) program (llama3fhe/operators/nonlinear/
    bootstrap.py:60-85, model.py:49-57)."""

    from easyfhe import fhe
    from easyfhe.bs import openfhe as bs

    deep = bs.BootstrapSpec(log_slots=15, level_budget=(3, 3), output_levels=21)
    slim = bs.BootstrapSpec(log_slots=7, level_budget=(4, 4), output_levels=19)
    rots = bs.requirements((deep, slim), 16).rotations
    client, ctx = fhe.generate_client_context(
        fhe.CKKSContextSpec(depth=37, log_n=16, dnum=5, dcrt_bits=59, first_mod=60,
                            rotations=rots, seed=7), "cuda:0")
    return client, ctx, bs.generate(ctx, deep), bs.generate(ctx, slim)


def test_bootstrap_deep_program():
    from easyfhe.bs import openfhe as bs

    client, ctx, deep, _ = _program_context()
    rng = np.random.default_rng(63)
    z = rng.uniform(-1, 1, ctx.max_slots) + 1j * rng.uniform(-1, 1, ctx.max_slots)
    out = bs.bootstrap(_encrypt(client, ctx, z, 2), ctx, deep)
    assert out.state.cur_limbs == 22  # depth 16 at (3, 3): output_levels 21
    err = np.max(np.abs(client.decrypt_complex(out) - z))
    print(f"deep (3, 3) bootstrap: max error 2^{np.log2(err):.1f}")
    assert err < 2.0 ** -17


def test_bootstrap_sparse_slots():
    from easyfhe.bs import openfhe as bs

    client, ctx, _, slim = _program_context()
    n = slim.spec.slots
    rng = np.random.default_rng(64)
    z = rng.uniform(-1, 1, n) + 1j * rng.uniform(-1, 1, n)
    ct = client.encrypt(z, slots=n, cur_limbs=2, scaling_factor=ctx.scale_at(2))
    out = bs.bootstrap(ct, ctx, slim)
    assert out.slots == n and out.state.cur_limbs == 20
    err = np.max(np.abs(client.decrypt_complex(out) - z))
    print(f"sparse (2^7 slots) bootstrap: max error 2^{np.log2(err):.1f}")
    assert err < 2.0 ** -17


def test_bootstrap_batch_matches_single():
    """Two ciphertexts bootstrapped as one batch equal the two bootstraps
    one at a time, bit for bit (every step is exact integer arithmetic on
    the same constants)."""

    from easyfhe import fhe
    from easyfhe.bs import openfhe as bs

    client, ctx, program = _layer_context()
    rng = np.random.default_rng(65)
    zs = [rng.uniform(-1, 1, ctx.max_slots) + 1j * rng.uniform(-1, 1, ctx.max_slots)
          for _ in range(2)]
    cts = [_encrypt(client, ctx, z, 2) for z in zs]
    batch = bs.bootstrap(fhe.pack_cipher_batch(cts), ctx, program)
    assert batch.batch_size == 2
    for i, c in enumerate(cts):
        one = bs.bootstrap(c, ctx, program)
        assert np.array_equal(to_host(batch.data[i]), to_host(one.data)), f"ct {i}"
        assert batch.state == one.state
