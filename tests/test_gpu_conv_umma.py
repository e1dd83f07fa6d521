"""GPU parity of the fast base conversion on tcgen05 (csrc/conv_umma.cu).

Every key switch converts digits to the other primes (ModUp) and the special
primes back to Q (ModDown).  On the tcgen05 path both conversions run on
tcgen05.mma with the accumulators in tensor memory (by default the ModDown
conversion of 16+ ciphertexts does);
the rotations below must be bit-identical on every path (tcgen05, mma.sync,
the default mix) and to the CPU oracle, at the layer's parameters (59/60-bit primes, dnum 5, K = 8:
ModUp digits of 13/16 targets at l = 13 and 38 targets at l = 38, which takes
two N-chunks of the MMA) and at 50-bit primes with three special primes."""

from __future__ import annotations

import functools

import numpy as np
import pytest

from _ckks import N, pair, rand_residues, to_dev, to_host

pytestmark = pytest.mark.gpu


@functools.lru_cache(maxsize=None)
def _layer_pair():
    from easyfhe import core
    from oracle.oracle import Oracle

    params = core.Params.from_depth(37, 16, 5, 59, 60)
    return core.NativeContext(params, "cuda:0"), Oracle(16, params.q, params.p, 5)


def _rotate_both_paths(ctx, ct, l, g, key):
    outs = {}
    for path in ("mma_sync", "tcgen05", "auto"):
        ctx.set_conv_path(path)
        outs[path] = to_host(ctx.rotate(to_dev(ct), l, g, key))
    ctx.set_conv_path("auto")
    assert np.array_equal(outs["auto"], outs["mma_sync"])
    return outs


@pytest.mark.parametrize("l", [13, 38])
def test_tcgen05_conversion_layer_parameters(l):
    from easyfhe import core

    ctx, orc = _layer_pair()
    s_ntt = ctx.secret_to_ntt(core.sample_secret(20 + l, 192))
    g = core.galois_element(3)
    key = ctx.keygen_rotation(s_ntt, g, seed=l)
    rng = np.random.default_rng(100 + l)
    cts = rand_residues(rng, ctx.primes[:l], 4).reshape(2, 2, l, N)
    outs = _rotate_both_paths(ctx, cts, l, g, key)
    assert np.array_equal(outs["tcgen05"], outs["mma_sync"])
    assert np.array_equal(outs["tcgen05"][1], orc.rotate(cts[1], l, g, to_host(key)))


def test_tcgen05_conversion_50bit_three_special_primes():
    from easyfhe import core

    L, l = 8, 7
    ctx, orc = pair(L, 3, 3)
    s_ntt = ctx.secret_to_ntt(core.sample_secret(7, 192))
    g = core.galois_element(9)
    key = ctx.keygen_rotation(s_ntt, g, seed=21)
    rng = np.random.default_rng(77)
    cts = rand_residues(rng, ctx.primes[:l], 6).reshape(3, 2, l, N)
    outs = _rotate_both_paths(ctx, cts, l, g, key)
    assert np.array_equal(outs["tcgen05"], outs["mma_sync"])
    for c in range(3):
        assert np.array_equal(outs["tcgen05"][c], orc.rotate(cts[c], l, g, to_host(key)))


def test_tcgen05_conversion_waits_never_time_out():
    import torch

    from easyfhe import _native

    torch.cuda.synchronize()
    assert _native.lib.b2f_conv_wait_errors() == 0


def test_set_conv_path_rejects_unknown():
    ctx, _ = _layer_pair()
    with pytest.raises(ValueError):
        ctx.set_conv_path("wgmma")
