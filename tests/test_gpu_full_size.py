"""Parity at the benchmark's full sizes.  HRotate at the primitive bench
configuration (l = 24, dnum 3, K = 2, 32 ciphertexts sharing one key): sampled
ciphertexts bit-exact against the CPU oracle, and the binary64 and 64-bit
integer kernels equal on the whole batch.  The layer parameters' top level
(l = 38, dnum 5, K = 8, 59/60-bit primes): rotation and the fused
relinearise + rescale bit-exact against the oracle, which reaches the widest
tensor-core conversions (K + 2 = 10 words) in integer arithmetic."""

from __future__ import annotations

import functools

import numpy as np
import pytest

from _ckks import N, rand_residues, to_dev, to_host

pytestmark = pytest.mark.gpu


@functools.lru_cache(maxsize=None)
def _bench_pair():
    from easyfhe import core
    from oracle.oracle import Oracle

    params = core.Params.uniform(24, 2, 3, bits=50)
    return core.NativeContext(params, "cuda:0"), Oracle(16, params.q, params.p, 3)


@functools.lru_cache(maxsize=None)
def _layer_pair():
    from easyfhe import core
    from oracle.oracle import Oracle

    params = core.Params.from_depth(37, 16, 5, 59, 60)
    return core.NativeContext(params, "cuda:0"), Oracle(16, params.q, params.p, 5)


def test_hrotate_bench_configuration():
    from easyfhe import core

    ctx, orc = _bench_pair()
    assert ctx.arith == "f64"
    l, C = 24, 32
    s_ntt = ctx.secret_to_ntt(core.sample_secret(2024, 192))
    g = core.galois_element(1)
    key = ctx.keygen_rotation(s_ntt, g, seed=7)
    rng = np.random.default_rng(24)
    cts = rand_residues(rng, ctx.primes[:l], 2 * C).reshape(C, 2, l, N)
    dev = to_dev(cts)
    got = to_host(ctx.rotate(dev, l, g, key))
    hkey = to_host(key)
    for c in (0, 17, 31):
        assert np.array_equal(got[c], orc.rotate(cts[c], l, g, hkey)), f"ct {c}"
    ctx.set_arith("int64")
    try:
        assert np.array_equal(to_host(ctx.rotate(dev, l, g, key)), got)
    finally:
        ctx.set_arith("auto")


def test_layer_top_level_rotation_and_relin_rescale():
    from easyfhe import core

    ctx, orc = _layer_pair()
    assert ctx.L == 38 and ctx.K == 8 and ctx.arith == "int64"
    l = 38
    s_ntt = ctx.secret_to_ntt(core.sample_secret(38, 192))
    g = core.galois_element(5)
    key = ctx.keygen_rotation(s_ntt, g, seed=3)
    rk = ctx.keygen_relin(s_ntt, seed=4)
    rng = np.random.default_rng(38)
    ct = rand_residues(rng, ctx.primes[:l], 2)
    got = to_host(ctx.rotate(to_dev(ct[None]), l, g, key))[0]
    assert np.array_equal(got, orc.rotate(ct, l, g, to_host(key)))
    ct3 = rand_residues(rng, ctx.primes[:l], 3)
    fused = to_host(ctx.relinearize_rescale(to_dev(ct3[None]), l, rk))[0]
    assert np.array_equal(fused, orc.relin_rescale(ct3, l, to_host(rk)))
