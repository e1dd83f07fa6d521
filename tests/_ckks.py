"""Shared helpers for the GPU parity tests: one GPU context and one CPU oracle
context over the same primes, and converters between the two."""

from __future__ import annotations

import functools

import numpy as np

N = 1 << 16


def rand_residues(rng, primes, polys: int) -> np.ndarray:
    """[polys, len(primes), N] uniform residues."""

    out = np.empty((polys, len(primes), N), dtype=np.uint64)
    for i, q in enumerate(primes):
        out[:, i, :] = rng.integers(0, q, size=(polys, N), dtype=np.uint64)
    return out


@functools.lru_cache(maxsize=None)
def pair(L: int, K: int, dnum: int, bits: int = 50):
    """(NativeContext, Oracle) over the same L + K primes of `bits` bits."""

    from easyfhe import core
    from oracle.oracle import Oracle

    params = core.Params.uniform(L, K, dnum, bits=bits)
    ctx = core.NativeContext(params, "cuda:0")
    orc = Oracle(16, params.q, params.p, dnum)
    return ctx, orc


def to_dev(a: np.ndarray):
    import torch

    from easyfhe import core

    return core.from_numpy_u64(a, torch.device("cuda:0"))


def to_host(t) -> np.ndarray:
    from easyfhe import core

    return core.to_numpy_u64(t)
