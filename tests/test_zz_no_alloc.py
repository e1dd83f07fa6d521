"""b2f_rescale_noalloc: the rescale entry point for callers that cannot
allocate device memory (their HBM belongs to another allocator, or the step
has a fixed memory budget).  It must give the same residues as b2f_rescale,
call after call, through the C ABI.  This file is collected last on purpose."""

from __future__ import annotations

import numpy as np
import pytest

from _ckks import pair, rand_residues, to_dev, to_host

pytestmark = pytest.mark.gpu


def _noalloc(ctx, data, num_polys, l):
    import torch

    from easyfhe import _native

    out = ctx.empty(num_polys, l - 1)
    _native.call("b2f_rescale_noalloc", ctx.handle, int(data.data_ptr()),
                 int(out.data_ptr()), num_polys, l,
                 int(torch.cuda.current_stream().cuda_stream))
    return out


def test_rescale_noalloc_matches_rescale_twice_in_a_row():
    ctx, orc = pair(16, 2, 4)
    rng = np.random.default_rng(99)
    for l in (16, 9):  # two calls in a row, different shapes and data
        x = rand_residues(rng, ctx.primes[:l], 2)
        d = to_dev(x)
        got = to_host(_noalloc(ctx, d, 2, l))
        want = to_host(ctx.rescale(d, 2, l))
        assert np.array_equal(got, want)
        assert np.array_equal(got, orc.rescale(x, 2, l))


def test_rescale_noalloc_rejects_oversized_requests():
    ctx, _ = pair(16, 2, 4)
    d = ctx.empty(3, 16)
    with pytest.raises(ValueError, match="scratch"):
        _noalloc(ctx, d, 3, 16)
