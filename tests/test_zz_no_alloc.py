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


@pytest.mark.parametrize("bits", [50, 60])
def test_rescale_noalloc_matches_rescale_twice_in_a_row(bits):
    """50-bit primes run the binary64 transforms, 60-bit ones the integer
    transforms; both must agree with b2f_rescale and the oracle."""

    ctx, orc = pair(16, 2, 4, bits=bits)
    rng = np.random.default_rng(99 + bits)
    for l, polys in ((16, 2), (9, 4)):  # two calls in a row, different shapes and data
        x = rand_residues(rng, ctx.primes[:l], polys)
        d = to_dev(x)
        got = to_host(_noalloc(ctx, d, polys, l))
        want = to_host(ctx.rescale(d, polys, l))
        assert np.array_equal(got, want)
        assert np.array_equal(got, orc.rescale(x, polys, l))


def test_rescale_noalloc_rejects_oversized_requests():
    ctx, _ = pair(16, 2, 4)
    d = ctx.empty(33, 2)
    with pytest.raises(ValueError, match="scratch"):
        _noalloc(ctx, d, 33, 2)  # the fixed scratch holds 32 polys' last limbs
