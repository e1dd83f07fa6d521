"""homo_mul_relin_rescale_postop with its post-operation fused (GPU).

The Chebyshev basis step of the reference's Paterson-Stockmeyer evaluator
(llama3fhe/operators/nonlinear/polynomial.py:108-159), out = 2 rescale(relin(a
b)) - T_{a-b} + c, runs its x2, subtraction and scalar in the epilogue of the
relinearise-rescale's last transform.  It must give the residues of the
unfused sequence (relinearise-rescale, homo_add, homo_sub of the aligned
subtrahend, homo_add_scalar) and launch no more kernels than the
relinearise-rescale alone.
"""

from __future__ import annotations

import numpy as np
import pytest

from _ckks import to_host

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("bits", [(50, 55), (59, 60)], ids=["binary64", "int64"])
@pytest.mark.parametrize("batch", [1, 3])
def test_fused_postop_equals_unfused_sequence(bits, batch):
    from easyfhe import _native, fhe

    spec = fhe.CKKSContextSpec(depth=5, log_n=16, dnum=3, dcrt_bits=bits[0],
                               first_mod=bits[1], seed=71)
    client, ctx = fhe.generate_client_context(spec, "cuda:0")
    rng = np.random.default_rng(72 + batch)
    l = 5

    def enc(limbs):
        cts = [client.encrypt(rng.uniform(-1, 1, ctx.max_slots), slots=ctx.max_slots,
                              cur_limbs=limbs, scaling_factor=ctx.scale_at(limbs))
               for _ in range(batch)]
        return cts[0] if batch == 1 else fhe.pack_cipher_batch(cts)

    a, b = enc(l), enc(l)
    sub = enc(l)  # one level above the result: read at its own level
    plain = fhe._relinearize_rescale(fhe.homo_mul_no_relin(a, b, ctx), ctx)
    scalar = fhe.encode_scalar(-0.75, cur_limbs=l - 1, scale_degree=1,
                               scaling_factor=plain.state.scaling_factor, context=ctx)
    want = fhe.homo_add(plain, plain, ctx)
    want = fhe.homo_sub(want, fhe.align_to(sub, want.state, ctx), ctx)
    want = fhe.homo_add_scalar(want, scalar, ctx)
    n0 = _native.lib.b2f_launch_count()
    fhe._relinearize_rescale(fhe.homo_mul_no_relin(a, b, ctx), ctx)
    n1 = _native.lib.b2f_launch_count()
    got = fhe.homo_mul_relin_rescale_postop(a, b, ctx, apply_double=True, sub=sub,
                                            scalar=scalar)
    n2 = _native.lib.b2f_launch_count()
    assert got.state == want.state
    assert np.array_equal(to_host(got.data), to_host(want.data))
    assert n2 - n1 == n1 - n0  # the post-operation adds no launch
    # the scalar alone and the doubling alone
    one = fhe.homo_mul_relin_rescale_postop(a, b, ctx, apply_double=True)
    assert np.array_equal(to_host(one.data), to_host(fhe.homo_add(plain, plain, ctx).data))
    two = fhe.homo_mul_relin_rescale_postop(a, b, ctx, scalar=scalar)
    assert np.array_equal(to_host(two.data),
                          to_host(fhe.homo_add_scalar(plain, scalar, ctx).data))
