"""Key residency on the GPU: clear_cuda_rotation_cache(keep_rotations=...) as the
reference calls it (llama3fhe/operators/nonlinear/bootstrap.py:191-215,
graph.py:1158) moves the other rotation keys to host memory and they come back
on their next use (auto_load_keys); level-truncated keys keep only the digits
their levels read.  Rotations through evicted, reloaded and truncated keys are
bit-identical to the resident full keys."""

from __future__ import annotations

import numpy as np
import pytest

from _ckks import to_host

pytestmark = pytest.mark.gpu


def _context(auto_load: bool):
    from easyfhe import fhe

    spec = fhe.CKKSContextSpec(depth=7, log_n=16, dnum=4, dcrt_bits=50, first_mod=55,
                               rotations=(1, 2, 5), auto_load_keys=auto_load, seed=11)
    return fhe.generate_client_context(spec, "cuda:0")


def test_evict_reload_and_truncate_rotation_keys():
    from easyfhe import fhe

    client, ctx = _context(True)
    rng = np.random.default_rng(3)
    z = rng.uniform(-1, 1, ctx.max_slots)
    top = ctx.L
    ct = client.encrypt(z, slots=ctx.max_slots, cur_limbs=top, scaling_factor=ctx.scale_at(top))
    low = fhe.align_to(ct, ct.state.replace(cur_limbs=2), ctx)
    want = {r: to_host(fhe.homo_rotate(ct, r, ctx).data) for r in (1, 2, 5)}
    want_low = to_host(fhe.homo_rotate(low, 5, ctx).data)
    before = ctx.key_bytes()

    freed = ctx.clear_cuda_rotation_cache(keep_rotations=[1])
    after = ctx.key_bytes()
    assert freed > 0 and after["device"] == before["device"] - freed
    assert after["host"] == freed
    g2 = fhe.galois_element(2, 16)
    assert not ctx.rotation_keys[g2].is_cuda
    for r in (1, 2, 5):  # 2 and 5 reload on use
        assert np.array_equal(to_host(fhe.homo_rotate(ct, r, ctx).data), want[r]), r
    assert ctx.rotation_keys[g2].is_cuda

    digits = ctx.rotation_keys[fhe.galois_element(5, 16)].shape[0]
    freed = ctx.truncate_rotation_keys(2, rotations=[5])
    kept = ctx.rotation_keys[fhe.galois_element(5, 16)].shape[0]
    assert kept == -(-2 // ctx.native.alpha) and kept < digits and freed > 0
    assert np.array_equal(to_host(fhe.homo_rotate(low, 5, ctx).data), want_low)
    with pytest.raises(ValueError):
        fhe.homo_rotate(ct, 5, ctx)  # the top level needs every digit


def test_evicted_key_without_auto_load_is_an_error():
    from easyfhe import fhe

    client, ctx = _context(False)
    ct = client.encrypt(np.zeros(ctx.max_slots), slots=ctx.max_slots, cur_limbs=3,
                        scaling_factor=ctx.scale_at(3))
    ctx.clear_cuda_rotation_cache()
    with pytest.raises(ValueError):
        fhe.homo_rotate(ct, 1, ctx)


def test_keys_materialised_on_first_use_equal_eager_keys():
    """With auto_load_keys each declared key is generated on its first use, with
    the digits that level reads (and regrown when a higher level needs more).
    Rotations through those keys equal rotations through the keys generated
    eagerly at the top level, at a low and at the top level."""

    from easyfhe import fhe

    client_l, lazy = _context(True)
    client_e, eager = _context(False)
    assert not lazy.rotation_keys and len(eager.rotation_keys) == 3
    z = np.random.default_rng(9).uniform(-1, 1, lazy.max_slots)
    for ctx, client in ((lazy, client_l), (eager, client_e)):
        ctx._probe = client.encrypt(z, slots=ctx.max_slots, cur_limbs=ctx.L,
                                    scaling_factor=ctx.scale_at(ctx.L))
    g5 = fhe.galois_element(5, 16)
    outs = {}
    for ctx in (lazy, eager):
        low = fhe.align_to(ctx._probe, ctx._probe.state.replace(cur_limbs=2), ctx)
        outs[id(ctx)] = [to_host(fhe.homo_rotate(low, 5, ctx).data)]
        if ctx is lazy:  # sized for two limbs: the first ceil(2 / alpha) digits
            assert lazy.rotation_keys[g5].shape[0] == -(-2 // lazy.native.alpha)
        outs[id(ctx)].append(to_host(fhe.homo_rotate(ctx._probe, 5, ctx).data))
    assert lazy.rotation_keys[g5].shape[0] == eager.rotation_keys[g5].shape[0]
    assert np.array_equal(outs[id(lazy)][0], outs[id(eager)][0])
    assert np.array_equal(outs[id(lazy)][1], outs[id(eager)][1])
    assert lazy.keys_generated == 2  # once at two limbs, once regrown at the top
    with pytest.raises(ValueError):
        fhe.homo_rotate(lazy._probe, 3, lazy)  # 3 was never declared
