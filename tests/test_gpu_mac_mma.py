"""GPU parity of the tensor-core BSGS multiply-accumulate (csrc/mac_mma.cu).

The byte-split u8 tensor-core MAC must give the same residues as the CPU
oracle's orc_bsgs_mac and as the CUDA-core mac_kernel on every shape the
reference's hoisted_mac_sum can hand it (llama3fhe/operators/linear/
operator.py:320-330, operators/transform.py:108-116): batches that span
several 8-ciphertext column groups, baby counts that are not multiples of the
64-baby stage, more than 8 giants (several launches), 50/60/61-bit primes, the
extended basis Q u P, and residues at the top of their range, where the exact
128-bit bound of the byte sums is met with equality in bits; one past that
bound the call must take the CUDA-core kernel and stay exact."""

from __future__ import annotations

import numpy as np
import pytest

from _ckks import N, pair, rand_residues, to_dev, to_host

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True, scope="module")
def _release_cached_blocks():
    """These tests hold several GB of torch-allocated operands; hand the
    cached blocks back so later tests' own allocations (the library's stream
    -ordered pool) find the memory."""

    yield
    import gc

    import torch

    gc.collect()
    torch.cuda.empty_cache()


@pytest.mark.parametrize("bits,C,B,G,l", [
    (60, 7, 37, 5, 1),    # ragged: fewer than 64 babies, 8 giants, 8 ciphertexts
    (60, 9, 70, 9, 1),    # three column groups, three baby stages, 8 giants on the
                          # tensor cores and the ninth on the CUDA cores
    (50, 2, 130, 4, 2),   # binary64-path primes, five baby stages
    (61, 3, 64, 4, 1),    # 61-bit primes at the 128-bit bound
    (60, 2, 16, 4, 1),    # the smallest shape the tensor cores take
    (60, 2, 1, 1, 1),     # one baby, one giant: the CUDA-core kernel
    (60, 1, 40, 3, 1),    # one ciphertext: the CUDA-core kernel
])
def test_mac_mma_matches_oracle(bits, C, B, G, l):
    ctx, orc = pair(4, 1, 2, bits)
    ctx.set_mac_path("auto")
    rng = np.random.default_rng(1000 + bits + C + B + G)
    babies = rand_residues(rng, ctx.primes[:l], C * B * 2).reshape(C, B, 2, l, N)
    pts = rand_residues(rng, ctx.primes[:l], G * B)
    got = to_host(ctx.mac(to_dev(babies.reshape(C * B, 2, l, N)), B, to_dev(pts), G, l,
                          num_cts=C))
    want = orc.bsgs_mac(babies, C, B, pts, G, l)
    assert np.array_equal(got, want)


def test_mac_mma_extended_basis_matches_oracle():
    """mac_ext over Q_2 u P (limb 2.. reduce modulo the special primes)."""

    ctx, orc = pair(4, 2, 2, 60)
    ctx.set_mac_path("auto")
    ql, K, C, B, G = 2, ctx.K, 3, 20, 4
    primes = ctx.primes[:ql] + ctx.primes[4:4 + K]
    rng = np.random.default_rng(77)
    babies = rand_residues(rng, primes, C * B * 2).reshape(C, B, 2, ql + K, N)
    pts = rand_residues(rng, primes, G * B)
    got = to_host(ctx.mac_ext(to_dev(babies.reshape(C * B, 2, ql + K, N)), B, to_dev(pts),
                              G, ql, num_cts=C))
    want = orc.bsgs_mac(babies, C, B, pts, G, ql, p_limbs=K)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("bits,B,kernel", [
    (61, 64, "mac_mma_kernel"),   # 64 (q-1)^2 < 2^128: tensor cores
    (60, 256, "mac_mma_kernel"),  # 256 (q-1)^2 < 2^128: tensor cores
    (61, 65, "mac_kernel"),       # past the bound: CUDA cores
])
def test_mac_extreme_residues_and_bound(bits, B, kernel):
    """Every residue q - 1: each sum is B (q-1)^2 = B mod q, the largest
    byte sums the path can see; the kernel the call takes is the one the
    bound selects."""

    import torch

    ctx, _ = pair(4, 1, 2, bits)
    ctx.set_mac_path("auto")
    C, G, l = 3, 4, 2
    q = np.array(ctx.primes[:l], dtype=np.uint64)
    top = torch.tensor([int(v) - 1 for v in q], dtype=torch.int64, device="cuda:0")
    db = top[None, None, :, None].expand(C * B, 2, l, N).contiguous()
    dp = top[None, :, None].expand(G * B, l, N).contiguous()
    assert ctx.mac_kernel(B, l, num_cts=C, giant_count=G) == kernel
    got = to_host(ctx.mac(db, B, dp, G, l, num_cts=C))
    want = np.broadcast_to((np.uint64(B) % q)[None, None, None, :, None], got.shape)
    assert np.array_equal(got, want)


def test_mac_mma_matches_cuda_cores_at_linear_block_shape():
    """The linear block's chunk (16 ciphertexts x 64 babies x 8 giants) at
    60-bit primes: tensor-core and CUDA-core kernels bit-identical, each path
    taking its own kernel."""

    import torch

    ctx, _ = pair(4, 1, 2, 60)
    C, B, G, l = 16, 64, 8, 3
    gen = torch.Generator(device="cuda:0").manual_seed(5)
    q = torch.tensor(ctx.primes[:l], dtype=torch.int64, device="cuda:0")

    def residues(polys):
        r = torch.randint(0, 1 << 62, (polys, l, N), generator=gen, device="cuda:0",
                          dtype=torch.int64)
        return (r % q[None, :, None]).contiguous()

    babies, pts = residues(C * B * 2), residues(G * B)
    outs = {}
    for path in ("cuda_cores", "auto"):
        ctx.set_mac_path(path)
        want = "mac_mma_kernel" if path == "auto" else "mac_kernel"
        assert ctx.mac_kernel(B, l, num_cts=C, giant_count=G) == want
        outs[path] = ctx.mac(babies, B, pts, G, l, num_cts=C)
    ctx.set_mac_path("auto")
    assert torch.equal(outs["auto"], outs["cuda_cores"])


def test_sparse_tiles_take_cuda_cores():
    """Auto routes a MAC to the tensor cores only where its tiles are full
    enough: two or more ciphertexts (of 4 columns pairs), 16 or more babies
    (of a 32-baby step), 4 or more giants in the launch (of 8); the
    bootstrap's transforms (4-8 babies, 4 giants) stay on the CUDA cores."""

    ctx, _ = pair(4, 1, 2, 60)
    ctx.set_mac_path("auto")
    assert ctx.mac_kernel(64, 3, num_cts=1) == "mac_kernel"
    assert ctx.mac_kernel(64, 3, num_cts=2) == "mac_mma_kernel"
    assert ctx.mac_kernel(8, 3, num_cts=16, giant_count=4) == "mac_kernel"
    assert ctx.mac_kernel(16, 3, num_cts=16, giant_count=4) == "mac_mma_kernel"
    assert ctx.mac_kernel(64, 3, num_cts=16, giant_count=3) == "mac_kernel"
    ctx.set_mac_path("cuda_cores")
    assert ctx.mac_kernel(64, 3, num_cts=16) == "mac_kernel"
    ctx.set_mac_path("auto")


def test_tensor_core_mac_waits_never_time_out():
    """Every stage the tensor-core MAC waited for in this process arrived (its
    bounded TMA waits count a timeout instead of hanging)."""

    from easyfhe import _native

    ctx, _ = pair(4, 1, 2, 60)
    ctx.set_mac_path("auto")
    C, B, G, l = 5, 40, 4, 2
    assert ctx.mac_kernel(B, l, num_cts=C, giant_count=G) == "mac_mma_kernel"
    rng = np.random.default_rng(9)
    babies = rand_residues(rng, ctx.primes[:l], C * B * 2)
    pts = rand_residues(rng, ctx.primes[:l], G * B)
    ctx.mac(to_dev(babies), B, to_dev(pts), G, l, num_cts=C)
    import torch

    torch.cuda.synchronize()
    assert _native.lib.b2f_mac_wait_errors() == 0


def test_set_mac_path_rejects_unknown():
    ctx, _ = pair(4, 1, 2, 60)
    with pytest.raises(ValueError):
        ctx.set_mac_path("tensor")
