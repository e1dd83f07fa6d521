"""The bootstrapping program's math on clear slot vectors (CPU): the merged
DFT levels reproduce the encoder/decoder of the CPU oracle, the baby-step /
giant-step row layout reproduces each level, and CoeffToSlot -> EvalMod ->
SlotToCoeff recovers the message from a ModRaise output t = Delta u 2^-k +
q_0 I (float64, no encryption)."""

from __future__ import annotations

import math

import numpy as np
import pytest
from numpy.polynomial import chebyshev as cheb


def _bitrev(log: int):
    return np.array([int(format(i, f"0{log}b")[::-1], 2) for i in range(1 << log)])


@pytest.mark.parametrize("log_n,budget", [(8, (3, 3)), (10, (4, 4)), (10, (2, 3))])
def test_dft_levels_match_oracle_fft(oracle_mod, log_n, budget):
    from easyfhe.bs import dft

    slots = 1 << (log_n - 1)
    rng = np.random.default_rng(log_n)
    z = rng.normal(size=slots) + 1j * rng.normal(size=slots)
    re, im = oracle_mod.special_fft(log_n, z.real, z.imag, inverse=True)
    v = (re + 1j * im)[_bitrev(log_n - 1)]
    w = z.copy()
    for lv in dft.coeff_to_slot_levels(log_n, log_n - 1, budget[0]):
        w = dft.apply(lv, w)
    assert np.max(np.abs(w - v)) < 1e-12
    x = v.copy()
    for lv in dft.slot_to_coeff_levels(log_n, log_n - 1, budget[1]):
        x = dft.apply(lv, x)
    assert np.max(np.abs(x - z)) < 1e-9


def _bsgs_apply(rows, plan, x):
    B, step = plan.babies, plan.step
    babies = [np.roll(x, -o) for o in plan.baby_offsets()]
    acc = None
    for gi in range(len(plan.giants) - 1, -1, -1):  # Horner over giants
        inner = sum(rows[gi * B + b] * babies[b] for b in range(B))
        acc = inner if acc is None else np.roll(acc, -B * step) + inner
    return acc


def test_bsgs_rows_reproduce_levels():
    from easyfhe.bs import openfhe as bs

    log_n = 12
    slots = 1 << (log_n - 1)
    cts, stc = bs._level_plans(log_n, log_n - 1, (4, 4))
    rng = np.random.default_rng(3)
    x = rng.normal(size=slots) + 1j * rng.normal(size=slots)
    from easyfhe.bs import dft

    for diags, plan in cts + stc:
        rows = bs.level_rows(diags, plan, slots)
        assert np.max(np.abs(_bsgs_apply(rows, plan, x) - dft.apply(diags, x))) < 1e-9


def test_requirements_cover_every_rotation():
    from easyfhe.bs import openfhe as bs

    spec = bs.BootstrapSpec(15, (4, 4), 19)
    rots = set(bs.requirements((spec,), 16).rotations)
    assert 131071 in rots and spec.depth == 18
    cts, stc = bs._level_plans(16, 15, (4, 4))
    for _, p in cts + stc:
        for o in p.baby_offsets():
            assert o % 32768 == 0 or o % 32768 in rots
        assert p.babies * p.step in rots


def test_bootstrap_pipeline_on_clear_slots(oracle_mod):
    """Clear-value run of bootstrap(): encode t = Delta u 2^-k + q_0 I as the
    slots of the raised ciphertext, apply the program, get u back."""

    from easyfhe.bs import dft
    from easyfhe.bs import openfhe as bs

    log_n = 10
    slots = 1 << (log_n - 1)
    n = 2 * slots
    delta, q0 = 2.0 ** 59, float((1 << 60) - 93)
    k = bs.PRESCALE_BITS
    rng = np.random.default_rng(9)
    u = rng.uniform(-1, 1, slots) + 1j * rng.uniform(-1, 1, slots)
    # message coefficients (scaled by Delta 2^-k) plus q_0 I
    re, im = oracle_mod.special_fft(log_n, u.real, u.imag, inverse=True)
    coef = np.concatenate([re, im]) * delta * 2.0 ** -k
    I = rng.integers(-bs.K_RANGE, bs.K_RANGE + 1, n)
    t = coef + q0 * I
    zr, zi = oracle_mod.special_fft(log_n, t[:slots] / delta, t[slots:] / delta, inverse=False)
    z = zr + 1j * zi  # slots of the raised ciphertext at scale Delta
    alpha = delta / (q0 * 2.0 * (bs.K_RANGE + 1))
    beta = q0 * 2.0 ** k / (2.0 * math.pi * delta)
    w = z
    for lv in dft.coeff_to_slot_levels(log_n, log_n - 1, 4, alpha):
        w = dft.apply(lv, w)
    x_re = (w + np.conj(w)).real
    x_im = (-1j * (w - np.conj(w))).real
    assert np.max(np.abs(np.concatenate([x_re, x_im]))) <= 1.0
    c = cheb.chebinterpolate(
        lambda v: np.cos(2 * np.pi * ((bs.K_RANGE + 1) * v - 0.25) / 2 ** bs.DOUBLINGS),
        bs.CHEB_DEGREE)

    def evalmod(v):
        s = cheb.chebval(v, c)
        for _ in range(bs.DOUBLINGS):
            s = 2 * s * s - 1
        return s

    s = evalmod(x_re) + 1j * evalmod(x_im)
    for lv in dft.slot_to_coeff_levels(log_n, log_n - 1, 4, beta):
        s = dft.apply(lv, s)
    assert np.max(np.abs(s - u)) < 2.0 ** -16
