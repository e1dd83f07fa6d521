"""Homomorphic DFT matrices of CKKS bootstrapping (CoeffToSlot / SlotToCoeff).

The CKKS decoder is the special FFT of Cheon-Kim-Kim-Song: bit reversal, then
log2(n) butterfly stages (len = 2, 4, ..., n); the encoder runs the inverse
stages (len = n, ..., 2), bit reversal and a division by n.  As slot-vector
maps each stage is out = sum_o D_o * rot(in, o) with three diagonals at
offsets 0 and +-len/2 (rot(v, o)[s] = v[s + o], the left rotation of
homo_rotate).  CoeffToSlot applies the inverse stages without the final bit
reversal and SlotToCoeff applies the forward stages without the initial bit
reversal, so coefficients sit in bit-reversed slot order in between -- EvalMod
is slot-wise, so the order never matters (Chen-Chillotti-Song 2019).
Consecutive stages are merged into `budget` levels; a level with s stages has
up to 2^(s+1) - 1 diagonals, evaluated by baby-step giant-step.

The twiddles are the encoder's: ksi_k = exp(2 pi i k / M), rotation group
5^j mod M, the same table the CUDA encoder uses.
"""

from __future__ import annotations

import numpy as np


def _tables(log_n: int):
    n = 1 << log_n
    m = 2 * n
    k = np.arange(m + 1, dtype=np.float64)
    ang = 2.0 * np.pi * k / float(m)
    ksi = np.cos(ang) + 1j * np.sin(ang)
    rot = np.empty(n // 2, dtype=np.int64)
    g = 1
    for j in range(n // 2):
        rot[j] = g
        g = (g * 5) % m
    return ksi, rot


def stage(log_n: int, slots: int, length: int, inverse: bool) -> dict[int, np.ndarray]:
    """Diagonals {offset: d} of one butterfly stage on `slots` slots."""

    ksi, rot = _tables(log_n)
    m = 2 << log_n
    lenh = length // 2
    lenq = length << 2
    gap = m // lenq
    s = np.arange(slots)
    j = s % length
    first = j < lenh
    jj = np.where(first, j, j - lenh)
    if inverse:
        w = ksi[((lenq - (rot[jj] % lenq)) * gap)]
        d0 = np.where(first, 1.0 + 0j, -w)
        dp = np.where(first, 1.0 + 0j, 0j)      # in[s + lenh]
        dm = np.where(first, 0j, w)             # in[s - lenh]
    else:
        w = ksi[((rot[jj] % lenq) * gap)]
        d0 = np.where(first, 1.0 + 0j, -w)
        dp = np.where(first, w, 0j)
        dm = np.where(first, 0j, 1.0 + 0j)
    out: dict[int, np.ndarray] = {0: d0}
    for o, d in ((lenh % slots, dp), ((-lenh) % slots, dm)):
        out[o] = out[o] + d if o in out else d  # +-len/2 coincide when len = slots
    return out


def compose(outer: dict[int, np.ndarray], inner: dict[int, np.ndarray],
            slots: int) -> dict[int, np.ndarray]:
    """outer(inner(x)) = sum_{a,b} D_a rot(E_b, a) rot(x, a + b)."""

    out: dict[int, np.ndarray] = {}
    for a, da in outer.items():
        for b, eb in inner.items():
            o = (a + b) % slots
            term = da * np.roll(eb, -a)
            out[o] = out[o] + term if o in out else term
    return {o: d for o, d in out.items() if np.any(d != 0)}


def apply(diags: dict[int, np.ndarray], x: np.ndarray) -> np.ndarray:
    return sum(d * np.roll(x, -o) for o, d in diags.items())


def stage_groups(log_slots: int, budget: int) -> list[int]:
    """Stages per level, as even as possible, larger groups first."""

    base, extra = divmod(log_slots, budget)
    return [base + (1 if i < extra else 0) for i in range(budget)]


def _spread(levels: list, scale: complex) -> list:
    """Multiply the product of `levels` by `scale`, |scale|^(1/levels) on each
    level and the phase on the first.  Each level's diagonals are encoded at
    the scale of one ~2^59 prime, so a factor like alpha / n ~ 2^-22 folded
    into one level would leave its plaintext with ~37 significant bits and
    put ~1e-11 of error into the EvalMod input; spread out, every level
    keeps ~53."""

    mag = abs(scale) ** (1.0 / len(levels))
    out = []
    for i, lv in enumerate(levels):
        f = mag * (scale / abs(scale) if i == 0 else 1.0)
        out.append({o: d * f for o, d in lv.items()})
    return out


def coeff_to_slot_levels(log_n: int, log_slots: int, budget: int,
                         factor: complex = 1.0) -> list[dict[int, np.ndarray]]:
    """Levels in application order: inverse stages len = n .. 2, times
    factor / n spread over the levels (no bit reversal)."""

    slots = 1 << log_slots
    lengths = [slots >> i for i in range(log_slots)]  # n, n/2, ..., 2
    levels, pos = [], 0
    for cnt in stage_groups(log_slots, budget):
        acc = None
        for length in lengths[pos:pos + cnt]:
            st = stage(log_n, slots, length, True)
            acc = st if acc is None else compose(st, acc, slots)
        pos += cnt
        levels.append(acc)
    return _spread(levels, complex(factor) / slots)


def slot_to_coeff_levels(log_n: int, log_slots: int, budget: int,
                         factor: complex = 1.0) -> list[dict[int, np.ndarray]]:
    """Levels in application order: forward stages len = 2 .. n, times
    factor spread over the levels (no bit reversal)."""

    slots = 1 << log_slots
    lengths = [2 << i for i in range(log_slots)]  # 2, 4, ..., n
    levels, pos = [], 0
    for cnt in reversed(stage_groups(log_slots, budget)):
        acc = None
        for length in lengths[pos:pos + cnt]:
            st = stage(log_n, slots, length, False)
            acc = st if acc is None else compose(st, acc, slots)
        pos += cnt
        levels.append(acc)
    return _spread(levels, complex(factor))


def bsgs_split(offsets, slots: int) -> tuple[int, int, list[int], int]:
    """(step, baby count B, giant indices, base giant) for offsets that are
    multiples of a power-of-two step in a symmetric range: offset =
    (g * B + b) * step with b in [0, B) and g from base upwards."""

    signed = sorted(((o + slots // 2) % slots) - slots // 2 for o in offsets)
    nz = [abs(o) for o in signed if o]
    step = min(nz) if nz else 1
    span = (max(signed) - min(signed)) // step + 1
    B = 1
    while B * B < span:
        B *= 2
    gmin = -((-min(signed) // step + B - 1) // B) if min(signed) < 0 else 0
    gmax = max(signed) // step // B
    return step, B, list(range(gmin, gmax + 1)), gmin
