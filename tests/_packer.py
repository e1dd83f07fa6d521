"""NumPy restatement of the reference's diagonal packers, used as the checker
for the CUDA packers.  It is pinned to the reference by the golden fixtures
generated from the reference's own ``_cpu_packer`` (tests/golden/)."""

from __future__ import annotations

import numpy as np


def pack_dense(weight: np.ndarray, *, dimension: int, token_lanes: int, baby_steps: int,
               giant_base: int, giant_count: int, slots: int) -> np.ndarray:
    """row(g,b)[s] = W[(f - g B) mod D, (f + b) mod D], f = s // lanes
    (llama3fhe/operators/linear/weight.py:18-47)."""

    feat = np.arange(slots) // token_lanes
    rows = []
    for gr in range(giant_count):
        g = giant_base + gr
        of = (feat - g * baby_steps) % dimension
        for b in range(baby_steps):
            rows.append(weight[of, (feat + b) % dimension])
    return np.array(rows)


def pack_structured(sources, maps: dict, *, dimension: int, token_lanes: int,
                    baby_steps: int, giant_base: int, giant_count: int,
                    slots: int) -> np.ndarray:
    """The structured GPU packer's arithmetic
    (llama3fhe/operators/linear/gpu_packer.py:346-424): selected source
    values summed, then times (row_scale * column_scale)."""

    feat = np.arange(slots) // token_lanes
    rows = []
    for gr in range(giant_count):
        g = giant_base + gr
        of = (feat - g * baby_steps) % dimension
        for b in range(baby_steps):
            inf = (feat + b) % dimension
            col = maps["column"][inf]
            valid = col >= 0
            re = np.zeros(slots)
            im = np.zeros(slots)
            for si, s in enumerate(sources):
                m = valid & (maps["real_source"][of] == si)
                re[m] += s[maps["real_row"][of][m], col[m]]
                m = valid & (maps["imag_source"][of] == si)
                im[m] += s[maps["imag_row"][of][m], col[m]]
            re = re * (maps["real_scale"][of] * maps["column_scale"][inf])
            im = im * (maps["imag_scale"][of] * maps["column_scale"][inf])
            rows.append(re + 1j * im)
    return np.array(rows)


def bsgs_left(x: np.ndarray, rows: np.ndarray, baby_offsets, giant_offset: int,
              chunks) -> np.ndarray:
    """sum over chunks of rot_{base G}(sum_g rot_{g G}(sum_b row * rot_{b T}(x)))
    with left rotations, the composition of fhe.hoisted_mac_sum and the chunk
    alignment rotation (llama3fhe/operators/linear/operator.py:320-351)."""

    out = np.zeros(x.shape, dtype=np.complex128)
    row = 0
    for _, base, count in chunks:
        acc = np.zeros_like(out)
        for g in range(count):
            inner = np.zeros_like(out)
            for off in baby_offsets:
                inner += rows[row] * np.roll(x, -off)
                row += 1
            acc += np.roll(inner, -g * giant_offset)
        out += np.roll(acc, -base * giant_offset)
    return out
