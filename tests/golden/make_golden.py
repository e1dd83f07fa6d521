"""Generate golden fixtures from the reference's own NumPy code.

Run in a container that has the reference tree (it is not needed on the GPU
box; the fixtures it writes are committed):

    python tests/golden/make_golden.py [/path/to/reference]

The reference package ``llama3fhe`` imports the external EasyFHE at module
load.  EasyFHE is not available, so a stub module named ``easyfhe`` is put in
``sys.modules`` first.  Nothing from the stub is used by the functions called
here: they are pure NumPy (``_cpu_packer``, ``LinearPlan``,
``linear_rotations``, ``FeatureMajorPrefillLayout``,
``StructuredLinearWeight.materialize``).

Fixtures written next to this script:
  linear_plans.json     LinearPlan geometry and evaluation-key unions for the
                        production schedule (llama3fhe/operators/linear/
                        config.py:163-317) at the four Llama-3 linear shapes.
  packer_small.npz      diagonal rows from ``_cpu_packer``
                        (llama3fhe/operators/linear/weight.py:18-47) for a
                        small plan, the input carrier, the BSGS result under
                        left rotations and the direct mat-vec it must equal.
  packer_structured.npz a StructuredLinearWeight and the rows the reference's
                        structured GPU packer computes
                        (llama3fhe/operators/linear/gpu_packer.py:346-424),
                        restated in NumPy in the kernel's operation order.
  layout_fm.npz         FeatureMajorPrefillLayout.pack for a small shape
                        (llama3fhe/layouts/feature_major.py:17-92).
"""

from __future__ import annotations

import json
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def _install_stub() -> None:
    stub = types.ModuleType("easyfhe")
    stub.fhe = types.ModuleType("easyfhe.fhe")
    stub.bs = types.ModuleType("easyfhe.bs")
    stub.bs.openfhe = types.ModuleType("easyfhe.bs.openfhe")
    sys.modules["easyfhe"] = stub
    sys.modules["easyfhe.fhe"] = stub.fhe
    sys.modules["easyfhe.bs"] = stub.bs
    sys.modules["easyfhe.bs.openfhe"] = stub.bs.openfhe


def _bsgs_left_rotation(x: np.ndarray, rows: np.ndarray, plan, chunks) -> np.ndarray:
    """sum_chunk rot_{base*G}( sum_g rot_{g*G}( sum_b row[g,b] * rot_{b*T}(x) ) ),
    rot_r(v)[s] = v[(s + r) mod n] (left rotation), as the linear operator
    composes hoisted_mac_sum with the chunk alignment rotation
    (llama3fhe/operators/linear/operator.py:320-351)."""

    out = np.zeros_like(x, dtype=np.complex128)
    row = 0
    for chunk in chunks:
        acc = np.zeros_like(out)
        for g in range(chunk.giant_count):
            inner = np.zeros_like(out)
            for b in range(plan.baby_steps):
                inner += rows[row] * np.roll(x, -plan.baby_offsets[b])
                row += 1
            acc += np.roll(inner, -g * plan.giant_offset)
        out += np.roll(acc, -chunk.giant_base * plan.giant_offset)
    return out


def main(reference: Path) -> None:
    _install_stub()
    sys.path.insert(0, str(reference))
    from llama3fhe.layouts import FeatureMajorPrefillLayout
    from llama3fhe.operators.linear.config import (
        LLAMA3_LINEAR_SCHEDULES,
        LinearOperatorConfig,
        linear_rotations,
    )
    from llama3fhe.operators.linear.structured_weight import (
        structured_linear_weight,
    )
    from llama3fhe.operators.linear.weight import _cpu_packer

    # ---- production plans -------------------------------------------------
    plans = {}
    cfg = LLAMA3_LINEAR_SCHEDULES.qkv
    for name, dim, lanes in (("fm4096", 4096, 8), ("fm2048", 2048, 16), ("fm1024", 1024, 32)):
        plan = cfg.plan(dimension=dim, token_lanes=lanes)
        plans[name] = {
            "dimension": dim,
            "token_lanes": lanes,
            "baby_steps": plan.baby_steps,
            "baby_offsets": list(plan.baby_offsets),
            "giant_offset": plan.giant_offset,
            "chunks": [[c.index, c.giant_base, c.giant_count] for c in plan.chunks],
            "baby_key_offsets": list(plan.baby_key_offsets),
            "rotations": list(
                linear_rotations(
                    dimension=dim,
                    token_lanes=lanes,
                    slots=32768,
                    include_conjugation=True,
                    operator_config=cfg,
                )
            ),
        }
    (HERE / "linear_plans.json").write_text(json.dumps(plans, indent=1) + "\n")

    # ---- small dense packer ------------------------------------------------
    rng = np.random.default_rng(20240611)
    dim, lanes, slots = 16, 4, 64
    small_cfg = LinearOperatorConfig(baby_steps=4, baby_anchor_step=4, max_plaintext_rows=8)
    plan = small_cfg.plan(dimension=dim, token_lanes=lanes)
    weight = rng.normal(0.0, 1.0, (dim, dim))
    ctx = types.SimpleNamespace(
        tensor=types.SimpleNamespace(from_numpy=lambda a: np.array(a)), device="cpu"
    )
    rows = np.concatenate(
        [
            _cpu_packer(weight, plan=plan, chunk=c, slots=slots, dtype=np.float64,
                        crypto_context=ctx)
            for c in plan.chunks
        ]
    )
    tokens = rng.normal(0.0, 1.0, (lanes, dim))
    x = np.zeros(slots)
    for f in range(dim):
        for t in range(lanes):
            x[f * lanes + t] = tokens[t, f]
    bsgs = _bsgs_left_rotation(x, rows, plan, plan.chunks)
    direct = np.zeros(slots)
    y = tokens @ weight.T
    for f in range(dim):
        for t in range(lanes):
            direct[f * lanes + t] = y[t, f]
    assert np.max(np.abs(bsgs.real - direct)) < 1e-9, "BSGS identity failed"
    np.savez(
        HERE / "packer_small.npz",
        weight=weight,
        rows=rows,
        x=x,
        bsgs=bsgs.real,
        direct=direct,
        meta=np.array([dim, lanes, slots, plan.baby_steps, plan.giant_offset,
                       small_cfg.max_plaintext_rows]),
        chunks=np.array([[c.index, c.giant_base, c.giant_count] for c in plan.chunks]),
        baby_offsets=np.array(plan.baby_offsets),
    )

    # ---- structured packer (the reference GPU kernel's arithmetic) --------
    dim, lanes, slots = 16, 4, 64
    src0 = rng.normal(0, 1, (12, 20))
    src1 = rng.normal(0, 1, (9, 20))
    real_source = rng.integers(-1, 2, dim)
    real_row = np.where(real_source == 0, rng.integers(0, 12, dim),
                        np.where(real_source == 1, rng.integers(0, 9, dim), -1))
    imag_source = rng.integers(-1, 2, dim)
    imag_row = np.where(imag_source == 0, rng.integers(0, 12, dim),
                        np.where(imag_source == 1, rng.integers(0, 9, dim), -1))
    column = rng.permutation(20)[:dim].copy()
    column[3] = -1
    sw = structured_linear_weight(
        (src0, src1), dimension=dim, real_source=real_source, real_row=real_row,
        real_scale=rng.normal(0, 1, dim), imag_source=imag_source, imag_row=imag_row,
        imag_scale=rng.normal(0, 1, dim), column=column,
        column_scale=rng.normal(0, 1, dim),
    )
    sources = (src0, src1)
    srows = []
    for c in plan.chunks:
        for gr in range(c.giant_count):
            g = c.giant_base + gr
            for b in range(plan.baby_steps):
                feat = np.arange(slots) // lanes
                of = (feat - g * plan.baby_steps) % dim
                inf = (feat + b) % dim
                col = sw.column[inf]
                valid = col >= 0
                re = np.zeros(slots)
                im = np.zeros(slots)
                for si, s in enumerate(sources):
                    m = valid & (sw.real_source[of] == si)
                    re[m] += s[sw.real_row[of][m], col[m]]
                    m = valid & (sw.imag_source[of] == si)
                    im[m] += s[sw.imag_row[of][m], col[m]]
                re = re * (sw.real_scale[of] * sw.column_scale[inf])
                im = im * (sw.imag_scale[of] * sw.column_scale[inf])
                srows.append(re + 1j * im)
    srows = np.array(srows)
    dense = sw.materialize(dtype=np.complex128)
    drows = np.concatenate(
        [
            _cpu_packer(dense, plan=plan, chunk=c, slots=slots, dtype=np.complex128,
                        crypto_context=ctx)
            for c in plan.chunks
        ]
    )
    assert np.max(np.abs(drows - srows)) < 1e-12, "structured packer restatement"
    np.savez(
        HERE / "packer_structured.npz",
        src0=src0, src1=src1,
        real_source=sw.real_source, real_row=sw.real_row, real_scale=sw.real_scale,
        imag_source=sw.imag_source, imag_row=sw.imag_row, imag_scale=sw.imag_scale,
        column=sw.column, column_scale=sw.column_scale,
        rows=srows,
        meta=np.array([dim, lanes, slots, plan.baby_steps, small_cfg.max_plaintext_rows]),
        chunks=np.array([[c.index, c.giant_base, c.giant_count] for c in plan.chunks]),
    )

    # ---- feature-major layout ----------------------------------------------
    layout = FeatureMajorPrefillLayout(seq_len=24, hidden_dim=16, slots=64)
    hidden = rng.normal(0, 1, (24, 16))
    packed = np.asarray(layout.pack(hidden, dtype=np.float64))
    np.savez(HERE / "layout_fm.npz", hidden=hidden, packed=packed)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <reference checkout>")
    main(Path(sys.argv[1]))
