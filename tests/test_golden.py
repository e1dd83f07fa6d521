"""Golden fixtures generated from the reference's own NumPy code
(tests/golden/make_golden.py) pin the packing and BSGS semantics the CUDA path
must reproduce.  Runs on CPU."""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np

from _packer import bsgs_left, pack_dense, pack_structured

G = Path(__file__).resolve().parent / "golden"


def test_dense_packer_restatement_matches_reference_rows():
    d = np.load(G / "packer_small.npz")
    dim, lanes, slots, B, giant_offset, max_rows = (int(v) for v in d["meta"])
    rows = np.concatenate([
        pack_dense(d["weight"], dimension=dim, token_lanes=lanes, baby_steps=B,
                   giant_base=int(base), giant_count=int(cnt), slots=slots)
        for _, base, cnt in d["chunks"]
    ])
    assert np.array_equal(rows, d["rows"])


def test_bsgs_identity_with_left_rotations():
    d = np.load(G / "packer_small.npz")
    dim, lanes, slots, B, giant_offset, _ = (int(v) for v in d["meta"])
    out = bsgs_left(d["x"], d["rows"], d["baby_offsets"], giant_offset, d["chunks"])
    assert np.max(np.abs(out.real - d["bsgs"])) < 1e-12
    assert np.max(np.abs(out.real - d["direct"])) < 1e-9
    assert np.max(np.abs(out.imag)) == 0


def test_structured_packer_restatement_matches_reference():
    d = np.load(G / "packer_structured.npz")
    dim, lanes, slots, B, _ = (int(v) for v in d["meta"])
    maps = {k: d[k] for k in ("real_source", "real_row", "real_scale", "imag_source",
                              "imag_row", "imag_scale", "column", "column_scale")}
    rows = np.concatenate([
        pack_structured((d["src0"], d["src1"]), maps, dimension=dim, token_lanes=lanes,
                        baby_steps=B, giant_base=int(base), giant_count=int(cnt),
                        slots=slots)
        for _, base, cnt in d["chunks"]
    ])
    assert np.array_equal(rows, d["rows"])


def test_production_linear_plans():
    plans = json.loads((G / "linear_plans.json").read_text())
    p = plans["fm4096"]
    assert p["giant_offset"] == 512 and p["baby_steps"] == 64
    assert p["baby_offsets"] == [8 * b for b in range(64)]
    assert [c[2] for c in p["chunks"]] == [8] * 8
    assert 131071 in p["rotations"]  # conjugation key M - 1
    assert 512 in p["rotations"]      # repeated Horner giant key


def test_feature_major_layout_fixture():
    d = np.load(G / "layout_fm.npz")
    hidden, packed = d["hidden"], d["packed"]
    # slot(dim, tok) = dim * tokens_per_cipher + tok, 4 tokens per cipher here
    tpc = 64 // 16
    for c in range(packed.shape[0]):
        for f in range(16):
            for t in range(tpc):
                tok = c * tpc + t
                want = hidden[tok, f] if tok < hidden.shape[0] else 0.0
                assert packed[c][f * tpc + t] == want
