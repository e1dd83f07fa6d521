"""The reference's ``llama3fhe`` on this backend, the parts that need no GPU.

* it imports, unchanged, with this repository's ``easyfhe`` as its backend;
* its static Layer-0 audit (``graph.operation_audit``, ``graph.py:348-542``,
  which asks this backend's ``bs.requirements`` for the bootstrap keys)
  reproduces the committed golden (``tests/golden/make_layer0_audit.py``) and
  the per-stage rotation counts measured in the reference under a stub;
* the fp64 layer the GPU test decrypts against agrees with the reference's own
  NumPy layer (``approx/layer.py:64-149``) on the seeded Layer-0 inputs;
* the chunk packer closure that ``LinearWeight`` hands to ``UnpackedRaw``
  (``operators/linear/weight.py:50-104, 309-310``) still binds the plan,
  chunk and weight this backend reads to pack on the GPU instead of Triton.

Every test skips when the reference tree is not installed.
"""

from __future__ import annotations

import dataclasses
import json
from pathlib import Path

import numpy as np
import pytest

import llama3_layer

GOLDEN = Path(__file__).resolve().parent / "golden" / "layer0_audit.json"

needs_ref = pytest.mark.skipif(llama3_layer.reference_root() is None,
                               reason="reference llama3fhe tree not installed")


@pytest.fixture(autouse=True)
def _reference_on_path():
    if llama3_layer.reference_root() is not None:
        llama3_layer.import_reference()


@needs_ref
def test_reference_imports_on_this_backend():
    mod = llama3_layer.import_reference()
    import easyfhe
    from easyfhe import fhe

    from llama3fhe import backend

    assert Path(mod.__file__).resolve().is_relative_to(llama3_layer.reference_root().resolve())
    assert backend.easyfhe is easyfhe and backend.fhe is fhe


@needs_ref
def test_layer0_audit_matches_golden():
    import sys

    sys.path.insert(0, str(GOLDEN.parent))
    from make_layer0_audit import audit_payload

    got = json.loads(json.dumps(audit_payload(), sort_keys=True))
    want = json.loads(GOLDEN.read_text())
    assert got == want
    st = got["audit"]["stages"]
    # per-layer rotation counts of the reference, measured under a stub backend
    assert st["feature_major_qkv_to_attention"]["stages"]["carrier_to_attention"][
        "rotations"] == 2390
    assert st["qk"]["rotations"] == 1528
    assert st["softmax"]["rotations"] == 956
    assert st["pv"]["rotations"] == 1572
    assert st["pairfm_output_conversion"]["conversion_rotations"] == 864
    assert st["mlp"]["rotations_including_conjugations"] == 9184
    assert got["rotation_key_count"] == 674


@needs_ref
def test_fp64_layer_matches_reference_numpy_layer():
    from llama3fhe.approx.layer import poly_transformer_layer_numpy
    from llama3fhe.layouts import AttentionPairLayout

    hidden, w, approx = llama3_layer.synthetic_layer()
    # the reference's NumPy layer applies no RMSNorm gammas: compare at gamma = 1
    ones = np.ones(4096, np.float32)
    w1 = dataclasses.replace(w, input_layernorm=ones, post_attention_layernorm=ones)
    ref = poly_transformer_layer_numpy(hidden, weights=w1, approximations=approx,
                                       attention_layout=AttentionPairLayout()).hidden
    mine = llama3_layer.layer_fp64(hidden, w1, approximations=approx)
    d = llama3_layer.diff_stats(mine, ref)
    assert d["max_rel"] < 2e-6, d  # float32 rounding of the reference's layer


@needs_ref
def test_chunk_packer_closure_binds_what_the_cuda_packers_read():
    llama3_layer.import_reference()
    from llama3fhe.operators.linear.config import LinearChunk, LinearPlan
    from llama3fhe.operators.linear.weight import _chunk_packer

    import inspect

    plan = LinearPlan.__new__(LinearPlan)
    chunk = LinearChunk.__new__(LinearChunk)
    fake_ctx = type("Ctx", (), {"max_slots": 32768, "device": "cuda"})()
    pack = _chunk_packer(np.zeros((4, 4), np.float32), plan=plan, chunk=chunk,
                         dtype=np.complex128, crypto_context=fake_ctx,
                         use_gpu_packer=True)
    assert pack.__qualname__ == "_chunk_packer.<locals>.pack"
    assert pack.__module__.endswith("operators.linear.weight")
    nl = inspect.getclosurevars(pack).nonlocals
    assert nl["plan"] is plan and nl["chunk"] is chunk and nl["slots"] == 32768
    for name in ("weight", "structured_device_sources", "structured_device_metadata"):
        assert name in nl
