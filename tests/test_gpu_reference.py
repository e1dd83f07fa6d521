"""The reference's own operators and Layer-0, unchanged, on this backend (GPU).

``llama3fhe`` is imported from its installed tree with this repository's
``easyfhe`` as the backend it calls (``easyfhe-llama3-8b_b200/llama3_layer.py``),
and its code drives every ciphertext operation:

* ``qkv_fhe`` (``operators/linear/qkv.py:144-273``; ``LinearOperator.apply`` at
  the production plan, ``operators/linear/operator.py:195-405``) and
  ``mlp_fhe`` (``operators/linear/mlp.py:524-1126``) decrypt, through their own
  ``verify`` paths, to their NumPy restatements, ``mlp_fhe`` also on one
  rank's shard at 8 GPUs (16 tokens, 2 ciphertexts);
* ``eval_chebyshev_series_cipher`` (``operators/nonlinear/polynomial.py:331-412``)
  at the layer's SiLU degree and at degree 384 matches
  ``eval_chebyshev_series_direct`` (``approx/chebyshev.py:136-163``);
* the Layer-0 preset through ``runner.run`` (``graph.evaluate``) decrypts to the
  fp64 layer within the tolerance below.

The linear weights are packed by the CUDA packers: Triton is never imported.
Skips when the reference tree is not installed.
"""

from __future__ import annotations

import functools
import sys

import numpy as np
import pytest

import llama3_layer

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(llama3_layer.reference_root() is None,
                                 reason="reference llama3fhe tree not installed")]

# decrypted Layer-0 output against the fp64 layer (exact RMSNorm, SiLU and
# softmax): the output's largest magnitude is 0.076; the encrypted graph's
# polynomial softmax and CKKS noise measured 1.6e-4 max-abs on B200
LAYER_MAX_ABS = 1e-3
LAYER_MEAN_ABS = 1e-4


@pytest.fixture(autouse=True)
def _reference_on_path():
    llama3_layer.import_reference()


@functools.lru_cache(maxsize=None)
def _session():
    return llama3_layer.ReferenceSession()


def _no_triton():
    assert "llama3fhe.operators.linear.gpu_packer" not in sys.modules
    assert "triton" not in sys.modules


def test_reference_qkv_decrypts_to_projection():
    from easyfhe import fhe

    from llama3fhe.operators.linear.qkv import qkv_fhe

    s = _session()
    hidden, w, _ = llama3_layer.synthetic_layer()
    x = np.random.default_rng(5).normal(size=hidden.shape).astype(np.float32)  # RMSNorm-like
    before = dict(fhe.PACK_STATS)
    cts = s.encrypt(x, 13)  # the QKV input level of the graph (graph.py:794-990)
    r = qkv_fhe(x, w.q_proj, w.k_proj, w.v_proj, attention_layout=s.attention_layout,
                layout=s.feature_layout, config=s.config, crypto_context=s.context,
                input_ciphers=cts, verify=True)
    q = x.astype(np.float64) @ w.q_proj.T.astype(np.float64)
    assert r.max_abs_diff is not None
    assert r.max_abs_diff < 1e-4 * np.abs(q).max(), (r.max_abs_diff, np.abs(q).max())
    assert fhe.PACK_STATS["structured"] > before["structured"]
    assert fhe.PACK_STATS["foreign"] == before["foreign"]
    _no_triton()


def test_reference_mlp_decrypts_to_swiglu():
    from llama3fhe.operators.linear.mlp import mlp_fhe

    s = _session()
    hidden, w, approx = llama3_layer.synthetic_layer()
    x = np.random.default_rng(6).normal(size=hidden.shape).astype(np.float32)
    cts = s.encrypt(x, 11)  # PS depth + 5 at Layer 0 (graph.py:1252-1259)
    r = mlp_fhe(x, w.gate_proj, w.up_proj, w.down_proj, silu_entry=approx.silu,
                layout=s.feature_layout, config=s.config, crypto_context=s.context,
                input_ciphers=cts, verify=True)
    ref = np.abs(r.expected).max()
    assert r.max_abs_diff < 1e-3 * ref, (r.max_abs_diff, ref)
    _no_triton()


def test_reference_mlp_on_one_rank_shard():
    """One rank's share of the MLP at 8 GPUs: ``mlp_fhe`` unchanged on the
    layout's smallest sharded shape (16 tokens, 2 ciphertexts: one complex
    pair), as ``bench.py --workload mlp`` runs it on every rank."""

    from llama3fhe.application import session
    from llama3fhe.layouts import FeatureMajorPrefillLayout
    from llama3fhe.operators.linear.mlp import mlp_fhe

    s = _session()
    _, w, approx = llama3_layer.synthetic_layer()
    layout = FeatureMajorPrefillLayout(seq_len=16)
    x = np.random.default_rng(8).normal(size=(16, 4096)).astype(np.float32)
    cts = session._encrypt_hidden(x, context=s.context, layout=layout,
                                  input_level=int(s.context.context.L) - 11)
    assert len(cts) == 2
    r = mlp_fhe(x, w.gate_proj, w.up_proj, w.down_proj, silu_entry=approx.silu,
                layout=layout, config=s.config, crypto_context=s.context,
                input_ciphers=cts, verify=True)
    assert len(r.ciphers) == 2
    ref = np.abs(r.expected).max()
    assert r.max_abs_diff < 1e-3 * ref, (r.max_abs_diff, ref)
    _no_triton()


@pytest.mark.parametrize("which", ["silu", "degree384"])
def test_reference_chebyshev_ps_matches_direct(which):
    from llama3fhe.approx.chebyshev import eval_chebyshev_series_direct
    from llama3fhe.operators.nonlinear.polynomial import eval_chebyshev_series_cipher

    s = _session()
    _, _, approx = llama3_layer.synthetic_layer()
    if which == "silu":  # the layer's own SiLU fit (degree 48 at Layer 0)
        entry = approx.silu
        coeffs = np.asarray(entry["coefficients"], np.float64)
        lo, hi = (float(v) for v in entry["fit_interval"])
    else:  # a smooth degree-384 series on [-8, 8]
        lo, hi = -8.0, 8.0
        k = np.arange(385)
        coeffs = np.exp(-k / 40.0) * np.cos(0.3 * k)
    ctx = s.context
    rng = np.random.default_rng(7)
    z = rng.uniform(lo, hi, ctx.max_slots)
    limbs = 20
    ct = ctx.client.encrypt(z, device=str(ctx.context.device), slots=ctx.max_slots,
                            cur_limbs=limbs, scaling_factor=ctx.context.scale_at(limbs))
    out = eval_chebyshev_series_cipher(ct, coeffs, lower_bound=lo, upper_bound=hi,
                                       crypto_context=ctx)
    got = np.asarray(ctx.decrypt(out), np.float64)
    want = eval_chebyshev_series_direct(z, coeffs, lo, hi).astype(np.float64)
    scale = max(1.0, float(np.abs(want).max()))
    assert np.abs(got - want).max() < 1e-5 * scale, (np.abs(got - want).max(), scale)


def test_reference_layer0_decrypts_to_fp64_layer():
    import torch

    from easyfhe import fhe

    torch.cuda.reset_peak_memory_stats()
    before = dict(fhe.PACK_STATS)
    r = llama3_layer.run_layer0(warmup=0, repetitions=1)
    c = r["checks"]["vs_fp64_exact"]
    print(f"layer0: {r['s_per_layer']:.2f} s/layer, max_abs {c['max_abs']:.3e}, "
          f"mean_abs {c['mean_abs']:.3e}, peak {torch.cuda.max_memory_allocated() / 2**30:.1f} GiB")
    assert r["payload"]["finite"]
    assert c["max_abs"] < LAYER_MAX_ABS and c["mean_abs"] < LAYER_MEAN_ABS, c
    assert fhe.PACK_STATS["structured"] > before["structured"]
    assert fhe.PACK_STATS["foreign"] == before["foreign"]
    _no_triton()


def test_reference_model_two_layers_decrypt_to_fp64_stack():
    """Two layers through the reference's own model loop (Llama3Model.forward,
    llama3fhe/model.py:171-364): layer 1 takes the steady-state path (the
    previous output refreshed inside its input RMSNorm) with no decryption in
    between.  The synthetic layers carry gains that keep every RMSNorm input
    inside the reference's per-layer fits (llama3_layer.tune_prefill_gains);
    the decrypted output is compared with the fp64 stack of the same layers
    with their own RMSNorm/SiLU fits (exact softmax)."""

    r = llama3_layer.run_prefill(2)
    c = r["checks"]["vs_fp64_poly"]
    print(f"prefill x2: {r['per_layer_seconds']} s, max_abs {c['max_abs']:.3e} "
          f"of {c['ref_max_abs']:.3e}")
    assert r["finite"] and r["bootstrap_calls"] > 0
    # measured on B200: 1.4e-3 max-abs, 1.2e-4 mean-abs against outputs up to 0.19
    assert c["max_abs"] < 5e-3 and c["mean_abs"] < 5e-4, c
    _no_triton()
