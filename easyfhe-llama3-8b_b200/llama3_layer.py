"""Encrypted Llama-3-8B Layer-0 through the reference's own ``llama3fhe``,
unchanged, on this backend.

The reference's entry point ``run_layer0.py`` calls
``llama3fhe.application.runner.main(layer0_preset=True)`` (``runner.py:778-786``),
whose ``run(args)`` (``runner.py:128-775``) creates the context and keys,
encrypts the seeded synthetic hidden state (``application/inputs.py:80-113``),
prepares the bootstrap program and evaluates one decoder layer through
``graph.evaluate`` (``graph.py:545``).  Every ciphertext operation it issues
goes through ``import easyfhe`` -- the package in this directory -- so the
whole layer runs in libb200fhe's CUDA kernels.  Nothing of the reference is
edited or copied: it is imported from its installed tree (``baseline/_ref``
beside this repository, or the directory named by ``LLAMA3FHE_ROOT``), with
this directory ahead of it on ``sys.path``.

The decrypted layer output is compared with two fp64 restatements of the same
layer (causal GQA attention with RoPE, SwiGLU MLP, RMSNorm with the gammas the
encrypted graph applies):

* ``exact``: exact RMSNorm, SiLU and softmax -- the model's mathematics;
* ``poly``:  the layer's own RMSNorm and SiLU Chebyshev approximations
  (evaluated in fp64) with exact softmax, which is what the encrypted graph
  approximates apart from its polynomial softmax and CKKS noise.
"""

from __future__ import annotations

import os
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent


def reference_root() -> Path | None:
    """Directory holding the reference's ``llama3fhe`` package and ``assets``."""

    for cand in (os.environ.get("LLAMA3FHE_ROOT"), REPO / "baseline" / "_ref"):
        if cand and (Path(cand) / "llama3fhe" / "__init__.py").is_file() \
                and (Path(cand) / "assets" / "feature_major.json").is_file():
            return Path(cand)
    return None


def import_reference():
    """Import the reference's ``llama3fhe`` with this backend as its ``easyfhe``.

    Raises ImportError when the reference tree is not installed."""

    root = reference_root()
    if root is None:
        raise ImportError("the reference llama3fhe tree is not installed "
                          "(baseline/_ref or LLAMA3FHE_ROOT)")
    for p in (str(root), str(HERE)):  # HERE ends up first
        if p in sys.path:
            sys.path.remove(p)
        sys.path.insert(0, p)
    import easyfhe
    import llama3fhe

    if Path(easyfhe.__file__).resolve().parent != HERE / "easyfhe":
        raise ImportError(f"easyfhe resolves to {easyfhe.__file__}, not this backend")
    return llama3fhe


# ---------------------------------------------------------------------------
# fp64 restatements of the layer
# ---------------------------------------------------------------------------


def chebyshev_fp64(x: np.ndarray, coefficients, a: float, b: float) -> np.ndarray:
    """sum_k' c_k T_k(y), y = (2x - a - b)/(b - a), with the first term halved
    (the convention of llama3fhe/approx/chebyshev.py:136-163), in fp64."""

    c = np.array(coefficients, dtype=np.float64)
    c[0] *= 0.5
    y = (2.0 * np.asarray(x, dtype=np.float64) - (a + b)) / (b - a)
    return np.polynomial.chebyshev.chebval(y, c)


def _rope(values: np.ndarray, heads: int, head_dim: int, theta: float) -> np.ndarray:
    """Rotate-half RoPE over each head, angles pos * theta^(-2i/d) for the
    first half repeated over the second (llama3fhe/approx/attention.py:23-59)."""

    seq = values.shape[0]
    inv = theta ** (-np.arange(0, head_dim, 2, dtype=np.float64) / head_dim)
    ang = np.outer(np.arange(seq, dtype=np.float64), inv)
    cos, sin = np.cos(ang)[:, None, :], np.sin(ang)[:, None, :]
    h = values.reshape(seq, heads, head_dim)
    half = head_dim // 2
    first, second = h[..., :half], h[..., half:]
    out = np.concatenate([first * cos - second * sin, second * cos + first * sin], axis=-1)
    return out.reshape(seq, heads * head_dim)


def layer_fp64(hidden, weights, *, query_heads: int = 32, kv_heads: int = 8,
               head_dim: int = 128, rope_theta: float = 500000.0, eps: float = 1e-5,
               approximations=None) -> np.ndarray:
    """One Llama-3 decoder layer in fp64.  With ``approximations`` (the
    layer's LayerApproximations) RMSNorm's rsqrt and SiLU are its Chebyshev
    series; softmax is always exact."""

    f64 = lambda a: np.asarray(a, dtype=np.float64)  # noqa: E731
    x = f64(hidden)

    def rmsnorm(v, gamma, entry):
        ms = np.mean(v * v, axis=-1, keepdims=True)
        if entry is None:
            scale = 1.0 / np.sqrt(ms + eps)
        else:  # the fitted target is rsqrt(ms + eps) (approx/rmsnorm.py:36-37)
            lo, hi = (float(t) for t in entry["fit_interval"])
            scale = chebyshev_fp64(ms, entry["coefficients"], lo, hi)
        return v * scale * f64(gamma)[None, :]

    def silu(v, entry):
        if entry is None:
            return v / (1.0 + np.exp(-v))
        lo, hi = (float(t) for t in entry["fit_interval"])
        return chebyshev_fp64(v, entry["coefficients"], lo, hi)

    ap = approximations
    h1 = rmsnorm(x, weights.input_layernorm, None if ap is None else ap.input_norm)
    q = _rope(h1 @ f64(weights.q_proj).T, query_heads, head_dim, rope_theta)
    k = _rope(h1 @ f64(weights.k_proj).T, kv_heads, head_dim, rope_theta)
    v = h1 @ f64(weights.v_proj).T
    seq = x.shape[0]
    qh = q.reshape(seq, query_heads, head_dim)
    rep = query_heads // kv_heads
    kh = k.reshape(seq, kv_heads, head_dim)[:, np.arange(query_heads) // rep]
    vh = v.reshape(seq, kv_heads, head_dim)[:, np.arange(query_heads) // rep]
    scores = np.einsum("qhd,khd->hqk", qh, kh) / np.sqrt(head_dim)
    mask = np.tril(np.ones((seq, seq), dtype=bool))
    scores = np.where(mask[None], scores, -np.inf)
    scores -= scores.max(axis=-1, keepdims=True)
    p = np.exp(scores)
    p /= p.sum(axis=-1, keepdims=True)
    attn = np.einsum("hqk,khd->qhd", p, vh).reshape(seq, -1)
    x2 = x + attn @ f64(weights.o_proj).T
    h2 = rmsnorm(x2, weights.post_attention_layernorm,
                 None if ap is None else ap.post_attention_norm)
    act = silu(h2 @ f64(weights.gate_proj).T, None if ap is None else ap.silu)
    return x2 + (act * (h2 @ f64(weights.up_proj).T)) @ f64(weights.down_proj).T


def diff_stats(got: np.ndarray, want: np.ndarray) -> dict:
    d = np.abs(np.asarray(got, np.float64) - np.asarray(want, np.float64))
    ref = float(np.max(np.abs(want)))
    return {"max_abs": float(d.max()), "mean_abs": float(d.mean()),
            "max_rel": float(d.max() / ref) if ref else float("inf"),
            "ref_max_abs": ref}


def synthetic_layer(seed: int = 26081461):
    """The reference's seeded Layer-0 inputs and first-layer approximations."""

    import_reference()
    from llama3fhe.application import args as ref_args
    from llama3fhe.application.approx_config import ApproximationConfig
    from llama3fhe.application.inputs import _synthetic_inputs
    from llama3fhe.layouts import AttentionPairLayout, FeatureMajorPrefillLayout

    hidden, weights = _synthetic_inputs(int(seed), layout=FeatureMajorPrefillLayout(),
                                        attention_layout=AttentionPairLayout())
    approx = ApproximationConfig(rmsnorm_path=ref_args.DEFAULT_RMS,
                                 silu_path=ref_args.DEFAULT_SILU,
                                 softmax_path=ref_args.DEFAULT_SOFTMAX).for_layer(0)
    return hidden, weights, approx


class ReferenceSession:
    """The reference's Layer-0 preset resolved as its runner resolves it
    (``runner.py:128-176``): CKKS config, frozen schedule, layouts, and the
    context with every rotation key the layer declares
    (``session._create_context``, ``session.py:24-53``), for driving single
    reference operators on this backend."""

    def __init__(self, extra_args=()):
        import_reference()
        from llama3fhe import Llama3CKKSConfig
        from llama3fhe.application import args as ref_args
        from llama3fhe.application import session, settings
        from llama3fhe.layouts import AttentionPairLayout, FeatureMajorPrefillLayout
        from llama3fhe.model import Llama3Model

        args = ref_args.resolve_poly_paths(
            ref_args.build_parser(layer0_preset=True).parse_args(list(extra_args)))
        self.config = Llama3CKKSConfig.from_json(args.config)
        resolved = settings.resolve_settings(args, self.config)
        self.schedule = settings.layer_schedule(args, resolved)
        self.feature_layout = FeatureMajorPrefillLayout()
        self.attention_layout = AttentionPairLayout()
        model = Llama3Model(config=self.config, num_layers=1,
                            feature_layout=self.feature_layout,
                            attention_layout=self.attention_layout)
        self.rotations = model.required_rotations(
            self.schedule, bootstrap_deep_level_budget=(
                (3, 3) if self.schedule.softmax_main_deep_bootstrap else None))
        self.context = session._create_context(self.config, self.rotations)

    def encrypt(self, values: np.ndarray, cur_limbs: int) -> tuple:
        """Pack [128, 4096] values feature-major and encrypt them at cur_limbs
        (``session._encrypt_hidden``, ``session.py:56-85``)."""

        from llama3fhe.application import session

        return session._encrypt_hidden(np.asarray(values), context=self.context,
                                       layout=self.feature_layout,
                                       input_level=int(self.context.context.L) - int(cur_limbs))


# ---------------------------------------------------------------------------
# the encrypted run
# ---------------------------------------------------------------------------


def run_layer0(*, warmup: int = 1, repetitions: int = 1, seed: int = 26081461,
               extra_args=(), check: bool = True) -> dict:
    """Run ``runner.run`` of the reference's Layer-0 preset on this backend and
    return ``{"payload": <the reference's report>, "decoded": hidden [128, 4096],
    "checks": {...}, "s_per_layer": ...}``."""

    import_reference()
    from llama3fhe.application import runner

    from easyfhe import fhe

    with tempfile.TemporaryDirectory() as tmp:
        out = Path(tmp) / "hidden.npy"
        argv = ["--weights-source", "synthetic", "--seed", str(int(seed)),
                "--warmup", str(int(warmup)), "--repetitions", str(int(repetitions)),
                "--output-hidden-npy", str(out), *map(str, extra_args)]
        args = runner.build_parser(layer0_preset=True).parse_args(argv)
        t0 = time.perf_counter()
        payload = runner.run(args)
        total = time.perf_counter() - t0
        decoded = np.load(out)
    perf = payload["performance"]
    result = {"payload": payload, "decoded": decoded, "run_seconds": total,
              "s_per_layer": float(perf["median_wall_seconds"]) / int(payload["num_layers"]),
              "pack_stats": dict(fhe.PACK_STATS)}
    if check:
        hidden, weights, approx = synthetic_layer(seed)
        result["checks"] = {
            "vs_fp64_exact": diff_stats(decoded, layer_fp64(hidden, weights)),
            "vs_fp64_poly": diff_stats(decoded, layer_fp64(hidden, weights,
                                                           approximations=approx)),
        }
    return result


if __name__ == "__main__":
    import json

    r = run_layer0()
    print(json.dumps({"s_per_layer": r["s_per_layer"], "checks": r.get("checks"),
                      "pack_stats": r["pack_stats"],
                      "performance": {k: v for k, v in r["payload"]["performance"].items()
                                      if k != "samples"}}, indent=1, default=str))
