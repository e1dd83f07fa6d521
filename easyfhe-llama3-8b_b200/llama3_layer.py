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


def _rmsnorm64(v, gamma, entry, eps: float = 1e-5):
    ms = np.mean(v * v, axis=-1, keepdims=True)
    if entry is None:
        scale = 1.0 / np.sqrt(ms + eps)
    else:  # the fitted target is rsqrt(ms + eps) (approx/rmsnorm.py:36-37)
        lo, hi = (float(t) for t in entry["fit_interval"])
        scale = chebyshev_fp64(ms, entry["coefficients"], lo, hi)
    return v * scale * np.asarray(gamma, np.float64)[None, :]


def attention_delta_fp64(x, weights, *, query_heads: int = 32, kv_heads: int = 8,
                         head_dim: int = 128, rope_theta: float = 500000.0,
                         approximations=None) -> np.ndarray:
    """The attention block's addition to the residual stream x, in fp64."""

    f64 = lambda a: np.asarray(a, dtype=np.float64)  # noqa: E731
    ap = approximations
    h1 = _rmsnorm64(x, weights.input_layernorm, None if ap is None else ap.input_norm)
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
    return attn @ f64(weights.o_proj).T


def mlp_delta_fp64(x2, weights, *, approximations=None) -> np.ndarray:
    """The SwiGLU MLP block's addition to the residual stream x2, in fp64."""

    f64 = lambda a: np.asarray(a, dtype=np.float64)  # noqa: E731
    ap = approximations
    h2 = _rmsnorm64(x2, weights.post_attention_layernorm,
                    None if ap is None else ap.post_attention_norm)
    g = h2 @ f64(weights.gate_proj).T
    if ap is None:
        act = g / (1.0 + np.exp(-g))
    else:
        lo, hi = (float(t) for t in ap.silu["fit_interval"])
        act = chebyshev_fp64(g, ap.silu["coefficients"], lo, hi)
    return (act * (h2 @ f64(weights.up_proj).T)) @ f64(weights.down_proj).T


def layer_fp64(hidden, weights, *, approximations=None, **kw) -> np.ndarray:
    """One Llama-3 decoder layer in fp64 (causal GQA with rotate-half RoPE,
    SwiGLU, RMSNorm with its gammas).  With ``approximations`` (the layer's
    LayerApproximations) RMSNorm's rsqrt and SiLU are its Chebyshev series;
    softmax is always exact."""

    x = np.asarray(hidden, dtype=np.float64)
    x2 = x + attention_delta_fp64(x, weights, approximations=approximations, **kw)
    return x2 + mlp_delta_fp64(x2, weights, approximations=approximations)


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


GAINS_PATH = HERE / "prefill_gains.json"
_GAIN_STEPS = [2.0 ** (k / 2) for k in range(0, 31)]  # 1 .. 32768, by sqrt(2)
_MARGIN = 1.5


def _gains() -> dict:
    import json

    if GAINS_PATH.is_file():
        return json.loads(GAINS_PATH.read_text())
    return {}


def layer_weights(index: int, seed: int = 26081461, gains: dict | None = None):
    """Seeded synthetic weights of layer `index`: the reference's Layer-0
    preset generator (application/inputs.py:80-113) with seed + index, with
    the two projections that write the residual stream (o_proj, down_proj)
    scaled by the layer's gains (tune_prefill_gains), so that a stack of such
    layers keeps every RMSNorm input inside the reference's per-layer fits."""

    import dataclasses

    import_reference()
    from llama3fhe.application.inputs import _synthetic_inputs
    from llama3fhe.layouts import AttentionPairLayout, FeatureMajorPrefillLayout

    w = _synthetic_inputs(int(seed) + int(index), layout=FeatureMajorPrefillLayout(),
                          attention_layout=AttentionPairLayout())[1]
    g = (_gains() if gains is None else gains).get(str(int(index)))
    if g and int(_gains().get("seed", seed)) == int(seed):
        w = dataclasses.replace(w, o_proj=(w.o_proj * np.float32(g[0])).astype(np.float32),
                                down_proj=(w.down_proj * np.float32(g[1])).astype(np.float32))
    return w


def _ms_range(x: np.ndarray) -> tuple[float, float]:
    ms = np.mean(x * x, axis=-1)
    return float(ms.min()), float(ms.max())


def _violation(x: np.ndarray, entry) -> float:
    """How far the tokens' mean squares are outside [1.5 lo, hi] of a fit
    (log2 ratio; 0 = inside)."""

    lo, hi = (float(t) for t in entry["fit_interval"])
    a, b = _ms_range(x)
    if not (np.isfinite(a) and np.isfinite(b)) or a <= 0:
        return float("inf")
    return max(0.0, np.log2(_MARGIN * lo / a)) + max(0.0, np.log2(b / hi))


def _pick_gain(x: np.ndarray, delta: np.ndarray, entry) -> float:
    """The smallest gain g putting x + g delta inside the fit, else the one
    closest to it."""

    best, best_v = 1.0, float("inf")
    for g in _GAIN_STEPS:
        v = _violation(x + g * delta, entry)
        if v == 0.0:
            return g
        if v < best_v:
            best, best_v = g, v
    return best


def tune_prefill_gains(num_layers: int = 32, seed: int = 26081461, log=print) -> dict:
    """Per-layer gains for layer_weights, found on the CPU with the fp64
    polynomial layer: for layer i, the smallest gain (a power of sqrt(2)) on
    o_proj whose attention output leaves every token's mean square inside the
    layer's post-attention RMSNorm fit (margin 1.5x at both ends), then the
    smallest on down_proj leaving it inside layer i+1's input RMSNorm fit.
    The reference's fits follow the real model's residual stream, whose mean
    square grows ~5000x over the 32 layers; the Layer-0 preset's weights add
    too little to it, and from layer 2 on the stack falls below the fits."""

    import_reference()
    from llama3fhe.application import args as ref_args
    from llama3fhe.application.approx_config import ApproximationConfig
    from llama3fhe.application.inputs import _synthetic_inputs
    from llama3fhe.layouts import AttentionPairLayout, FeatureMajorPrefillLayout

    a = ref_args.resolve_poly_paths(ref_args.build_parser().parse_args([]))
    approx = ApproximationConfig(rmsnorm_path=a.rms_coeffs, silu_path=a.silu_coeffs,
                                 softmax_path=a.softmax_coeffs)
    x = np.asarray(_synthetic_inputs(int(seed), layout=FeatureMajorPrefillLayout(),
                                     attention_layout=AttentionPairLayout())[0], np.float64)
    gains = {"seed": int(seed)}
    for i in range(int(num_layers)):
        ap = approx.for_layer(i)
        if _violation(x, ap.input_norm):
            log(f"layer {i}: input mean squares {_ms_range(x)} outside "
                f"{ap.input_norm['fit_interval']}")
        w = layer_weights(i, seed, gains={})
        d_att = attention_delta_fp64(x, w, approximations=ap)
        go = _pick_gain(x, d_att, ap.post_attention_norm)
        x2 = x + go * d_att
        d_mlp = mlp_delta_fp64(x2, w, approximations=ap)
        nxt = approx.for_layer(i + 1).input_norm if i + 1 < 32 else None
        gd = 1.0 if nxt is None else _pick_gain(x2, d_mlp, nxt)
        x = x2 + gd * d_mlp
        gains[str(i)] = [go, gd]
        log(f"layer {i}: gains o {go:.3g} down {gd:.3g}; output mean squares {_ms_range(x)}")
    return gains


def run_prefill(num_layers: int = 32, *, seed: int = 26081461, check: bool = True,
                progress=None, diagnostic=None) -> dict:
    """An encrypted prefill of `num_layers` decoder layers through the reference's
    own model loop, unchanged, on this backend.

    The reference's runner accepts a multi-layer run only with a checkpoint
    (application/settings.py:89-93: synthetic weights are its one-layer
    preset), so this resolves the settings and schedule a checkpoint run of
    `num_layers` layers resolves (resolve_settings / layer_schedule,
    settings.py:65-231: input at the bootstrap-output level, the pre-exp
    softmax refresh), builds the context with every rotation those layers
    declare, encrypts the preset's seeded hidden state and streams seeded
    synthetic layers (layer_weights) with each layer's own approximations into
    Llama3Model.forward (model.py:171-364): layer 0 consumes the encrypted
    input, every later layer refreshes the previous output inside its input
    RMSNorm, and no boundary is decrypted until the end."""

    import_reference()
    from llama3fhe import Llama3CKKSConfig
    from llama3fhe.application import args as ref_args
    from llama3fhe.application import session, settings
    from llama3fhe.application.approx_config import ApproximationConfig
    from llama3fhe.application.client import decrypt_hidden
    from llama3fhe.application.inputs import _synthetic_inputs
    from llama3fhe.layouts import AttentionPairLayout, FeatureMajorPrefillLayout
    from llama3fhe.model import Llama3Model, TransformerLayer, prepare_bootstrap_operator

    import torch

    n = int(num_layers)
    args = ref_args.resolve_poly_paths(ref_args.build_parser().parse_args(
        ["--num-layers", str(n), "--weights-source", "real"]))
    config = Llama3CKKSConfig.from_json(args.config)
    resolved = settings.resolve_settings(args, config)
    schedule = settings.layer_schedule(args, resolved)
    approx = ApproximationConfig(rmsnorm_path=args.rms_coeffs, silu_path=args.silu_coeffs,
                                 softmax_path=args.softmax_coeffs)
    approx.validate_layers(n)
    fl, al = FeatureMajorPrefillLayout(), AttentionPairLayout()
    model = Llama3Model(config=config, num_layers=n, feature_layout=fl, attention_layout=al)
    t0 = time.perf_counter()
    rotations = model.required_rotations(
        schedule, bootstrap_deep_level_budget=(
            (3, 3) if schedule.softmax_main_deep_bootstrap else None))
    context = session._create_context(config, rotations)
    hidden, _ = _synthetic_inputs(int(seed), layout=fl, attention_layout=al)
    ciphers = session._encrypt_hidden(hidden, context=context, layout=fl,
                                      input_level=resolved.input_level)
    op = prepare_bootstrap_operator(context, schedule)
    setup = time.perf_counter() - t0

    from concurrent.futures import ThreadPoolExecutor

    def layers():
        # the next layer's weights are generated on a background thread while
        # this one runs, as the reference streams checkpoint layers
        # (application/layer_stream.py:23-186)
        with ThreadPoolExecutor(1) as pool:
            nxt = pool.submit(layer_weights, 0, seed)
            for i in range(n):
                w = nxt.result()
                if i + 1 < n:
                    nxt = pool.submit(layer_weights, i + 1, seed)
                yield TransformerLayer(index=i, weights=w,
                                       approximations=approx.for_layer(i), config=config,
                                       feature_layout=fl, attention_layout=al)

    torch.cuda.synchronize()
    t0 = time.perf_counter()
    diag = None
    if diagnostic is not None:  # diagnostic(index, decrypted hidden) after every layer
        def diag(index, cts, layer):
            diagnostic(int(index), decrypt_hidden(cts, crypto_context=context, layout=fl))
            return {}
    result = model.forward(hidden, crypto_context=context, input_ciphers=ciphers,
                           layers=layers(), bootstrap_operator=op, schedule=schedule,
                           progress_callback=progress, diagnostic_callback=diag)
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    decoded = decrypt_hidden(result.ciphers, crypto_context=context, layout=fl)
    out = {"num_layers": n, "wall_seconds": wall, "s_per_layer": wall / n,
           "setup_seconds": setup,
           "per_layer_seconds": [float(r["wall_seconds"]) for r in result.per_layer],
           "bootstrap_calls": int(result.bootstrap_calls),
           "input_level": int(resolved.input_level), "decoded": decoded,
           "finite": bool(np.all(np.isfinite(decoded)))}
    if check:
        exact = poly = np.asarray(hidden, np.float64)
        for i in range(n):
            w = layer_weights(i, seed)
            exact = layer_fp64(exact, w)
            poly = layer_fp64(poly, w, approximations=approx.for_layer(i))
        out["checks"] = {"vs_fp64_exact": diff_stats(decoded, exact),
                         "vs_fp64_poly": diff_stats(decoded, poly)}
    return out


if __name__ == "__main__":
    import json

    if sys.argv[1:2] == ["--tune-gains"]:  # writes prefill_gains.json beside this file
        GAINS_PATH.write_text(json.dumps(tune_prefill_gains(), indent=1) + "\n")
        sys.exit(0)

    r = run_layer0()
    print(json.dumps({"s_per_layer": r["s_per_layer"], "checks": r.get("checks"),
                      "pack_stats": r["pack_stats"],
                      "performance": {k: v for k, v in r["payload"]["performance"].items()
                                      if k != "samples"}}, indent=1, default=str))
