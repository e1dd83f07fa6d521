"""``easyfhe.bs.openfhe`` -- CKKS bootstrapping on libb200fhe.

The surface the reference calls (llama3fhe/operators/nonlinear/bootstrap.py:
59-85, 113-130, 188, 370): ``BootstrapSpec(log_slots, level_budget,
output_levels, mode)``, ``requirements(specs, log_n).rotations``,
``generate(context, spec)`` returning a program with ``.spec.slots`` and
``.constants.set_cache_mode``, and ``bootstrap(ct, context, program)``.

Algorithm, mode "modraise_first" (Cheon-Han-Kim-Kim-Song 2018 with the
Chen-Chillotti-Song 2019 ordering):

  0. pre-scale: multiply by 2^-k and rescale (the input carries at least two
     limbs), so the message part of t / q_0 is at most 2^-(k+1);
  1. ModRaise: drop to q_0 and lift the coefficients to all L primes:
     t = Delta u 2^-k + q_0 I; a sparse message (n = 2^log_slots < N/2 slots,
     coefficients on Z[X^gap], gap = N / 2n) is then projected back onto
     that subring by SubSum, t <- t + rot_{n 2^i}(t) for i < log2(gap),
     which multiplies it by gap (1/gap is folded into step 2);
  2. CoeffToSlot: the encoder's inverse butterfly stages (len = n .. 2)
     merged into level_budget[0] levels, times Delta / (q_0 2 (K+1)): the slots
     hold (t_j + i t_{j+n}) / (2 q_0 (K+1)) in bit-reversed order;
  3. real / imaginary split with the conjugation key;
  4. EvalMod on both: a degree-63 Chebyshev series of
     cos(2 pi ((K+1) x - 1/4) / 2^3) (depth 7) and three double-angle steps
     (depth 3) give sin(2 pi t / q_0) ~ 2 pi (t / q_0 mod 1);
  5. recombine, then SlotToCoeff: the decoder's butterfly stages (len =
     2 .. n) merged into level_budget[1] levels, times q_0 2^k / (2 pi Delta).

Depth: level_budget[0] + 10 + level_budget[1] levels after ModRaise (18 at
(4, 4)), the "approx(10) + b1 + b2" of llama3fhe/model.py:50-53.  Linear
levels run baby-step / giant-step with hoisted baby rotations
(fhe.prepare_hoisted_baby_rotations + fhe.hoisted_mac_sum); every diagonal
plaintext is encoded at the scale of the prime its level's rescale drops, so
the ciphertext scale is unchanged across the transforms.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np
import torch
from numpy.polynomial import chebyshev as cheb

from .. import fhe
from . import dft

K_RANGE = 28          # |I| bound of the ModRaise overflow (sparse ternary, h = 192)
DOUBLINGS = 3
CHEB_DEGREE = 63
PRESCALE_BITS = 10
EVALMOD_DEPTH = 7 + DOUBLINGS


@dataclass(frozen=True)
class BootstrapSpec:
    log_slots: int
    level_budget: tuple = (4, 4)
    output_levels: int = 0
    mode: str = "modraise_first"

    @property
    def slots(self) -> int:
        return 1 << int(self.log_slots)

    @property
    def depth(self) -> int:
        return int(self.level_budget[0]) + EVALMOD_DEPTH + int(self.level_budget[1])


@dataclass(frozen=True)
class Requirements:
    rotations: tuple


@dataclass(frozen=True)
class _Plan:
    """Offsets (g B + b) step, g in giants (from gmin), b < B.  The babies are
    the hoisted rotations by (gmin B + b) step, so the Horner chain over the
    giants 0 .. G-1 needs no final rotation by gmin B step."""

    step: int
    babies: int
    giants: tuple
    gmin: int

    def baby_offsets(self) -> tuple:
        return tuple((self.gmin * self.babies + b) * self.step for b in range(self.babies))


def _check(spec: BootstrapSpec, log_n: int) -> None:
    if str(spec.mode) != "modraise_first":
        raise NotImplementedError(f"bootstrap mode {spec.mode!r} is not implemented")
    if not 1 <= int(spec.log_slots) <= int(log_n) - 1:
        raise ValueError(f"log_slots {spec.log_slots} outside [1, {int(log_n) - 1}]")
    b1, b2 = (int(v) for v in spec.level_budget)
    if not (1 <= b1 <= spec.log_slots and 1 <= b2 <= spec.log_slots):
        raise ValueError(f"level budget {spec.level_budget} outside [1, log_slots]")


def _level_plans(log_n: int, log_slots: int, budget, alpha=1.0, beta=1.0):
    cts = dft.coeff_to_slot_levels(log_n, log_slots, int(budget[0]), alpha)
    stc = dft.slot_to_coeff_levels(log_n, log_slots, int(budget[1]), beta)
    slots = 1 << log_slots
    out = []
    for diags in cts + stc:
        step, B, giants, gmin = dft.bsgs_split(diags.keys(), slots)
        out.append((diags, _Plan(step, B, tuple(giants), gmin)))
    return out[: len(cts)], out[len(cts):]


def requirements(specs, log_n: int) -> Requirements:
    """Rotation indices every program of `specs` uses (keys to generate)."""

    rots = {(2 << int(log_n)) - 1}  # conjugation, index M - 1
    for spec in specs:
        _check(spec, log_n)
        rots.update(_subsum_rotations(spec, log_n))
        cts, stc = _level_plans(int(log_n), int(spec.log_slots), spec.level_budget)
        slots = 1 << int(spec.log_slots)
        for _, plan in cts + stc:
            rots.update(o % slots for o in plan.baby_offsets() if o % slots)
            if len(plan.giants) > 1:
                rots.add(plan.babies * plan.step)
    return Requirements(tuple(sorted(rots)))


def _gap(spec: BootstrapSpec, log_n: int) -> int:
    """Replication factor of a sparse message: (N/2) / slots."""

    return (1 << (int(log_n) - 1)) // spec.slots


def _subsum_rotations(spec: BootstrapSpec, log_n: int) -> list[int]:
    """Rotations n 2^i (i < log2 gap) of the SubSum of a sparse bootstrap."""

    gap = _gap(spec, log_n)
    return [spec.slots << i for i in range(gap.bit_length() - 1)]


class _Constants:
    """Encoded diagonal plaintexts of a program; they are always kept."""

    def __init__(self, plaintexts):
        self._pts = plaintexts
        self.cache_mode = "plain"

    def set_cache_mode(self, mode: str, clear: bool = False) -> None:
        self.cache_mode = str(mode)

    def clear_cache(self) -> None:
        return None

    def cache_info(self) -> dict:
        total = sum(int(p.data.numel()) * 8 for p in self._pts)
        return {"plain_entries": len(self._pts), "plain_bytes": total, "total_bytes": total}


@dataclass
class _Level:
    plan: _Plan
    pts: fhe.Plaintext
    limbs: int


@dataclass
class Program:
    spec: BootstrapSpec
    cts: list
    stc: list
    cheb: np.ndarray
    constants: _Constants = field(repr=False, default=None)

    def release(self) -> None:
        """Drop the encoded diagonals (BootstrapOperator.release at teardown,
        llama3fhe/operators/nonlinear/bootstrap.py); the program is unusable
        afterwards."""

        for lv in self.cts + self.stc:
            lv.pts = None
        if self.constants is not None:
            self.constants._pts = []


def level_rows(diags: dict, plan: _Plan, slots: int) -> np.ndarray:
    """Row (g - gmin) B + b (g over plan.giants) = D_{(gB+b) step} rotated by
    -(g - gmin) B step: with babies rot_{(gmin B + b) step}(ct), the Horner
    giant rotations put every term back."""

    rows = []
    for g in plan.giants:
        for b in range(plan.babies):
            o = ((g * plan.babies + b) * plan.step) % slots
            d = diags.get(o)
            if d is None:
                d = np.zeros(slots, dtype=np.complex128)
            rows.append(np.roll(d, (g - plan.gmin) * plan.babies * plan.step))
    return np.array(rows)


def _encode_level(ctx: fhe.Context, diags: dict, plan: _Plan, slots: int,
                  limbs: int) -> _Level:
    values = torch.from_numpy(level_rows(diags, plan, slots)).to(ctx.device)
    scale = float(ctx.params.q[limbs - 1])  # the prime this level's rescale drops
    data = ctx.native.encode(values, scale, limbs)
    pt = fhe.Plaintext(data, fhe.CipherState(limbs, 1, scale), slots, False)
    return _Level(plan, pt, limbs)


def generate(context, spec: BootstrapSpec) -> Program:
    """Precompute the CoeffToSlot / SlotToCoeff plaintexts and the EvalMod
    series for `spec` on `context` (llama3fhe/operators/nonlinear/bootstrap.py:113)."""

    ctx = fhe._ctx_of(context)
    _check(spec, ctx.logN)
    L = ctx.L
    out_limbs = L - spec.depth
    if out_limbs < 1:
        raise ValueError(f"depth {spec.depth} of the program exceeds the {L} limbs")
    if int(spec.output_levels) and int(spec.output_levels) + 1 > out_limbs:
        raise ValueError(f"output_levels={spec.output_levels} needs {spec.output_levels + 1} "
                         f"limbs, the program leaves {out_limbs}")
    delta = ctx.scale_at(L)
    q0 = float(ctx.params.q[0])
    # the SubSum of a sparse message multiplies it by the gap (N/2)/slots
    alpha = delta / (q0 * 2.0 * (K_RANGE + 1) * _gap(spec, ctx.logN))
    beta = q0 * 2.0 ** PRESCALE_BITS / (2.0 * math.pi * delta)
    cts, stc = _level_plans(ctx.logN, int(spec.log_slots), spec.level_budget, alpha, beta)
    slots = spec.slots
    b1 = int(spec.level_budget[0])
    cts_levels = [_encode_level(ctx, d, p, slots, L - i) for i, (d, p) in enumerate(cts)]
    s0 = L - b1 - EVALMOD_DEPTH
    stc_levels = [_encode_level(ctx, d, p, slots, s0 - i) for i, (d, p) in enumerate(stc)]

    def g(x):
        return np.cos(2.0 * np.pi * ((K_RANGE + 1) * x - 0.25) / 2 ** DOUBLINGS)

    coeffs = cheb.chebinterpolate(g, CHEB_DEGREE)
    pts = [lv.pts for lv in cts_levels + stc_levels]
    return Program(spec, cts_levels, stc_levels, coeffs, _Constants(pts))


# ---------------------------------------------------------------------------
# evaluation
# ---------------------------------------------------------------------------


def _linear(ct: fhe.Ciphertext, level: _Level, ctx: fhe.Context) -> fhe.Ciphertext:
    p = level.plan
    slots = int(ct.slots)
    offsets = tuple(o % slots for o in p.baby_offsets())
    babies = fhe.prepare_hoisted_baby_rotations(ct, offsets, ctx)
    acc = fhe.hoisted_mac_sum(ct, offsets, level.pts, p.babies * p.step, len(p.giants), ctx,
                              baby_rotations=babies)
    return fhe.rescale(acc, ctx)


def _post_scalar(value: float, a: fhe.Ciphertext, b: fhe.Ciphertext, ctx: fhe.Context):
    """`value` encoded for the state of rescale(a * b) (polynomial.py:50-70)."""

    limbs = min(int(a.state.cur_limbs), int(b.state.cur_limbs)) - 1
    scale = (float(a.state.scaling_factor) * float(b.state.scaling_factor)
             / ctx.rescale_divisor_at(limbs))
    return fhe.encode_scalar(value, cur_limbs=limbs, scale_degree=1, scaling_factor=scale,
                             context=ctx)


def _to_scale(ct: fhe.Ciphertext, target: float, ctx: fhe.Context) -> fhe.Ciphertext:
    """ct at one level lower with tracked scale exactly `target`: times the
    integer round(target q / scale(ct)), then rescale by q."""

    limbs = int(ct.state.cur_limbs)
    factor = target * ctx.rescale_divisor_at(limbs - 1) / float(ct.state.scaling_factor)
    enc = fhe.encode_scalar(1.0, cur_limbs=limbs, scale_degree=1, scaling_factor=factor,
                            context=ctx)
    return fhe.rescale(fhe.homo_mul_scalar(ct, enc, ctx), ctx)


def _cheb_basis(x: fhe.Ciphertext, ctx: fhe.Context) -> dict:
    """T_1..T_7 and the giants T_8, T_16, T_32 by T_{a+b} = 2 T_a T_b - T_{a-b};
    the subtracted T_{a-b} is first brought to the product's tracked scale."""

    mul = fhe.homo_mul_relin_rescale_postop

    def double_minus(a, b, low):
        prod = mul(a, b, ctx, apply_double=True)
        if low is None:  # T_0 = 1
            return fhe.homo_add_scalar(prod, fhe.encode_scalar(
                -1.0, cur_limbs=int(prod.state.cur_limbs), scale_degree=1,
                scaling_factor=prod.state.scaling_factor, context=ctx), ctx)
        fix = _to_scale(low, float(prod.state.scaling_factor), ctx)
        return fhe.homo_sub(prod, fhe.align_to(fix, prod.state, ctx), ctx)

    T = {1: x}
    T[2] = double_minus(x, x, None)
    T[3] = double_minus(T[2], T[1], T[1])
    T[4] = double_minus(T[2], T[2], None)
    T[5] = double_minus(T[3], T[2], T[1])
    T[6] = double_minus(T[3], T[3], None)
    T[7] = double_minus(T[4], T[3], T[1])
    for m in (8, 16, 32):
        T[m] = double_minus(T[m // 2], T[m // 2], None)
    return T


def _split(c: np.ndarray):
    """p = q T_m + r for the largest power of two m below deg p + 1."""

    m = 1
    while 2 * m < len(c):
        m *= 2
    q = np.zeros(len(c) - m)
    r = np.array(c[:m], dtype=np.float64)
    q[0] = c[m]
    for j in range(1, len(c) - m):
        q[j] = 2.0 * c[m + j]
        r[m - j] -= c[m + j]
    return m, q, r


def _cheb_limbs(c: np.ndarray, T: dict) -> int:
    """Limbs of _cheb_eval's output for coefficients c (no computation)."""

    if len(c) <= 8:
        ks = [k for k in range(1, len(c)) if abs(c[k]) >= 1e-30]
        if not ks:
            raise ValueError("Chebyshev leaf without a non-constant term")
        return min(int(T[k].state.cur_limbs) for k in ks) - 1
    m, q, r = _split(c)
    prod = min(_cheb_limbs(q, T), int(T[m].state.cur_limbs)) - 1
    return min(prod, _cheb_limbs(r, T))


def _cheb_eval(T: dict, coeffs: np.ndarray, target: float, ctx: fhe.Context) -> fhe.Ciphertext:
    """sum_k c_k T_k(x) with tracked scale exactly `target`, split recursively
    as p = q T_m + r.

    The scaling primes differ from 2^dcrt_bits by up to ~2^-33 relative and
    their products drift further, so scales are not taken as nominal: each
    leaf encodes its coefficients per term (c_k at target q / scale(T_k)),
    and a product q T_m asks its factor for target q_drop / scale(T_m).
    Every sum is then formed between operands of one exact scale, which the
    double angles and the SlotToCoeff gain would otherwise turn into error."""

    mul = fhe.homo_mul_relin_rescale_postop

    def leaf(c: np.ndarray, target: float) -> fhe.Ciphertext:
        ks = [k for k in range(1, len(c)) if abs(c[k]) >= 1e-30]
        limbs = min(int(T[k].state.cur_limbs) for k in ks)
        pre = target * ctx.rescale_divisor_at(limbs - 1)  # scale before the rescale
        encs = [fhe.encode_scalar(float(c[k]), cur_limbs=limbs, scale_degree=1,
                                  scaling_factor=pre / float(T[k].state.scaling_factor),
                                  context=ctx) for k in ks]
        # one pass over the terms at their own levels: sum_k c_k T_k, every
        # product at scale pre (up to the rounding of each encoded c_k)
        acc = fhe.homo_linear_combination([T[k] for k in ks], encs, ctx)
        acc.state = acc.state.replace(scaling_factor=pre)
        acc = fhe.rescale(acc, ctx)
        acc.state = acc.state.replace(scaling_factor=target)
        if abs(c[0]) >= 1e-30:
            acc = fhe.homo_add_scalar(acc, fhe.encode_scalar(
                float(c[0]), cur_limbs=int(acc.state.cur_limbs), scale_degree=1,
                scaling_factor=target, context=ctx), ctx)
        return acc

    def rec(c: np.ndarray, target: float) -> fhe.Ciphertext:
        if len(c) <= 8:
            return leaf(c, target)
        m, q, r = _split(c)
        tm = T[m]
        drop = min(_cheb_limbs(q, T), int(tm.state.cur_limbs)) - 1
        q_target = target * ctx.rescale_divisor_at(drop) / float(tm.state.scaling_factor)
        prod = mul(rec(q, q_target), tm, ctx)
        prod.state = prod.state.replace(scaling_factor=target)
        rest = rec(r, target)
        limbs = min(int(prod.state.cur_limbs), int(rest.state.cur_limbs))
        prod = fhe.align_to(prod, prod.state.replace(cur_limbs=limbs), ctx)
        rest = fhe.align_to(rest, rest.state.replace(cur_limbs=limbs), ctx)
        return fhe.homo_add(prod, rest, ctx)

    return rec(np.asarray(coeffs, dtype=np.float64), float(target))


def _evalmod(x: fhe.Ciphertext, coeffs: np.ndarray, target: float,
             ctx: fhe.Context) -> fhe.Ciphertext:
    """Chebyshev series, then DOUBLINGS steps v <- 2 v^2 - 1, ending at tracked
    scale exactly `target`: the series is evaluated at the scale S_0 with
    S_{i+1} = S_i^2 / q_drop(i), solved backwards from S_DOUBLINGS = target."""

    T = _cheb_basis(x, ctx)
    limbs = _cheb_limbs(np.asarray(coeffs, dtype=np.float64), T)
    s = float(target)
    for i in reversed(range(DOUBLINGS)):
        s = math.sqrt(s * ctx.rescale_divisor_at(limbs - 1 - i))
    v = _cheb_eval(T, coeffs, s, ctx)
    for _ in range(DOUBLINGS):
        v = fhe.homo_mul_relin_rescale_postop(v, v, ctx, apply_double=True,
                                              scalar=_post_scalar(-1.0, v, v, ctx))
    v.state = v.state.replace(scaling_factor=float(target))
    return v


def bootstrap(ct: fhe.Ciphertext, context, program: Program) -> fhe.Ciphertext:
    """Refresh `ct` (at least two limbs, scale degree 1, |slots| <= 1) to the
    program's output level (llama3fhe/operators/nonlinear/bootstrap.py:370)."""

    ctx = fhe._ctx_of(context)
    spec = program.spec
    C = ct.batch_size  # a ciphertext batch goes through every step together
    if int(ct.slots) != spec.slots:
        raise ValueError(f"bootstrap input slots={ct.slots}, program slots={spec.slots}")
    if int(ct.state.scale_degree) != 1 or ct.is_ext or ct.polys != 2:
        raise ValueError("bootstrap needs a relinearised, rescaled, non-extended ciphertext")
    l_in = int(ct.state.cur_limbs)
    if l_in < 2:
        raise ValueError("bootstrap needs an input with at least two limbs")
    in_scale = float(ct.state.scaling_factor)
    # read t + q_0 I at the scale the CoeffToSlot factor alpha assumes
    delta = ctx.scale_at(ctx.L)
    # 0. pre-scale by 2^-k delta / in_scale at the scale of the dropped prime:
    # t = u delta 2^-k for the message u, whatever scale the input tracked
    enc = fhe.encode_scalar(2.0 ** -PRESCALE_BITS * delta / in_scale, cur_limbs=l_in,
                            scale_degree=1, scaling_factor=ctx.rescale_divisor_at(l_in - 1),
                            context=ctx)
    x = fhe.rescale(fhe.homo_mul_scalar(ct, enc, ctx), ctx)
    x = fhe.align_to(x, x.state.replace(cur_limbs=1), ctx)
    # 1. ModRaise to all limbs
    raised = ctx.native.modraise(x.data, 2 * C, ctx.L)
    raised = raised.view((2, ctx.L, -1) if x.data.dim() == 3 else (C, 2, ctx.L, -1))
    y = fhe.Ciphertext(raised, fhe.CipherState(ctx.L, 1, delta), x.slots, ctx)
    # 1b. sparse messages: SubSum (trace onto Z[X^gap]) keeps the subring
    # coefficients of t = Delta u 2^-k + q_0 I, times the gap (folded into alpha)
    for r in _subsum_rotations(spec, ctx.logN):
        y = fhe.homo_add(y, fhe.homo_rotate(y, r, ctx), ctx)
    # 2. CoeffToSlot
    for level in program.cts:
        y = _linear(y, level, ctx)
    # 3. real / imaginary parts
    conj = fhe.homo_rotate(y, ctx.M - 1, ctx)
    x_re = fhe.homo_add(y, conj, ctx)
    x_im = fhe.homo_mul_i(fhe.homo_sub(y, conj, ctx), ctx, negative=True)
    # 4. EvalMod on both parts as one batch (real parts, then imaginary parts)
    both = _evalmod(fhe.pack_cipher_batch((x_re, x_im)), program.cheb, delta, ctx)
    halves = both.data.view((2, C) + tuple(both.data.shape[-3:]))
    s_re, s_im = (fhe.Ciphertext(h if C > 1 else h[0], both.state, both.slots, ctx)
                  for h in halves)
    # 5. recombine and SlotToCoeff
    z = fhe.homo_add(s_re, fhe.homo_mul_i(s_im, ctx), ctx)
    for level in program.stc:
        z = _linear(z, level, ctx)
    # the slots hold u at tracked scale delta = scale_at(L), the nominal scale:
    # a refresh starts its output's scale afresh, so the ratio of a tracked
    # scale to 2^dcrt_bits, which every product squares (e.g. the
    # Paterson-Stockmeyer doubling basis, operators/nonlinear/polynomial.py:
    # 138-151), does not compound from one polynomial-and-refresh to the next
    out = fhe.Ciphertext(z.data, z.state.replace(scale_degree=1, scaling_factor=delta),
                         ct.slots, ctx)
    if int(spec.output_levels):
        out = fhe.align_to(out, out.state.replace(cur_limbs=int(spec.output_levels) + 1), ctx)
    return out
