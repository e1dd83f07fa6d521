"""``easyfhe.fhe`` -- the CKKS evaluation surface llama3fhe calls, on libb200fhe.

Names, argument meanings, ownership and error types follow the reference's
call sites (each function cites one).  Every
operation runs in the CUDA kernels of libb200fhe on the current torch stream;
Python only validates levels and bookkeeps ciphertext state.

Ciphertexts are torch.int64 tensors [polys, limbs, N] of uint64 residues in
the evaluation (NTT) form, with a CipherState(cur_limbs, scale_degree,
scaling_factor).  Scale management is FIXEDMANUAL: scale_at(l) is
2^dcrt_bits at every level, rescale divides the tracked scaling factor by
the dropped prime (rescale_divisor_at), align_to drops limbs and keeps it.
"""

from __future__ import annotations

import dataclasses
import math
import sys
from dataclasses import dataclass, field
from typing import Any, Iterable

import numpy as np
import torch

from . import core
from .core import N, NativeContext, Params, galois_element, sample_secret

# ---------------------------------------------------------------------------
# states, specs
# ---------------------------------------------------------------------------


@dataclass(frozen=True)
class CipherState:
    """(cur_limbs, scale_degree, scaling_factor), as the reference builds it
    (llama3fhe/backend.py:248-254; primitives.py:130-134 uses .replace)."""

    cur_limbs: int
    scale_degree: int = 1
    scaling_factor: float | None = None

    def replace(self, **changes) -> "CipherState":
        return dataclasses.replace(self, **changes)


@dataclass(frozen=True)
class CKKSContextSpec:
    """fhe.CKKSContextSpec(depth, log_n, dnum, dcrt_bits, first_mod,
    secret_key_dist, scale_mode, rescale_policy, rotations, auto_load_keys)
    (llama3fhe/application/session.py:31-45)."""

    depth: int
    log_n: int
    dnum: int
    dcrt_bits: int
    first_mod: int
    secret_key_dist: str = "SPARSE_TERNARY"
    scale_mode: str = "fixed"
    rescale_policy: str = "manual"
    rotations: tuple = ()
    auto_load_keys: bool = True
    seed: int = 0x5EEDB200
    hamming_weight: int = 192
    special_bits: int = 60
    relin_key: bool = True


# ---------------------------------------------------------------------------
# context, client, ciphertexts, plaintexts
# ---------------------------------------------------------------------------


class Context:
    """Evaluation context: primes, device tables and evaluation keys."""

    def __init__(self, spec: CKKSContextSpec, params: Params, device: str):
        if str(spec.scale_mode).lower() != "fixed":
            raise NotImplementedError("only scale_mode='fixed' is implemented")
        self.spec = spec
        self.params = params
        self.native = NativeContext(params, device)
        self.device = str(self.native.device)
        self.logN = params.log_n
        self.N = 1 << self.logN
        self.M = 2 * self.N
        self.L = params.L
        self.K = params.K
        self.max_slots = self.N // 2
        self.rotation_keys: dict[int, torch.Tensor] = {}
        self.relin_key: torch.Tensor | None = None
        self._ws: dict[str, torch.Tensor] = {}
        # Declared rotations whose keys materialise on first use (auto_load_keys):
        # galois element -> True.  _keygen holds (secret in NTT form, seed).
        self._deferred: set[int] = set()
        self._keygen: tuple[torch.Tensor, int] | None = None
        self.keys_generated = 0

    def scale_at(self, cur_limbs: int) -> float:
        return float(2.0 ** int(self.spec.dcrt_bits))

    def rescale_divisor_at(self, cur_limbs: int) -> float:
        """Prime removed by the rescale that lands on cur_limbs."""

        return float(self.params.q[int(cur_limbs)])

    def clear_cuda_rotation_cache(self, keep_rotations=None) -> int:
        """Evict rotation keys from HBM (llama3fhe/operators/nonlinear/bootstrap.py:
        191-215, graph.py:1158): every key whose rotation is not in keep_rotations
        (None: every key) moves to pinned host memory; with spec.auto_load_keys the
        next use copies it back.  Returns the HBM bytes released to the caching
        allocator."""

        keep = set() if keep_rotations is None else {
            galois_element(int(r), self.logN) for r in keep_rotations}
        freed = 0
        for g, key in list(self.rotation_keys.items()):
            if g in keep or not key.is_cuda:
                continue
            host = torch.empty(key.shape, dtype=key.dtype, pin_memory=True)
            host.copy_(key)
            self.rotation_keys[g] = host
            freed += key.numel() * key.element_size()
        return freed

    def truncate_rotation_keys(self, max_limbs: int, rotations=None) -> int:
        """Keep only the digits a key needs up to max_limbs limbs (the first
        ceil(max_limbs / alpha) of dnum; the key inner product at l limbs reads
        digits j < ceil(l / alpha)).  For keys only used at low levels (the
        linears at 13 limbs read 2 of 5 digits at the layer parameters).  A
        truncated key used above max_limbs raises ValueError.  Returns the
        bytes released."""

        digits = -(-int(max_limbs) // self.native.alpha)
        if not 1 <= int(max_limbs) <= self.L:
            raise ValueError(f"max_limbs {max_limbs} outside [1, {self.L}]")
        sel = None if rotations is None else {
            galois_element(int(r), self.logN) for r in rotations}
        freed = 0
        for g, key in list(self.rotation_keys.items()):
            if (sel is not None and g not in sel) or key.shape[0] <= digits:
                continue
            freed += (key.shape[0] - digits) * key[0].numel() * key.element_size()
            self.rotation_keys[g] = key[:digits].clone()
            self._deferred.discard(g)  # an explicit truncation is final
        return freed

    def key_bytes(self) -> dict:
        """Bytes of evaluation keys in HBM and in host memory."""

        out = {"device": 0, "host": 0}
        keys = list(self.rotation_keys.values()) + (
            [self.relin_key] if self.relin_key is not None else [])
        for key in keys:
            out["device" if key.is_cuda else "host"] += key.numel() * key.element_size()
        return out

    def _materialize_key(self, g: int, digits: int) -> torch.Tensor:
        """Generate the key for galois element g and keep its first `digits`
        digits.  Keygen is deterministic in (seed, g), so this equals the key
        generate_client_context makes eagerly, truncated."""

        secret, seed = self._keygen
        full = self.native.keygen_rotation(secret, g, seed ^ g)
        self.keys_generated += 1
        key = full if digits >= full.shape[0] else full[:digits].clone()
        self.rotation_keys[g] = key
        return key

    def rotation_key(self, rotation: int, limbs: int | None = None) -> tuple[int, torch.Tensor]:
        g = galois_element(int(rotation), self.logN)
        key = self.rotation_keys.get(g)
        need = self.native.digits if limbs is None else -(-int(limbs) // self.native.alpha)
        if g in self._deferred and (key is None or key.shape[0] < need):
            # auto_load_keys: a declared key appears (or grows to the digits
            # this level reads) on first use, sized for that level: a key used
            # by the 13-limb linears keeps 2 of 5 digits at the layer parameters
            key = self._materialize_key(g, need)
        if key is None:
            raise ValueError(
                f"no rotation key for index {rotation} (galois {g}); the context "
                "rotation set must include every rotation used")
        if not key.is_cuda:
            if not bool(self.spec.auto_load_keys):
                raise ValueError(f"rotation key {rotation} was evicted from the device and "
                                 "the context has auto_load_keys=False")
            key = key.to(self.native.device)
            self.rotation_keys[g] = key
        if limbs is not None and key.shape[0] < -(-int(limbs) // self.native.alpha):
            raise ValueError(f"rotation key {rotation} keeps {key.shape[0]} digits, too few "
                             f"for {limbs} limbs")
        return g, key

    def workspace(self, name: str, nbytes: int) -> torch.Tensor:
        """A reusable scratch buffer (one per name; single-stream use)."""

        buf = self._ws.get(name)
        if buf is None or buf.numel() < nbytes:
            buf = self.native.workspace(nbytes)
            self._ws[name] = buf
        return buf


class Ciphertext:
    """A (batch of) ciphertext(s): data [polys, limbs, N] or
    [batch, polys, limbs, N]."""

    __slots__ = ("data", "state", "slots", "is_ext", "context")

    def __init__(self, data: torch.Tensor, state: CipherState, slots: int,
                 context: Context, is_ext: bool = False):
        self.data = data
        self.state = state
        self.slots = int(slots)
        self.context = context
        self.is_ext = bool(is_ext)

    @property
    def batch_size(self) -> int:
        return 1 if self.data.dim() == 3 else int(self.data.shape[0])

    @property
    def polys(self) -> int:
        return int(self.data.shape[-3])

    @property
    def cv(self) -> list[torch.Tensor]:
        return [self.data.select(-3, p) for p in range(self.polys)]

    def deep_copy(self) -> "Ciphertext":
        return Ciphertext(self.data.clone(), self.state, self.slots, self.context,
                          self.is_ext)

    def cipher_like(self, cv, slots: int | None = None,
                    batch_size: int | None = None) -> "Ciphertext":
        data = torch.stack([torch.as_tensor(c) for c in cv], dim=-3).contiguous()
        return Ciphertext(data, self.state, self.slots if slots is None else slots,
                          self.context, self.is_ext)

    # No release(): handles use Python ownership, as the EasyFHE the reference
    # targets does (llama3fhe/backend.py:336-346).  The reference's helpers
    # "release" values that other names still alias (the PS evaluator's
    # `su = t_basis[k - 1]`, operators/nonlinear/polynomial.py:300-324), which
    # is safe only because release_if_supported finds no release method; the
    # device memory goes back to the caching allocator with the last reference.


class Plaintext:
    """Encoded plaintext(s): data [rows, limbs, N] (ext: l Q-limbs + K)."""

    __slots__ = ("data", "state", "slots", "is_ext", "rows")

    def __init__(self, data: torch.Tensor, state: CipherState, slots: int, is_ext: bool):
        self.data = data
        self.state = state
        self.slots = int(slots)
        self.is_ext = bool(is_ext)
        self.rows = int(data.shape[0]) if data.dim() == 3 else 1

    @property
    def batch_size(self) -> int:
        return self.rows

    @property
    def cv(self) -> list[torch.Tensor]:
        return [self.data if self.data.dim() == 3 else self.data.unsqueeze(0)]

    def cipher_like(self, cv, slots: int | None = None,
                    batch_size: int | None = None) -> "Plaintext":
        """A plaintext batch over cv[0] (rows sliced by the caller,
        llama3fhe/operators/attention/input.py:1108-1115)."""

        return Plaintext(cv[0], self.state, self.slots if slots is None else slots,
                         self.is_ext)

    def q_part(self, limbs: int) -> torch.Tensor:
        """[rows, limbs, N] view of the Q limbs (contiguous when not ext)."""

        d = self.data if self.data.dim() == 3 else self.data.unsqueeze(0)
        if d.shape[1] == limbs:
            return d
        return d[:, :limbs].contiguous()



class Client:
    """Holds the secret key; client.encrypt / client.decrypt
    (llama3fhe/application/session.py:71-77, llama3fhe/backend.py:305-313)."""

    def __init__(self, context: Context, secret: np.ndarray, seed: int):
        self.context = context
        self._s_ntt = context.native.secret_to_ntt(secret)
        self._seed = int(seed)
        self._nonce = 0

    def encode(self, values, slots: int, cur_limbs: int, scaling_factor: float,
               ext: bool = False) -> torch.Tensor:
        v = torch.as_tensor(np.asarray(values)).reshape(-1)
        if v.numel() > slots:
            raise ValueError(f"{v.numel()} values do not fit {slots} slots")
        z = torch.zeros(slots, dtype=torch.complex128)
        z[: v.numel()] = v.to(torch.complex128)
        return self.context.native.encode(z.to(self.context.device), scaling_factor,
                                          cur_limbs, self.context.K if ext else 0)

    def encrypt(self, values, device=None, slots: int | None = None,
                cur_limbs: int | None = None, scaling_factor: float | None = None):
        ctx = self.context
        slots = ctx.max_slots if slots is None else int(slots)
        cur_limbs = ctx.L if cur_limbs is None else int(cur_limbs)
        scale = ctx.scale_at(cur_limbs) if scaling_factor is None else float(scaling_factor)
        m = self.encode(values, slots, cur_limbs, scale)
        self._nonce += 1
        data = ctx.native.encrypt(m, cur_limbs, self._s_ntt, self._seed, self._nonce)
        return Ciphertext(data, CipherState(cur_limbs, 1, scale), slots, ctx)

    def decrypt(self, cipher: Ciphertext) -> np.ndarray:
        """Real parts of the slots (float64)."""

        return self.decrypt_complex(cipher).real.copy()

    def decrypt_complex(self, cipher: Ciphertext) -> np.ndarray:
        ctx = self.context
        if cipher.is_ext:
            raise ValueError("decrypt needs a non-extended ciphertext")
        l = int(cipher.state.cur_limbs)
        data = cipher.data
        if cipher.polys == 3:
            data = homo_relinearize(cipher, ctx).data
        m = ctx.native.decrypt(data, l, self._s_ntt)
        scale = float(cipher.state.scaling_factor or ctx.scale_at(l))
        return ctx.native.decode(m, l, cipher.slots, scale)


def generate_client_context(spec: CKKSContextSpec, device: str = "cuda"):
    """fhe.generate_client_context (llama3fhe/application/session.py:31-45):
    primes, device tables, secret key, relinearisation and rotation keys."""

    if int(spec.log_n) != core.LOG_N:
        raise NotImplementedError("libb200fhe kernels are built for log_n = 16")
    params = Params.from_depth(spec.depth, spec.log_n, spec.dnum, spec.dcrt_bits,
                               spec.first_mod, special_bits=spec.special_bits)
    ctx = Context(spec, params, device)
    dist = str(spec.secret_key_dist).upper()
    hamming = int(spec.hamming_weight) if dist.startswith("SPARSE") else 0
    secret = sample_secret(int(spec.seed), hamming, spec.log_n)
    client = Client(ctx, secret, int(spec.seed) ^ 0xC1)
    s = client._s_ntt
    if spec.relin_key:
        ctx.relin_key = ctx.native.keygen_relin(s, int(spec.seed) ^ 0xE1)
    # auto_load_keys (the reference's setting, session.py:42): each declared
    # rotation key is generated on its first use with the digits that level
    # reads, instead of all of them at the top level up front (the layer
    # preset declares 674 rotations: 163 GB at 230 MiB each would not fit
    # beside the working set in one GPU's HBM).  Otherwise: every key now.
    ctx._keygen = (s, int(spec.seed))
    for r in sorted({int(v) for v in spec.rotations}):
        g = galois_element(r, spec.log_n)
        if g == 1 or g in ctx.rotation_keys:
            continue
        if bool(spec.auto_load_keys):
            ctx._deferred.add(g)
        else:
            ctx._materialize_key(g, ctx.native.digits)
    return client, ctx


# ---------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------


def _ctx_of(context) -> Context:
    c = getattr(context, "context", context)
    if not isinstance(c, Context):
        raise TypeError(f"expected an easyfhe.fhe.Context, got {type(context)!r}")
    return c


def _limbs(ct) -> int:
    return int(ct.state.cur_limbs)


def _drop(ct: Ciphertext, target: int) -> Ciphertext:
    l = _limbs(ct)
    if target == l:
        return ct
    if target > l or target < 1:
        raise ValueError(f"cannot align {l} limbs to {target}")
    polys = ct.polys * ct.batch_size
    data = ct.context.native.drop_limbs(ct.data, polys, l, target)
    shape = list(ct.data.shape)
    shape[-2] = target
    return Ciphertext(data.view(shape), ct.state.replace(cur_limbs=target), ct.slots,
                      ct.context, ct.is_ext)


def _match(a: Ciphertext, b: Ciphertext) -> tuple[Ciphertext, Ciphertext]:
    la, lb = _limbs(a), _limbs(b)
    if la > lb:
        a = _drop(a, lb)
    elif lb > la:
        b = _drop(b, la)
    return a, b


def _check_scales(a: Ciphertext, b, what: str) -> None:
    if int(a.state.scale_degree) != int(b.state.scale_degree):
        raise ValueError(f"{what}: scale degrees differ ({a.state.scale_degree} vs "
                         f"{b.state.scale_degree})")


def _new(data: torch.Tensor, like: Ciphertext, state: CipherState | None = None) -> Ciphertext:
    return Ciphertext(data, like.state if state is None else state, like.slots, like.context,
                      like.is_ext)


def _polys_total(ct: Ciphertext) -> int:
    return ct.polys * ct.batch_size


# ---------------------------------------------------------------------------
# additive ops
# ---------------------------------------------------------------------------


def _addsub(op: int, a: Ciphertext, b: Ciphertext, context) -> Ciphertext:
    ctx = _ctx_of(context)
    a, b = _match(a, b)
    _check_scales(a, b, "homo_add" if op == 0 else "homo_sub")
    if a.polys != b.polys:
        if a.polys < b.polys:
            a = _pad_polys(a, b.polys)
        else:
            b = _pad_polys(b, a.polys)
    l = _limbs(a)
    out = ctx.native.elementwise(op, a.data, b.data, _polys_total(a), l)
    return _new(out.view(a.data.shape), a)


def _pad_polys(ct: Ciphertext, polys: int) -> Ciphertext:
    extra = torch.zeros((polys - ct.polys,) + tuple(ct.data.shape[-2:]), dtype=ct.data.dtype,
                        device=ct.data.device)
    return _new(torch.cat([ct.data, extra], dim=0), ct)


def homo_add(a: Ciphertext, b: Ciphertext, context) -> Ciphertext:
    """a + b (28 call sites, e.g. llama3fhe/operators/linear/operator.py:345-351)."""

    return _addsub(0, a, b, context)


def homo_sub(a: Ciphertext, b: Ciphertext, context) -> Ciphertext:
    """a - b (llama3fhe/operators/linear/complex.py:60-62)."""

    return _addsub(1, a, b, context)


def homo_add_pt(ct: Ciphertext, pt: Plaintext, context) -> Ciphertext:
    """ct + pt, the plaintext added to c0."""

    ctx = _ctx_of(context)
    l = _limbs(ct)
    if int(pt.state.cur_limbs) < l:
        raise ValueError(f"plaintext at {pt.state.cur_limbs} limbs, ciphertext at {l}")
    if int(pt.state.scale_degree) != int(ct.state.scale_degree):
        raise ValueError("homo_add_pt: scale degrees differ")
    p = pt.q_part(l)[0]
    out = ct.data.clone()
    ctx.native.elementwise(0, ct.data[0], p, 1, l, out=out[0])
    return _new(out, ct)


def homo_mul_pt(ct: Ciphertext, pt: Plaintext, context) -> Ciphertext:
    """ct * pt (llama3fhe/operators/primitives.py:40-49); scale degree adds."""

    ctx = _ctx_of(context)
    l = _limbs(ct)
    if int(pt.state.cur_limbs) < l:
        raise ValueError(f"plaintext at {pt.state.cur_limbs} limbs, ciphertext at {l}")
    p = pt.q_part(l)[0]
    out = ctx.native.elementwise(2, ct.data, p, _polys_total(ct), l, b_polys=1)
    state = ct.state.replace(
        scale_degree=int(ct.state.scale_degree) + int(pt.state.scale_degree),
        scaling_factor=float(ct.state.scaling_factor) * float(pt.state.scaling_factor))
    return _new(out.view(ct.data.shape), ct, state)


def homo_mul_i(ct: Ciphertext, context, negative: bool = False) -> Ciphertext:
    """Multiply every slot by i (or -i): the monomial X^(N/2), no key
    (llama3fhe/operators/linear/complex.py:22; attention/codec.py:42)."""

    ctx = _ctx_of(context)
    out = ctx.native.mul_i(ct.data, _polys_total(ct), _limbs(ct), bool(negative))
    return _new(out.view(ct.data.shape), ct)


# ---------------------------------------------------------------------------
# scalars
# ---------------------------------------------------------------------------


@dataclass(frozen=True)
class EncodedScalar:
    residues: tuple[int, ...]
    state: CipherState
    value: float


def encode_scalar(value, cur_limbs: int, scale_degree: int = 1, scaling_factor=None,
                  context=None, mode: str = "double") -> EncodedScalar:
    """fhe.encode_scalar(v, cur_limbs, scale_degree, scaling_factor | mode,
    context) (llama3fhe/operators/nonlinear/bootstrap.py:331-349,
    polynomial.py:41-47): the constant round(v * scale^degree) in RNS."""

    ctx = _ctx_of(context)
    cur_limbs = int(cur_limbs)
    if str(mode) == "integer":
        integer = int(value)
        scale = 1.0
        degree = 0
    else:
        degree = int(scale_degree)
        scale = float(scaling_factor if scaling_factor is not None
                      else ctx.scale_at(cur_limbs)) if degree else 1.0
        x = float(value) * (scale if degree else 1.0)
        if not math.isfinite(x):
            raise ValueError("encoded scalar overflows")
        integer = int(round(x))
    residues = tuple(integer % q for q in ctx.params.q[:cur_limbs])
    return EncodedScalar(residues, CipherState(cur_limbs, degree, scale), float(value))


def _enc_for(ct: Ciphertext, enc: EncodedScalar) -> tuple[int, ...]:
    l = _limbs(ct)
    if len(enc.residues) < l:
        raise ValueError(f"scalar encoded for {len(enc.residues)} limbs, cipher has {l}")
    return enc.residues[:l]


def homo_mul_scalar(ct: Ciphertext, enc: EncodedScalar, context) -> Ciphertext:
    """ct * scalar without rescale (llama3fhe/operators/nonlinear/bootstrap.py:338)."""

    ctx = _ctx_of(context)
    l = _limbs(ct)
    out = ctx.native.scalar_op(ct.data, _polys_total(ct), l, mul=_enc_for(ct, enc))
    state = ct.state.replace(
        scale_degree=int(ct.state.scale_degree) + int(enc.state.scale_degree),
        scaling_factor=float(ct.state.scaling_factor) * float(enc.state.scaling_factor))
    return _new(out.view(ct.data.shape), ct, state)


def homo_mul_scalar_rescale(ct: Ciphertext, enc: EncodedScalar, context) -> Ciphertext:
    """ct * scalar, rescaled (llama3fhe/operators/norm/refresh.py:28-30)."""

    return rescale(homo_mul_scalar(ct, enc, context), context)


def homo_linear_combination(cts, scalars, context) -> Ciphertext:
    """sum_k scalars[k] * cts[k] in one pass, at the fewest limbs among the
    terms (no modulus drop of the others first).  Every product must land on
    the same state (scale degree and tracked scaling factor), as the caller
    arranges by encoding each scalar for its term.  No reference counterpart:
    the fused form of homo_mul_scalar + homo_add chains
    (llama3fhe/operators/nonlinear/polynomial.py:41-88)."""

    ctx = _ctx_of(context)
    cts, scalars = list(cts), list(scalars)
    if not cts or len(cts) != len(scalars):
        raise ValueError("homo_linear_combination needs one scalar per ciphertext")
    first = cts[0]
    for c in cts:
        if c.is_ext or c.polys != first.polys or c.batch_size != first.batch_size:
            raise ValueError("homo_linear_combination: terms differ in basis, polys or batch")
    l = min(_limbs(c) for c in cts)
    states = set()
    for c, e in zip(cts, scalars):
        states.add((int(c.state.scale_degree) + int(e.state.scale_degree),
                    float(c.state.scaling_factor) * float(e.state.scaling_factor)))
    degree, scale = states.pop()
    if any(d != degree or abs(sf - scale) > 1e-9 * abs(scale) for d, sf in states):
        raise ValueError("homo_linear_combination: the products do not share one state")
    weights = []
    for e in scalars:
        if len(e.residues) < l:
            raise ValueError(f"scalar encoded for {len(e.residues)} limbs, terms have {l}")
        weights.append(e.residues[:l])
    state = first.state.replace(cur_limbs=l, scale_degree=degree, scaling_factor=scale)
    try:
        data = ctx.native.linear_combination([c.data for c in cts], [_limbs(c) for c in cts],
                                             weights, first.batch_size, first.polys, l)
    except NotImplementedError:  # more terms or limbs than one pass carries
        acc = None
        for c, e in zip(cts, scalars):
            t = homo_mul_scalar(align_to(c, c.state.replace(cur_limbs=l), ctx), e, ctx)
            acc = t if acc is None else _addsub(0, acc, t, ctx)
        return Ciphertext(acc.data, state, first.slots, ctx)
    shape = list(first.data.shape)
    shape[-2] = l
    return Ciphertext(data.view(shape), state, first.slots, ctx)


def homo_add_scalar(ct: Ciphertext, enc: EncodedScalar, context) -> Ciphertext:
    """ct + scalar, added to c0 (llama3fhe/operators/nonlinear/polynomial.py:84-88)."""

    ctx = _ctx_of(context)
    l = _limbs(ct)
    if ct.batch_size != 1 and ct.polys != 2:
        raise NotImplementedError("homo_add_scalar on a batch of degree-2 ciphertexts")
    out = ctx.native.scalar_op(ct.data, _polys_total(ct), l, add=_enc_for(ct, enc),
                               add_poly=0 if ct.batch_size == 1 else -2)
    return _new(out.view(ct.data.shape), ct)


# ---------------------------------------------------------------------------
# levels
# ---------------------------------------------------------------------------


def rescale(ct: Ciphertext, context) -> Ciphertext:
    """Divide by the last prime (57 sites; llama3fhe/operators/linear/operator.py:386-388)."""

    ctx = _ctx_of(context)
    l = _limbs(ct)
    if l < 2:
        raise ValueError("rescale needs at least two limbs")
    out = ctx.native.rescale(ct.data, _polys_total(ct), l)
    shape = list(ct.data.shape)
    shape[-2] = l - 1
    return _new(out.view(shape), ct, _rescaled_state(ct, ctx))


def _rescaled_state(ct: Ciphertext, ctx) -> CipherState:
    l = _limbs(ct)
    return ct.state.replace(
        cur_limbs=l - 1,
        scale_degree=max(1, int(ct.state.scale_degree) - 1),
        scaling_factor=float(ct.state.scaling_factor) / ctx.rescale_divisor_at(l - 1))


def align_to(ct: Ciphertext, state: CipherState, context) -> Ciphertext:
    """Scale-preserving modulus drop to state.cur_limbs; returns ct itself when
    nothing changes (llama3fhe/operators/primitives.py:100-155)."""

    _ctx_of(context)
    target = int(state.cur_limbs)
    if target == _limbs(ct):
        return ct
    if target > _limbs(ct):
        raise ValueError(f"cannot raise {_limbs(ct)} limbs to {target}")
    return _drop(ct, target)


# ---------------------------------------------------------------------------
# rotations and multiplication
# ---------------------------------------------------------------------------


def homo_rotate(ct: Ciphertext, rotation: int, context) -> Ciphertext:
    """Left rotation of the slots by `rotation` (M - 1: conjugation) with hybrid
    key switching (34 sites, e.g. llama3fhe/operators/linear/operator.py:333-337)."""

    ctx = _ctx_of(context)
    if ct.is_ext:
        raise ValueError("homo_rotate needs a non-extended ciphertext")
    if ct.polys != 2:
        raise ValueError("homo_rotate needs a relinearised ciphertext")
    g = galois_element(int(rotation), ctx.logN)
    if g == 1:
        return ct.deep_copy()
    l = _limbs(ct)
    _, key = ctx.rotation_key(int(rotation), l)
    out = ctx.native.rotate(ct.data, l, g, key)
    return _new(out, ct)


def homo_mul_no_relin(a: Ciphertext, b: Ciphertext, context) -> Ciphertext:
    """Tensor product (d0, d1, d2) (llama3fhe/operators/attention/qk.py:399)."""

    ctx = _ctx_of(context)
    a, b = _match(a, b)
    if a.polys != 2 or b.polys != 2:
        raise ValueError("homo_mul_no_relin needs degree-1 ciphertexts")
    if a.batch_size != b.batch_size:
        raise ValueError(f"homo_mul_no_relin: batches of {a.batch_size} and {b.batch_size}")
    l = _limbs(a)
    out = ctx.native.tensor(a.data, b.data, a.batch_size, l)
    out = out.view((3,) + tuple(a.data.shape[-2:]) if a.data.dim() == 3
                   else (a.batch_size, 3) + tuple(a.data.shape[-2:]))
    state = a.state.replace(
        scale_degree=int(a.state.scale_degree) + int(b.state.scale_degree),
        scaling_factor=float(a.state.scaling_factor) * float(b.state.scaling_factor))
    return _new(out, a, state)


def homo_relinearize(ct: Ciphertext, context) -> Ciphertext:
    """(d0, d1, d2) -> (d0, d1) + KeySwitch_{s^2 -> s}(d2)
    (llama3fhe/operators/attention/kernel_helpers.py:155)."""

    ctx = _ctx_of(context)
    if ct.polys == 2:
        return ct.deep_copy()
    if ctx.relin_key is None:
        raise ValueError("context has no relinearisation key")
    l = _limbs(ct)
    out = ctx.native.relinearize(ct.data, l, ctx.relin_key)
    return _new(out, ct)


def _relinearize_rescale(ct: Ciphertext, context) -> Ciphertext:
    """rescale(homo_relinearize(ct)) as one native pass (b2f_relinearize_rescale):
    the ModDown by P and the division by the last prime merged into one
    rounding division."""

    ctx = _ctx_of(context)
    if ct.polys == 2:
        return rescale(ct, context)
    if ctx.relin_key is None:
        raise ValueError("context has no relinearisation key")
    l = _limbs(ct)
    if l < 2:
        raise ValueError("rescale needs at least two limbs")
    out = ctx.native.relinearize_rescale(ct.data, l, ctx.relin_key)
    return _new(out, ct, _rescaled_state(ct, ctx))


def homo_mul_relin(a: Ciphertext, b: Ciphertext, context) -> Ciphertext:
    """a * b, relinearised (llama3fhe/operators/primitives.py:21-31)."""

    return homo_relinearize(homo_mul_no_relin(a, b, context), context)


def homo_mul_relin_rescale_postop(left: Ciphertext, right: Ciphertext, context,
                                  apply_double: bool = False, sub=None,
                                  scalar: EncodedScalar | None = None) -> Ciphertext:
    """rescale(relin(l * r)), then optionally times 2, minus `sub`, plus `scalar`
    (llama3fhe/operators/nonlinear/polynomial.py:108-159): the Chebyshev step
    T_{a+b} = 2 T_a T_b - T_{a-b}.  The post-operation runs in the epilogue of
    the relinearise-rescale's last transform (b2f_relinearize_rescale_postop):
    no extra launch, and sub is read at its own level (no alignment copy).
    The residues equal relinearise-rescale followed by homo_add(out, out),
    homo_sub(out, align_to(sub)) and homo_add_scalar."""

    ctx = _ctx_of(context)
    prod = homo_mul_no_relin(left, right, context)
    if prod.polys == 2 or not (apply_double or sub is not None or scalar is not None):
        out = _relinearize_rescale(prod, context)
        if apply_double:
            out = homo_add(out, out, context)
        if sub is not None:
            out = homo_sub(out, align_to(sub, out.state, context), context)
        if scalar is not None:
            out = homo_add_scalar(out, scalar, context)
        return out
    if ctx.relin_key is None:
        raise ValueError("context has no relinearisation key")
    l = _limbs(prod)
    if l < 2:
        raise ValueError("rescale needs at least two limbs")
    state = _rescaled_state(prod, ctx)
    sub_data, sub_limbs = None, 0
    if sub is not None:
        if sub.is_ext or sub.polys != 2 or sub.batch_size != prod.batch_size:
            raise ValueError("homo_mul_relin_rescale_postop: sub must be a relinearised "
                             "ciphertext of the product's batch")
        if int(sub.state.scale_degree) != int(state.scale_degree):
            raise ValueError("homo_sub: scale degrees differ "
                             f"({state.scale_degree} vs {sub.state.scale_degree})")
        sub_limbs = _limbs(sub)
        if sub_limbs < l - 1:
            raise ValueError(f"cannot align {sub_limbs} limbs to {l - 1}")
        sub_data = sub.data.contiguous()
    residues = None
    if scalar is not None:
        if len(scalar.residues) < l - 1:
            raise ValueError(f"scalar encoded for {len(scalar.residues)} limbs, the result "
                             f"has {l - 1}")
        residues = scalar.residues[: l - 1]
    out = ctx.native.relinearize_rescale(prod.data, l, ctx.relin_key,
                                         apply_double=bool(apply_double), sub=sub_data,
                                         sub_limbs=sub_limbs, scalar=residues)
    return _new(out, prod, state)


# ---------------------------------------------------------------------------
# baby-step / giant-step
# ---------------------------------------------------------------------------


class BabyRotations(tuple):
    """Hoisted baby rotations of one ciphertext: block 0 is a Ciphertext batch
    [B, 2, l, N] (baby b = rotation by baby_offsets[b]); for a batch of C
    ciphertexts it is [C * B, 2, l, N], ciphertext-major.  With an extended
    strategy the block is in Q_l u P ([.., 2, l + K, N], P times the
    rotation, before ModDown).  Iterable like the reference's block tuple
    (llama3fhe/operators/linear/operator.py:119-122)."""

    offsets: tuple[int, ...] = ()
    cts: int = 1
    strategy: str = "normal"


HOIST_STRATEGIES = ("normal", "ext_normal", "ext_double_hoist")


def _strategy(strategy) -> str:
    """The reference's hoist strategies (llama3fhe/operators/linear/config.py:9)."""

    s = str(strategy).lower()
    if s not in HOIST_STRATEGIES:
        raise ValueError(f"unknown hoist strategy {strategy!r}; expected one of "
                         f"{', '.join(HOIST_STRATEGIES)}")
    return s


def _baby_blocks(offsets: tuple[int, ...], anchor: int) -> list[tuple[int, int]]:
    """(start, width) blocks of the babies: one block, or blocks of `anchor`
    babies when 2 <= anchor < B (llama3fhe/operators/linear/config.py:207-240).
    Anchored blocks need arithmetic offsets b * step."""

    B = len(offsets)
    if not (int(anchor) >= 2 and B > int(anchor)):
        return [(0, B)]
    step = offsets[1] - offsets[0] if B > 1 else 0
    if any(offsets[b] != offsets[0] + b * step for b in range(B)):
        raise ValueError("baby_anchor_step needs baby offsets b * step")
    return [(start, min(int(anchor), B - start)) for start in range(0, B, int(anchor))]


def _hoisted_block(ct: Ciphertext, rel: tuple[int, ...], ext: bool, ctx) -> torch.Tensor:
    """Hoisted rotations of ct by `rel` (one ModUp): [C, n, 2, l(+K), N]."""

    l = _limbs(ct)
    nat = ctx.native
    gal, keys = [], []
    for off in rel:
        g = galois_element(off, ctx.logN)
        gal.append(g)
        keys.append(None if g == 1 else ctx.rotation_key(off, l)[1])
    C = ct.batch_size
    if not ext:
        mod = nat.modup(ct.data, l, C) if any(g != 1 for g in gal) else None
        out = nat.rotate_hoisted(ct.data, l, mod, gal, keys, num_cts=C)
        return out.reshape(C, len(rel), 2, l, -1)
    items = [ct.data] if C == 1 else [ct.data[c] for c in range(C)]
    outs = []
    for d in items:
        mod = nat.modup(d, l) if any(g != 1 for g in gal) else None
        outs.append(nat.rotate_hoisted_ext(d, l, mod, gal, keys))
    return torch.stack(outs)


def prepare_hoisted_baby_rotations(ct: Ciphertext, baby_offsets, context,
                                   strategy: str = "normal",
                                   baby_anchor_step: int = -1) -> BabyRotations:
    """Baby rotations of ct by every baby offset (llama3fhe/operators/linear/
    operator.py:105-111).  One block: one ModUp of c1 and one key inner
    product (+ ModDown) per offset.  With 2 <= baby_anchor_step < B, blocks of
    baby_anchor_step babies, each hoisted from an anchor that the one anchor
    key (baby_anchor_step * step) reaches from the previous anchor
    (llama3fhe/operators/linear/config.py:50-57, 207-233).  The extended
    strategies leave the babies in Q_l u P for hoisted_mac_sum."""

    ctx = _ctx_of(context)
    s = _strategy(strategy)
    ext = s != "normal"
    offsets = tuple(int(v) for v in baby_offsets)
    C = ct.batch_size
    blocks = _baby_blocks(offsets, int(baby_anchor_step))
    parts, anchor = [], ct
    for k, (start, width) in enumerate(blocks):
        if k:
            anchor = homo_rotate(anchor, offsets[start] - offsets[blocks[k - 1][0]], ctx)
        rel = tuple(offsets[start + b] - offsets[start] + offsets[0] for b in range(width))
        parts.append(_hoisted_block(anchor, rel, ext, ctx))
    data = parts[0] if len(parts) == 1 else torch.cat(parts, dim=1)
    l = _limbs(ct)
    # a ciphertext batch keeps its babies ciphertext-major: [C * B, 2, l(+K), N]
    data = data.reshape(C * len(offsets), 2, data.shape[-2], data.shape[-1])
    block = Ciphertext(data, ct.state, ct.slots, ctx, is_ext=ext)
    babies = BabyRotations((block,))
    babies.offsets = offsets
    babies.cts = C
    babies.strategy = s
    return babies


def hoisted_mac_sum(ct: Ciphertext, baby_offsets, plaintexts: Plaintext, giant_offset: int,
                    giant_count: int, context, strategy: str = "normal",
                    baby_anchor_step: int = -1, baby_rotations=None) -> Ciphertext:
    """sum_{g<G} rot_{g*giant_offset}(sum_b pt[g*B+b] * rot_{baby_offsets[b]}(ct))
    (llama3fhe/operators/linear/operator.py:320-330, transform.py:108-116).
    The result is at the input level with scale degree 2; the caller rescales.

    strategy (llama3fhe/operators/linear/config.py:9, 286-305):
      normal           babies and MAC in Q_l; Horner over the giants with the
                       one giant key (by default the chain stays in Q_l u P
                       and ModDowns once; NativeContext.set_giant_chain);
      ext_normal       babies left in Q_l u P, plaintexts encoded there
                       (is_ext), MAC over Q_l u P, then the same Horner chain
                       over the extended sums;
      ext_double_hoist as ext_normal, but every giant sum but the first is
                       ModDown'ed, rotated by g * giant_offset with its own
                       key into Q_l u P, and the sum is ModDown'ed once."""

    ctx = _ctx_of(context)
    s = _strategy(strategy)
    ext = s != "normal"
    offsets = tuple(int(v) for v in baby_offsets)
    B, G = len(offsets), int(giant_count)
    l = _limbs(ct)
    if baby_rotations is None:
        baby_rotations = prepare_hoisted_baby_rotations(ct, offsets, ctx, s, baby_anchor_step)
    block = tuple(baby_rotations)[0]
    if int(block.state.cur_limbs) != l:
        raise ValueError("baby rotations were prepared at a different level")
    if bool(block.is_ext) != ext:
        raise ValueError(f"baby rotations were prepared for a {'n extended' if block.is_ext else ' normal'} "
                         f"strategy, hoisted_mac_sum called with {s!r}")
    C = ct.batch_size
    if block.batch_size != C * B:
        raise ValueError(f"{block.batch_size} baby rotations for {C} ciphertexts x {B} "
                         "offsets")
    if plaintexts.rows < G * B:
        raise ValueError(f"{plaintexts.rows} plaintext rows < giants*babies = {G * B}")
    state = ct.state.replace(
        scale_degree=int(ct.state.scale_degree) + int(plaintexts.state.scale_degree),
        scaling_factor=float(ct.state.scaling_factor) * float(plaintexts.state.scaling_factor))
    if not ext:
        pts = plaintexts.q_part(l)
        if G > 1:
            gg, gkey = ctx.rotation_key(int(giant_offset), l)
        else:
            gg, gkey = 1, None
        out = ctx.native.bsgs_mac(block.data, B, pts, G, l, gg, gkey, num_cts=C)
        return Ciphertext(out, state, ct.slots, ctx)
    if not plaintexts.is_ext or int(plaintexts.state.cur_limbs) != l:
        raise ValueError(f"strategy {s!r} needs plaintexts encoded at the ciphertext's level "
                         "in the extended basis (ConstantBundle.plaintext(is_ext=True))")
    K = ctx.K
    pts = plaintexts.cv[0]
    inner = ctx.native.mac_ext(block.data, B, pts, G, l, num_cts=C)  # [C, G, 2, l+K, N]
    n = inner.shape[-1]
    shape = (2, l, n) if C == 1 else (C, 2, l, n)
    if s == "ext_normal" and G > 1 and ctx.native.giant_chain_mode == "extended":
        # the Horner chain straight from the extended sums, kept in Q_l u P:
        # one ModDown per chain
        gg, gkey = ctx.rotation_key(int(giant_offset), l)
        out = ctx.native.giant_chain(inner, True, C, G, l, gg, gkey)
        return Ciphertext(out.view(shape), state, ct.slots, ctx)

    # one ModDown launch for every giant's sum of every ciphertext
    first = 0 if s == "ext_normal" else 1
    down = ctx.native.moddown_ext(inner[:, first:].reshape(-1, 2, l + K, n), C * (G - first), l)
    down = down.view(C, G - first, 2, l, n)

    def giant(g: int) -> Ciphertext:  # giant g's ModDown'ed sum, all ciphertexts
        d = down[:, g - first]
        return Ciphertext(d.reshape(shape) if C > 1 else d[0], state, ct.slots, ctx)

    if s == "ext_normal":
        acc = giant(G - 1)
        for g in range(G - 2, -1, -1):
            acc = homo_add(homo_rotate(acc, int(giant_offset), ctx), giant(g), ctx)
        return acc
    # ext_double_hoist: sum_g P rot_{g off}(giant g) in Q_l u P, one ModDown
    acc = inner[:, 0].contiguous()  # P * giant 0, as the MAC left it
    for g in range(1, G):
        r = _hoisted_block(giant(g), (g * int(giant_offset),), True, ctx)[:, 0]
        ctx.native.elementwise_ext(0, acc, r.contiguous(), 2 * C, l, out=acc)
    out = ctx.native.moddown_ext(acc, C, l)
    return Ciphertext(out.view(shape), state, ct.slots, ctx)


# ---------------------------------------------------------------------------
# constants
# ---------------------------------------------------------------------------


class PackedRaw:
    """Slot values already packed: [rows, slots] or [slots] (llama3fhe/backend.py:282)."""

    def __init__(self, tensor):
        self.tensor = tensor


class UnpackedRaw:
    """Raw weight plus the packer that lays out its diagonals
    (llama3fhe/operators/linear/weight.py:309-310)."""

    def __init__(self, source, packer):
        self.source = source
        self.packer = packer


# Counters of how linear-weight chunks were packed (tests read them).
PACK_STATS = {"dense": 0, "structured": 0, "foreign": 0}


def _native_chunk_pack(raw: UnpackedRaw, slots: int, context) -> torch.Tensor | None:
    """Pack a linear-weight chunk with the CUDA packers when `raw.packer` is the
    reference's chunk packer (the `pack` closure of
    llama3fhe/operators/linear/weight.py:50-104).  That closure would call the
    Triton kernels of gpu_packer.py:144-184 / 317-424 (or the NumPy
    `_cpu_packer`, weight.py:18-47); its bound plan, chunk and weight give every
    argument those kernels take, so the same rows come from
    b2f_pack_diagonals / b2f_pack_structured instead and Triton is never
    imported.  Returns None for any other packer callable."""

    import inspect

    fn = raw.packer
    if (getattr(fn, "__qualname__", "") != "_chunk_packer.<locals>.pack"
            or not str(getattr(fn, "__module__", "")).endswith("operators.linear.weight")):
        PACK_STATS["foreign"] += 1
        return None
    nl = inspect.getclosurevars(fn).nonlocals
    plan, chunk, weight = nl["plan"], nl["chunk"], nl["weight"]
    bound_slots = int(nl["slots"])
    if int(slots) != bound_slots:
        raise ValueError(f"linear weight expects slots={bound_slots}, got {slots}.")
    ctx = _ctx_of(context)
    geometry = dict(dimension=int(plan.dimension), token_lanes=int(plan.token_lanes),
                    baby_steps=int(plan.baby_steps), giant_base=int(chunk.giant_base),
                    giant_count=int(chunk.giant_count), slots=bound_slots)
    if hasattr(weight, "real_source") and hasattr(weight, "sources"):
        # StructuredLinearWeight (structured_weight.py:47-192): reuse the device
        # copies LinearWeight.prepare made when it made them, else its arrays.
        dev_src = tuple(nl.get("structured_device_sources") or ())
        dev_meta = nl.get("structured_device_metadata") or {}
        sources = dev_src if dev_src else tuple(weight.sources)
        maps = {n: dev_meta.get(n, getattr(weight, n)) for n in NativeContext._STRUCT_MAPS}
        PACK_STATS["structured"] += 1
        return ctx.native.pack_structured(sources, maps, **geometry)
    # dense square page: the raw source handed to UnpackedRaw (a device or host
    # tensor of the weight), or the NumPy weight the closure holds
    src = raw.source if torch.is_tensor(raw.source) else torch.as_tensor(np.asarray(weight))
    if src.dim() != 2 or tuple(src.shape) != (geometry["dimension"],) * 2:
        src = torch.as_tensor(np.asarray(weight))
    PACK_STATS["dense"] += 1
    return ctx.native.pack_diagonals(src.to(ctx.device), **geometry)


class ConstantBundle:
    """Named constant vectors encoded on demand at a requested state
    (llama3fhe/backend.py:231-297, llama3fhe/operators/linear/weight.py:344-357).
    cache_mode 'plain'/'both' keeps the encoded plaintexts; 'middle' keeps the
    packed slot values; 'none' keeps nothing."""

    _MODES = {"none", "middle", "plain", "both"}

    def __init__(self, vectors: dict, cache_mode: str = "none"):
        if str(cache_mode) not in self._MODES:
            raise ValueError(f"cache_mode must be one of {sorted(self._MODES)}")
        self.vectors = dict(vectors)
        self.cache_mode = str(cache_mode)
        self._middle: dict[Any, torch.Tensor] = {}
        self._plain: dict[Any, Plaintext] = {}
        self._stats = {"middle_hits": 0, "middle_misses": 0, "plain_hits": 0,
                       "plain_misses": 0}

    def set_cache_mode(self, mode: str) -> None:
        if str(mode) not in self._MODES:
            raise ValueError(f"cache_mode must be one of {sorted(self._MODES)}")
        self.cache_mode = str(mode)

    def _slots_values(self, name: str, slots: int, context: Context) -> torch.Tensor:
        key = (name, slots)
        if key in self._middle:
            self._stats["middle_hits"] += 1
            return self._middle[key]
        self._stats["middle_misses"] += 1
        raw = self.vectors[name]
        if isinstance(raw, UnpackedRaw):
            values = _native_chunk_pack(raw, slots, context)
            if values is None:  # a caller's own packer: run it as given
                values = raw.packer(raw.source, slots, context)
        elif isinstance(raw, PackedRaw):
            values = raw.tensor
        else:
            values = raw
        t = torch.as_tensor(values)
        if t.device.type != "cuda":
            # through pinned memory, without blocking the host on the GPU: a
            # pageable copy would wait for every kernel queued before it (the
            # reference builds many mask bundles from NumPy inside a layer);
            # torch keeps the pinned block until the copy has run
            t = t.pin_memory().to(context.device, non_blocking=True)
        t = t.to(torch.complex128)
        if t.dim() == 1:
            t = t.unsqueeze(0)
        if t.shape[-1] != slots:
            if t.shape[-1] > slots:
                raise ValueError(f"{t.shape[-1]} values do not fit {slots} slots")
            pad = torch.zeros(t.shape[0], slots - t.shape[-1], dtype=t.dtype, device=t.device)
            t = torch.cat([t, pad], dim=1)
        if self.cache_mode in ("middle", "both"):
            self._middle[key] = t
        return t

    def plaintext(self, name: str, state: CipherState | None = None, slots: int | None = None,
                  context=None, is_ext: bool = False, cache: bool = False) -> Plaintext:
        ctx = _ctx_of(context)
        slots = ctx.max_slots if slots is None else int(slots)
        state = state or CipherState(ctx.L, 1, ctx.scale_at(ctx.L))
        l = int(state.cur_limbs)
        scale = float(state.scaling_factor if state.scaling_factor is not None
                      else ctx.scale_at(l))
        key = (name, slots, l, scale, bool(is_ext))
        if key in self._plain:
            self._stats["plain_hits"] += 1
            return self._plain[key]
        self._stats["plain_misses"] += 1
        values = self._slots_values(name, slots, ctx)
        data = ctx.native.encode(values, scale, l, ctx.K if is_ext else 0)
        pt = Plaintext(data, CipherState(l, int(state.scale_degree or 1), scale), slots,
                       bool(is_ext))
        if self.cache_mode in ("plain", "both") and cache is not False:
            self._plain[key] = pt
        return pt

    def cache_info(self) -> dict:
        mb = sum(int(t.numel() * t.element_size()) for t in self._middle.values())
        pb = sum(int(p.data.numel() * 8) for p in self._plain.values() if p.data is not None)
        return {"middle_entries": len(self._middle), "plain_entries": len(self._plain),
                "middle_bytes": mb, "plain_bytes": pb, "total_bytes": mb + pb, **self._stats}

    def clear_cache(self) -> None:
        self._middle.clear()
        self._plain.clear()


# ---------------------------------------------------------------------------
# extended-basis batches (double hoisting): attention input layout
# ---------------------------------------------------------------------------


def fast_rotate(ct: Ciphertext, offsets, context, output_ext: bool = False) -> Ciphertext:
    """Hoisted rotations of ct by every offset as one batch [count, 2, limbs, N].
    output_ext=True leaves them in the extended basis Q_l u P (P times the
    rotation, before ModDown) for grouped_pairwise_mac + moddown_from_ext
    (llama3fhe/operators/attention/input.py:792-797, 1143-1148)."""

    ctx = _ctx_of(context)
    offsets = tuple(int(v) for v in offsets)
    if not offsets:
        raise ValueError("fast_rotate needs at least one offset")
    if not output_ext:
        block = tuple(prepare_hoisted_baby_rotations(ct, offsets, ctx))[0]
        return block
    l = _limbs(ct)
    gal, keys = [], []
    for off in offsets:
        g = galois_element(off, ctx.logN)
        gal.append(g)
        keys.append(None if g == 1 else ctx.rotation_key(off, l)[1])
    ext = ctx.native.modup(ct.data, l) if any(g != 1 for g in gal) else None
    out = ctx.native.rotate_hoisted_ext(ct.data, l, ext, gal, keys)
    return Ciphertext(out, ct.state, ct.slots, ctx, is_ext=True)


def unpack_cipher_batch(batch: Ciphertext) -> tuple[Ciphertext, ...]:
    """The items of a batch as borrowed views (llama3fhe/operators/attention/input.py:798)."""

    if batch.data.dim() == 3:
        return (batch,)
    return tuple(Ciphertext(batch.data[i], batch.state, batch.slots, batch.context,
                            batch.is_ext) for i in range(batch.batch_size))


def pack_cipher_batch(items: Iterable[Ciphertext]) -> Ciphertext:
    """One contiguous batch of same-shape ciphertexts
    (llama3fhe/operators/attention/input.py:810-813, 1142)."""

    items = tuple(items)
    if not items:
        raise ValueError("pack_cipher_batch needs at least one ciphertext")
    first = items[0]
    for it in items:
        if it.data.shape[-2:] != first.data.shape[-2:] or it.is_ext != first.is_ext:
            raise ValueError("pack_cipher_batch: items differ in limbs or basis")
    shape = tuple(first.data.shape[-3:])
    # items may themselves be batches: they are concatenated ciphertext-wise
    data = torch.cat([it.data.reshape((-1,) + shape) for it in items]).contiguous()
    return Ciphertext(data, first.state, first.slots, first.context, first.is_ext)


# ---------------------------------------------------------------------------
# encrypted-state serialisation (resumable runs: limbs + state at a stage
# boundary; the reference has no counterpart of its own)
# ---------------------------------------------------------------------------


def save_ciphertext(ct: Ciphertext, path) -> None:
    """Write a (batch of) ciphertext(s) to `path` (.npz): the uint64 limbs as
    they sit in HBM plus state, slots and basis."""

    import numpy as np

    st = ct.state
    np.savez(path, limbs=ct.data.detach().cpu().numpy(),
             cur_limbs=int(st.cur_limbs), scale_degree=int(st.scale_degree),
             scaling_factor=np.float64(st.scaling_factor if st.scaling_factor is not None
                                       else np.nan),
             slots=int(ct.slots), is_ext=bool(ct.is_ext))


def load_ciphertext(path, context) -> Ciphertext:
    """Read a ciphertext written by save_ciphertext onto the context's device;
    the limb count must match the stored state."""

    import numpy as np

    ctx = _ctx_of(context)
    with np.load(path) as f:
        limbs = f["limbs"]
        sf = float(f["scaling_factor"])
        state = CipherState(int(f["cur_limbs"]), int(f["scale_degree"]),
                            None if np.isnan(sf) else sf)
        slots, is_ext = int(f["slots"]), bool(f["is_ext"])
    expect = state.cur_limbs + (ctx.K if is_ext else 0)
    if limbs.dtype != np.int64 or limbs.shape[-1] != ctx.N or limbs.shape[-2] != expect:
        raise ValueError(f"{path}: limbs {limbs.shape} {limbs.dtype} do not match "
                         f"{expect} limbs of {ctx.N} words")
    data = torch.from_numpy(limbs).to(ctx.device)
    return Ciphertext(data, state, slots, ctx, is_ext)


def grouped_pairwise_mac(batch: Ciphertext, plaintexts: Plaintext, groups: int,
                         context) -> Ciphertext:
    """sum_i batch[i] * plaintexts[i] in `groups` consecutive groups; extended
    batches multiply extended plaintexts over Q_l u P and stay extended
    (llama3fhe/operators/attention/input.py:814-819, 1274-1279)."""

    ctx = _ctx_of(context)
    groups = int(groups)
    count = batch.batch_size
    data = batch.data if batch.data.dim() == 4 else batch.data.unsqueeze(0)
    if plaintexts.rows < count:
        raise ValueError(f"{plaintexts.rows} plaintext rows for {count} ciphertexts")
    l = _limbs(batch)
    pts = plaintexts.cv[0]
    pt_limbs = int(pts.shape[1])
    if batch.is_ext:
        if not plaintexts.is_ext:
            raise ValueError("an extended batch needs extended plaintexts")
        q_limbs, p_limbs = l, ctx.K
        if pt_limbs != l + ctx.K or int(plaintexts.state.cur_limbs) != l:
            raise ValueError("extended plaintexts are not at the batch's level")
    else:
        q_limbs, p_limbs = l, 0
        if int(plaintexts.state.cur_limbs) < l:
            raise ValueError("plaintexts are below the batch's level")
    out = ctx.native.pairwise_mac(data, pts, count, groups, q_limbs, p_limbs, pt_limbs)
    state = batch.state.replace(
        scale_degree=int(batch.state.scale_degree) + int(plaintexts.state.scale_degree),
        scaling_factor=float(batch.state.scaling_factor) * float(plaintexts.state.scaling_factor))
    res = out[0] if groups == 1 else out
    return Ciphertext(res, state, batch.slots, ctx, batch.is_ext)


def moddown_from_ext(ct: Ciphertext, context) -> Ciphertext:
    """ModDown of an extended (batch of) ciphertext(s) to Q_l
    (llama3fhe/operators/attention/input.py:821-826)."""

    ctx = _ctx_of(context)
    if not ct.is_ext:
        return ct.deep_copy()
    l = _limbs(ct)
    data = ct.data if ct.data.dim() == 4 else ct.data.unsqueeze(0)
    out = ctx.native.moddown_ext(data, data.shape[0], l)
    res = out[0] if ct.data.dim() == 3 else out
    return Ciphertext(res, ct.state, ct.slots, ctx, False)
