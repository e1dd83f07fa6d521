"""ctypes binding of the CPU oracle (ckks_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, ``__graft_entry__.smoke()`` and
bench.py's CPU-baseline / reference arm, never by the product package.
Residue parity against the reference's EasyFHE is unpinned (the library is not
in the reference tree); ckks_oracle.h lists what pins this restatement.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "build" / "libckks_oracle.so"

_u64p = ctypes.POINTER(ctypes.c_uint64)
_i64p = ctypes.POINTER(ctypes.c_int64)
_i32p = ctypes.POINTER(ctypes.c_int32)
_dp = ctypes.POINTER(ctypes.c_double)


def build(force: bool = False) -> Path:
    src = HERE / "ckks_oracle.c"
    if force or not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = ctypes.CDLL(str(LIB_PATH))
        L.orc_is_prime.argtypes = [ctypes.c_uint64]
        L.orc_is_prime.restype = ctypes.c_int
        L.orc_find_psi.argtypes = [ctypes.c_uint64, ctypes.c_int]
        L.orc_find_psi.restype = ctypes.c_uint64
        L.orc_gen_primes.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                     _u64p, ctypes.c_int, _u64p]
        L.orc_gen_primes.restype = ctypes.c_int
        L.orc_chacha_block.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, _u64p]
        L.orc_ctx_create.argtypes = [ctypes.c_int, _u64p, ctypes.c_int, _u64p, ctypes.c_int,
                                     ctypes.c_int]
        L.orc_ctx_create.restype = ctypes.c_void_p
        L.orc_ctx_free.argtypes = [ctypes.c_void_p]
        L.orc_alpha.argtypes = [ctypes.c_void_p]
        L.orc_num_digits.argtypes = [ctypes.c_void_p]
        L.orc_ntt_forward.argtypes = [ctypes.c_void_p, _u64p, ctypes.c_int]
        L.orc_ntt_inverse.argtypes = [ctypes.c_void_p, _u64p, ctypes.c_int]
        L.orc_poly_ntt.argtypes = [ctypes.c_void_p, _u64p, ctypes.c_int, ctypes.c_int,
                                   ctypes.c_int, ctypes.c_int]
        L.orc_automorphism_perm.argtypes = [ctypes.c_int, ctypes.c_uint64, _i32p]
        L.orc_galois_element.argtypes = [ctypes.c_int, ctypes.c_int64]
        L.orc_galois_element.restype = ctypes.c_uint64
        L.orc_modup_digit.argtypes = [ctypes.c_void_p, _u64p, ctypes.c_int, ctypes.c_int, _u64p]
        L.orc_keyswitch.argtypes = [ctypes.c_void_p, _u64p, ctypes.c_int, _u64p, _u64p, _u64p]
        L.orc_rotate.argtypes = [ctypes.c_void_p, _u64p, ctypes.c_int, ctypes.c_uint64, _u64p,
                                 _u64p]
        L.orc_rotate_hoisted.argtypes = [ctypes.c_void_p, _u64p, ctypes.c_int, ctypes.c_int,
                                         _u64p, ctypes.POINTER(_u64p), _u64p]
        L.orc_rotate_hoisted_ext.argtypes = [ctypes.c_void_p, _u64p, ctypes.c_int,
                                             ctypes.c_int, _u64p, ctypes.POINTER(_u64p),
                                             _u64p]
        L.orc_moddown.argtypes = [ctypes.c_void_p, _u64p, ctypes.c_int, ctypes.c_int, _u64p]
        L.orc_rescale.argtypes = [ctypes.c_void_p, _u64p, ctypes.c_int, ctypes.c_int, _u64p]
        L.orc_relin_rescale.argtypes = [ctypes.c_void_p, _u64p, ctypes.c_int, _u64p, _u64p]
        L.orc_modraise.argtypes = [ctypes.c_void_p, _u64p, ctypes.c_int, ctypes.c_int, _u64p]
        L.orc_mul_i.argtypes = [ctypes.c_void_p, _u64p, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.orc_sample_secret.argtypes = [ctypes.c_int, ctypes.c_uint64, ctypes.c_int, _i64p]
        L.orc_secret_to_ntt.argtypes = [ctypes.c_void_p, _i64p, _u64p]
        L.orc_keygen_switch.argtypes = [ctypes.c_void_p, _u64p, _u64p, ctypes.c_uint64,
                                        ctypes.c_uint32, _u64p]
        L.orc_keygen_rotation.argtypes = [ctypes.c_void_p, _u64p, ctypes.c_uint64,
                                          ctypes.c_uint64, _u64p]
        L.orc_keygen_relin.argtypes = [ctypes.c_void_p, _u64p, ctypes.c_uint64, _u64p]
        L.orc_encrypt.argtypes = [ctypes.c_void_p, _u64p, ctypes.c_int, _u64p, ctypes.c_uint64,
                                  ctypes.c_uint64, _u64p]
        L.orc_decrypt.argtypes = [ctypes.c_void_p, _u64p, ctypes.c_int, _u64p, _u64p]
        L.orc_encode.argtypes = [ctypes.c_void_p, _dp, _dp, ctypes.c_int, ctypes.c_double,
                                 ctypes.c_int, ctypes.c_int, _u64p]
        L.orc_decode.argtypes = [ctypes.c_void_p, _u64p, ctypes.c_int, ctypes.c_int,
                                 ctypes.c_double, _dp, _dp]
        L.orc_special_fft.argtypes = [ctypes.c_int, _dp, _dp, ctypes.c_int, ctypes.c_int]
        L.orc_bsgs_mac.argtypes = [ctypes.c_void_p, _u64p, ctypes.c_int, ctypes.c_int, _u64p,
                                   ctypes.c_int, ctypes.c_int, ctypes.c_int, _u64p]
        L.orc_mul_plain.argtypes = [ctypes.c_void_p, _u64p, _u64p, ctypes.c_int, ctypes.c_int,
                                    _u64p]
        _lib = L
    return _lib


def _p(a: np.ndarray, kind=_u64p):
    return a.ctypes.data_as(kind)


def _u64(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.uint64)


def is_prime(n: int) -> bool:
    return bool(lib().orc_is_prime(int(n)))


def find_psi(q: int, log_n: int) -> int:
    return int(lib().orc_find_psi(int(q), int(log_n)))


def gen_primes(log_n: int, bits: int, count: int, mode: int = 0, exclude=()) -> list[int]:
    out = np.zeros(count, dtype=np.uint64)
    ex = _u64(list(exclude) or [0])
    rc = lib().orc_gen_primes(log_n, bits, count, mode, _p(ex), len(exclude), _p(out))
    if rc:
        raise ValueError("not enough primes")
    return [int(v) for v in out]


def chacha_block(seed: int, stream: int, counter: int) -> np.ndarray:
    out = np.zeros(8, dtype=np.uint64)
    lib().orc_chacha_block(seed, stream, counter, _p(out))
    return out


def galois_element(log_n: int, rotation: int) -> int:
    return int(lib().orc_galois_element(log_n, int(rotation)))


def automorphism_perm(log_n: int, g: int) -> np.ndarray:
    out = np.zeros(1 << log_n, dtype=np.int32)
    lib().orc_automorphism_perm(log_n, int(g), _p(out, _i32p))
    return out


def special_fft(log_n: int, re, im, inverse: bool):
    re = np.array(re, dtype=np.float64)
    im = np.array(im, dtype=np.float64)
    lib().orc_special_fft(log_n, _p(re, _dp), _p(im, _dp), len(re), int(inverse))
    return re, im


def sample_secret(log_n: int, seed: int, hamming: int) -> np.ndarray:
    s = np.zeros(1 << log_n, dtype=np.int64)
    lib().orc_sample_secret(log_n, seed, hamming, _p(s, _i64p))
    return s


class Oracle:
    """CPU CKKS context over Q = q[0..L) and P = p[0..K) (test use only)."""

    def __init__(self, log_n: int, q, p, dnum: int):
        self.log_n = int(log_n)
        self.n = 1 << self.log_n
        self.q = [int(v) for v in q]
        self.p = [int(v) for v in p]
        self.L = len(self.q)
        self.K = len(self.p)
        self.dnum = int(dnum)
        qa, pa = _u64(self.q), _u64(self.p or [0])
        self._h = lib().orc_ctx_create(self.log_n, _p(qa), self.L, _p(pa), self.K, self.dnum)
        self.alpha = int(lib().orc_alpha(self._h))
        self.digits = int(lib().orc_num_digits(self._h))

    def close(self):
        if self._h:
            lib().orc_ctx_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def primes(self) -> list[int]:
        return self.q + self.p

    def ntt(self, data: np.ndarray, q_limbs: int, p_limbs: int = 0, inverse=False) -> np.ndarray:
        a = _u64(data).copy()
        limbs = q_limbs + p_limbs
        polys = a.size // (limbs * self.n)
        lib().orc_poly_ntt(self._h, _p(a), polys, q_limbs, p_limbs, int(inverse))
        return a

    def modup_digit(self, x_coeff: np.ndarray, l: int, digit: int) -> np.ndarray:
        out = np.zeros((l + self.K, self.n), dtype=np.uint64)
        lib().orc_modup_digit(self._h, _p(_u64(x_coeff)), l, digit, _p(out))
        return out

    def keyswitch(self, c1: np.ndarray, l: int, key: np.ndarray):
        d0 = np.zeros((l, self.n), dtype=np.uint64)
        d1 = np.zeros((l, self.n), dtype=np.uint64)
        lib().orc_keyswitch(self._h, _p(_u64(c1)), l, _p(_u64(key)), _p(d0), _p(d1))
        return d0, d1

    def rotate(self, ct: np.ndarray, l: int, g: int, key: np.ndarray) -> np.ndarray:
        out = np.zeros((2, l, self.n), dtype=np.uint64)
        lib().orc_rotate(self._h, _p(_u64(ct)), l, int(g), _p(_u64(key)), _p(out))
        return out

    def rotate_hoisted(self, ct: np.ndarray, l: int, galois, keys) -> np.ndarray:
        count = len(galois)
        out = np.zeros((count, 2, l, self.n), dtype=np.uint64)
        g = _u64(galois)
        keys = [_u64(k) for k in keys]
        arr = (_u64p * count)(*[_p(k) for k in keys])
        lib().orc_rotate_hoisted(self._h, _p(_u64(ct)), l, count, _p(g), arr, _p(out))
        return out

    def rotate_hoisted_ext(self, ct: np.ndarray, l: int, galois, keys) -> np.ndarray:
        count = len(galois)
        out = np.zeros((count, 2, l + self.K, self.n), dtype=np.uint64)
        g = _u64(galois)
        keys = [_u64(k) if k is not None else np.zeros(1, dtype=np.uint64) for k in keys]
        arr = (_u64p * count)(*[_p(k) for k in keys])
        lib().orc_rotate_hoisted_ext(self._h, _p(_u64(ct)), l, count, _p(g), arr, _p(out))
        return out

    def relin_rescale(self, ct3: np.ndarray, l: int, key: np.ndarray) -> np.ndarray:
        """Relinearise (3 x l limbs) and rescale in one division by P q_{l-1}."""

        out = np.zeros((2, l - 1, self.n), dtype=np.uint64)
        lib().orc_relin_rescale(self._h, _p(_u64(ct3)), l, _p(_u64(key)), _p(out))
        return out

    def moddown(self, data: np.ndarray, num_polys: int, l: int) -> np.ndarray:
        out = np.zeros((num_polys, l, self.n), dtype=np.uint64)
        lib().orc_moddown(self._h, _p(_u64(data)), num_polys, l, _p(out))
        return out

    def rescale(self, data: np.ndarray, num_polys: int, l: int) -> np.ndarray:
        out = np.zeros((num_polys, l - 1, self.n), dtype=np.uint64)
        lib().orc_rescale(self._h, _p(_u64(data)), num_polys, l, _p(out))
        return out

    def modraise(self, data: np.ndarray, num_polys: int, l_out: int) -> np.ndarray:
        out = np.zeros((num_polys, l_out, self.n), dtype=np.uint64)
        lib().orc_modraise(self._h, _p(_u64(data)), num_polys, l_out, _p(out))
        return out

    def mul_i(self, data: np.ndarray, num_polys: int, l: int, negative=False) -> np.ndarray:
        a = _u64(data).copy()
        lib().orc_mul_i(self._h, _p(a), num_polys, l, int(negative))
        return a

    def secret_to_ntt(self, s: np.ndarray) -> np.ndarray:
        out = np.zeros((self.L + self.K, self.n), dtype=np.uint64)
        lib().orc_secret_to_ntt(self._h, _p(np.ascontiguousarray(s, dtype=np.int64), _i64p),
                                _p(out))
        return out

    def key_shape(self):
        return (self.digits, 2, self.L + self.K, self.n)

    def keygen_switch(self, s_from, s_to, seed: int, tag: int) -> np.ndarray:
        key = np.zeros(self.key_shape(), dtype=np.uint64)
        lib().orc_keygen_switch(self._h, _p(_u64(s_from)), _p(_u64(s_to)), seed, tag, _p(key))
        return key

    def keygen_rotation(self, s_ntt, g: int, seed: int) -> np.ndarray:
        key = np.zeros(self.key_shape(), dtype=np.uint64)
        lib().orc_keygen_rotation(self._h, _p(_u64(s_ntt)), int(g), seed, _p(key))
        return key

    def keygen_relin(self, s_ntt, seed: int) -> np.ndarray:
        key = np.zeros(self.key_shape(), dtype=np.uint64)
        lib().orc_keygen_relin(self._h, _p(_u64(s_ntt)), seed, _p(key))
        return key

    def encrypt(self, m_ntt, l: int, s_ntt, seed: int, nonce: int) -> np.ndarray:
        ct = np.zeros((2, l, self.n), dtype=np.uint64)
        lib().orc_encrypt(self._h, _p(_u64(m_ntt)), l, _p(_u64(s_ntt)), seed, nonce, _p(ct))
        return ct

    def decrypt(self, ct, l: int, s_ntt) -> np.ndarray:
        m = np.zeros((l, self.n), dtype=np.uint64)
        lib().orc_decrypt(self._h, _p(_u64(ct)), l, _p(_u64(s_ntt)), _p(m))
        return m

    def encode(self, values, scale: float, q_limbs: int, p_limbs: int = 0) -> np.ndarray:
        v = np.asarray(values, dtype=np.complex128).reshape(-1)
        re = np.ascontiguousarray(v.real)
        im = np.ascontiguousarray(v.imag)
        out = np.zeros((q_limbs + p_limbs, self.n), dtype=np.uint64)
        lib().orc_encode(self._h, _p(re, _dp), _p(im, _dp), len(v), float(scale), q_limbs,
                         p_limbs, _p(out))
        return out

    def decode(self, m_ntt, l: int, slots: int, scale: float) -> np.ndarray:
        re = np.zeros(slots, dtype=np.float64)
        im = np.zeros(slots, dtype=np.float64)
        lib().orc_decode(self._h, _p(_u64(m_ntt)), l, slots, float(scale), _p(re, _dp),
                         _p(im, _dp))
        return re + 1j * im

    def mul_plain(self, ct, pt, l: int) -> np.ndarray:
        out = np.zeros((2, l, self.n), dtype=np.uint64)
        lib().orc_mul_plain(self._h, _p(_u64(ct)), _p(_u64(pt)), l, 0, _p(out))
        return out

    def bsgs_mac(self, babies, num_cts: int, baby_count: int, pts, giant_count: int,
                 l: int, p_limbs: int = 0) -> np.ndarray:
        """[C, G, 2, l + p_limbs, N]: out[c][g] = sum_b pts[g B + b] * babies[c][b]
        over Q_l (u P when p_limbs > 0)."""

        out = np.zeros((num_cts, giant_count, 2, l + p_limbs, self.n), dtype=np.uint64)
        lib().orc_bsgs_mac(self._h, _p(_u64(babies)), num_cts, baby_count, _p(_u64(pts)),
                           giant_count, l, p_limbs, _p(out))
        return out

    def giant_chain_ext(self, inner, giant_count: int, l: int, g: int, key,
                        extended: bool = False) -> np.ndarray:
        """The BSGS giant sum sum_j rot_{j G}(inner[j]) by Horner with the one
        giant key (llama3fhe/operators/linear/config.py:292-305: `normal` and
        `ext_normal` repeat one giant rotation key within a chunk), the chain
        kept in Q_l u P.  Each step ModDowns only the state's second poly,
        key-switches that with the giant key into Q_l u P (P times the
        result, no ModDown) and adds the automorphism of the state's first
        poly; the next giant's sum joins (P times a Q_l sum on the Q limbs, or
        an extended sum as it is); one ModDown of both polys ends the chain.
        A Q_l top sum is its own second poly after the ModDown, so its first
        step is rotate_hoisted_ext itself.
        inner [G, 2, l, N] (extended: [G, 2, l+K, N], P times the sums) ->
        [2, l, N]."""

        G, n = int(giant_count), self.n
        primes = self.q[:l] + self.p
        q = np.array(primes, dtype=object)[:, None]
        pm = np.array([int(np.prod([p % qi for p in self.p], dtype=object) % qi)
                       for qi in self.q[:l]], dtype=object)[:, None]
        perm = automorphism_perm(self.log_n, g)
        key = _u64(key)

        def plus(state, ct):  # + the next giant's sum
            out = state.astype(object)
            if extended:
                out = (out + ct.astype(object)) % q[None]
            else:  # P ct on the Q limbs (P = 0 mod p_k)
                out[:, :l] = (out[:, :l] + pm[None] * ct.astype(object)) % q[None, :l]
            return out.astype(np.uint64)

        if extended:
            state, first = _u64(inner[G - 1]).copy(), G - 2
        else:
            state = plus(self.rotate_hoisted_ext(inner[G - 1], l, [g], [key])[0], inner[G - 2])
            first = G - 3
        for j in range(first, -1, -1):
            c1 = self.moddown(state[1][None], 1, l)[0]
            zero_c0 = np.stack([np.zeros((l, n), dtype=np.uint64), c1])
            r = self.rotate_hoisted_ext(zero_c0, l, [g], [key])[0]
            r0 = (r[0].astype(object) + state[0][:, perm].astype(object)) % q
            state = plus(np.stack([r0.astype(np.uint64), r[1]]), inner[j])
        return self.moddown(state, 2, l)
