"""Device-level host layer over libb200fhe: parameters, context, keys, buffers.

Everything here is plumbing around the C ABI: torch provides device memory,
streams and the caching allocator; all arithmetic runs in the CUDA kernels of
libb200fhe.  Residue buffers are torch.int64 tensors holding uint64 values
([polys, limbs, N], limbs contiguous), handed to the library as raw pointers.
"""

from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass, field

import numpy as np
import torch

from . import _native
from ._native import call, lib

LOG_N = 16
N = 1 << LOG_N


def gen_primes(log_n: int, bits: int, count: int, mode: int = 0, exclude=()) -> list[int]:
    out = (ctypes.c_uint64 * max(count, 1))()
    ex = (ctypes.c_uint64 * max(len(exclude), 1))(*[int(v) for v in exclude])
    call("b2f_generate_primes", log_n, bits, count, mode, ex, len(exclude), out)
    return [int(out[i]) for i in range(count)]


@dataclass(frozen=True)
class Params:
    """RNS-CKKS parameter set: Q = q[0..L), special primes P = p[0..K)."""

    log_n: int
    q: tuple[int, ...]
    p: tuple[int, ...]
    dnum: int
    scale_bits: int

    @property
    def L(self) -> int:
        return len(self.q)

    @property
    def K(self) -> int:
        return len(self.p)

    @property
    def alpha(self) -> int:
        return -(-self.L // self.dnum)

    @staticmethod
    def from_depth(depth: int, log_n: int, dnum: int, dcrt_bits: int, first_mod: int,
                   special_bits: int = 60) -> "Params":
        """The layer configuration (assets/feature_major.json): q_0 of
        first_mod bits, depth scaling primes alternating just below / above
        2^dcrt_bits, and enough special primes of special_bits bits for P to
        exceed the largest digit (ceil(digit bits / special_bits))."""

        L = int(depth) + 1
        q0 = gen_primes(log_n, first_mod, 1, 0)
        scaling = gen_primes(log_n, dcrt_bits, L - 1, 1, exclude=q0)
        q = tuple(q0 + scaling)
        alpha = -(-L // int(dnum))
        digit_bits = max(
            sum(math.log2(v) for v in q[j:j + alpha]) for j in range(0, L, alpha)
        )
        K = int(math.ceil(digit_bits / special_bits))
        p = tuple(gen_primes(log_n, special_bits, K, 0, exclude=q))
        return Params(log_n, q, p, int(dnum), int(dcrt_bits))

    @staticmethod
    def uniform(L: int, K: int, dnum: int, bits: int = 50, log_n: int = LOG_N,
                scale_bits: int = 40) -> "Params":
        """L + K primes of `bits` bits, q = 1 mod 2N (the primitive microbench:
        50-bit primes, q = 1 mod 2^17 at N = 2^16)."""

        allp = gen_primes(log_n, bits, L + K, 0)
        return Params(log_n, tuple(allp[:L]), tuple(allp[L:]), int(dnum), int(scale_bits))


def _ptr(t: torch.Tensor) -> int:
    return int(t.data_ptr())


def _stream() -> int:
    """The raw cudaStream_t of the current device's current torch stream
    (torch.cuda.current_stream() costs ~15 us per call in Python)."""

    return torch._C._cuda_getCurrentRawStream(torch._C._cuda_getDevice())


class NativeContext:
    """A libb200fhe context on one CUDA device."""

    def __init__(self, params: Params, device: str | torch.device = "cuda"):
        self.params = params
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("libb200fhe runs on CUDA devices only (no CPU fallback)")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        q = (ctypes.c_uint64 * params.L)(*params.q)
        p = (ctypes.c_uint64 * max(params.K, 1))(*params.p)
        handle = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            call("b2f_context_create", params.log_n, q, params.L, p, params.K, params.dnum,
                 self.device.index, ctypes.byref(handle))
        self.handle = handle
        info = (ctypes.c_int * 6)()
        call("b2f_context_info", self.handle, info)
        self.log_n, self.L, self.K, self.dnum, self.alpha, self.digits = list(info)
        self.n = 1 << self.log_n
        self.primes = list(params.q) + list(params.p)

    def close(self) -> None:
        if getattr(self, "handle", None):
            lib.b2f_context_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- buffers --------------------------------------------------------
    def empty(self, *shape: int) -> torch.Tensor:
        return torch.empty(*shape, self.n, dtype=torch.int64, device=self.device)

    def workspace(self, nbytes: int) -> torch.Tensor:
        return torch.empty(max(int(nbytes), 16), dtype=torch.uint8, device=self.device)

    def key_shape(self) -> tuple[int, int, int, int]:
        return (self.digits, 2, self.L + self.K, self.n)

    # ---- transforms -----------------------------------------------------
    def ntt(self, data: torch.Tensor, q_limbs: int, p_limbs: int = 0,
            inverse: bool = False) -> torch.Tensor:
        limbs = q_limbs + p_limbs
        polys = data.numel() // (limbs * self.n)
        call("b2f_ntt", self.handle, _ptr(data), polys, q_limbs, p_limbs, int(inverse),
             _stream())
        return data

    # ---- keys -----------------------------------------------------------
    def secret_to_ntt(self, s_coeff: np.ndarray) -> torch.Tensor:
        s8 = np.ascontiguousarray(s_coeff, dtype=np.int8)
        out = self.empty(self.L + self.K)
        call("b2f_secret_to_ntt", self.handle, s8.ctypes.data, _ptr(out), _stream())
        return out

    def keygen_rotation(self, s_ntt: torch.Tensor, galois: int, seed: int) -> torch.Tensor:
        key = torch.empty(self.key_shape(), dtype=torch.int64, device=self.device)
        call("b2f_keygen_rotation", self.handle, _ptr(s_ntt), int(galois), int(seed),
             _ptr(key), _stream())
        return key

    def keygen_relin(self, s_ntt: torch.Tensor, seed: int) -> torch.Tensor:
        key = torch.empty(self.key_shape(), dtype=torch.int64, device=self.device)
        call("b2f_keygen_relin", self.handle, _ptr(s_ntt), int(seed), _ptr(key), _stream())
        return key

    def keygen_switch(self, s_from: torch.Tensor, s_to: torch.Tensor, seed: int,
                      tag: int) -> torch.Tensor:
        key = torch.empty(self.key_shape(), dtype=torch.int64, device=self.device)
        call("b2f_keygen_switch", self.handle, _ptr(s_from), _ptr(s_to), int(seed), int(tag),
             _ptr(key), _stream())
        return key

    # ---- (de)cryption -----------------------------------------------------
    def encode(self, values: torch.Tensor, scale: float, q_limbs: int,
               p_limbs: int = 0) -> torch.Tensor:
        """values: complex128 [rows, slots] (or [slots]) on the device."""

        v = values.to(device=self.device, dtype=torch.complex128).contiguous()
        rows = 1 if v.dim() == 1 else v.shape[0]
        slots = v.shape[-1]
        out = self.empty(rows, q_limbs + p_limbs)
        ws = self.workspace(lib.b2f_encode_workspace(self.handle, rows, slots))
        call("b2f_encode", self.handle, _ptr(v), rows, slots, float(scale), q_limbs, p_limbs,
             _ptr(out), _ptr(ws), ws.numel(), _stream())
        return out if v.dim() > 1 else out[0]

    def decode(self, pt: torch.Tensor, l: int, slots: int, scale: float) -> np.ndarray:
        out = torch.empty(slots, dtype=torch.complex128, device=self.device)
        ws = self.workspace(lib.b2f_decode_workspace(self.handle, slots))
        call("b2f_decode", self.handle, _ptr(pt), l, slots, float(scale), _ptr(out), _ptr(ws),
             ws.numel(), _stream())
        return out.cpu().numpy()

    def encrypt(self, m_ntt: torch.Tensor, l: int, s_ntt: torch.Tensor, seed: int,
                nonce: int) -> torch.Tensor:
        ct = self.empty(2, l)
        call("b2f_encrypt", self.handle, _ptr(m_ntt), l, _ptr(s_ntt), int(seed), int(nonce),
             _ptr(ct), _stream())
        return ct

    def decrypt(self, ct: torch.Tensor, l: int, s_ntt: torch.Tensor) -> torch.Tensor:
        m = self.empty(l)
        call("b2f_decrypt", self.handle, _ptr(ct), l, _ptr(s_ntt), _ptr(m), _stream())
        return m

    # ---- evaluation -------------------------------------------------------
    def rotate(self, ct: torch.Tensor, l: int, galois: int, key: torch.Tensor,
               out: torch.Tensor | None = None, ws: torch.Tensor | None = None) -> torch.Tensor:
        num = ct.numel() // (2 * l * self.n)
        if out is None:
            out = torch.empty_like(ct)
        if ws is None:
            ws = self.workspace(lib.b2f_rotate_workspace(self.handle, num, l))
        call("b2f_rotate", self.handle, _ptr(ct), _ptr(out), num, l, int(galois), _ptr(key),
             _ptr(ws), ws.numel(), _stream())
        return out

    def relinearize(self, ct3: torch.Tensor, l: int, key: torch.Tensor) -> torch.Tensor:
        num = ct3.numel() // (3 * l * self.n)
        out = self.empty(num, 2, l) if ct3.dim() == 4 else self.empty(2, l)
        ws = self.workspace(lib.b2f_relinearize_workspace(self.handle, num, l))
        call("b2f_relinearize", self.handle, _ptr(ct3), _ptr(out), num, l, _ptr(key),
             _ptr(ws), ws.numel(), _stream())
        return out

    def relinearize_rescale(self, ct3: torch.Tensor, l: int, key: torch.Tensor,
                            apply_double: bool = False, sub: torch.Tensor | None = None,
                            sub_limbs: int = 0, scalar=None) -> torch.Tensor:
        """Relinearise and rescale in one pass: [.., 3, l, N] -> [.., 2, l-1, N];
        with a post-operation (x2, minus sub's first l-1 limbs, plus the scalar
        residues on poly 0) folded into the final transform's epilogue."""

        num = ct3.numel() // (3 * l * self.n)
        out = self.empty(num, 2, l - 1) if ct3.dim() == 4 else self.empty(2, l - 1)
        ws = self.workspace(lib.b2f_relinearize_rescale_workspace(self.handle, num, l))
        if not apply_double and sub is None and scalar is None:
            call("b2f_relinearize_rescale", self.handle, _ptr(ct3), _ptr(out), num, l,
                 _ptr(key), _ptr(ws), ws.numel(), _stream())
            return out
        res = None
        if scalar is not None:  # the l-1 residues, by value (host array)
            vals = [int(v) for v in scalar][: l - 1]
            if len(vals) != l - 1:
                raise ValueError(f"scalar has {len(vals)} residues, the result {l - 1} limbs")
            res = (ctypes.c_uint64 * (l - 1))(*vals)
        call("b2f_relinearize_rescale_postop", self.handle, _ptr(ct3), _ptr(out), num, l,
             _ptr(key), int(bool(apply_double)), _ptr(sub) if sub is not None else None,
             int(sub_limbs), res, _ptr(ws), ws.numel(),
             _stream())
        return out

    def modup(self, ct: torch.Tensor, l: int, num_cts: int = 1) -> torch.Tensor:
        """ModUp digits of c1: [beta, l+K, N] (one ciphertext) or
        [num_cts, beta, l+K, N]."""

        beta = -(-l // self.alpha)
        ext = self.empty(beta, l + self.K) if num_cts == 1 else \
            self.empty(num_cts * beta, l + self.K).view(num_cts, beta, l + self.K, self.n)
        ws = self.workspace(lib.b2f_modup_batch_workspace(self.handle, num_cts, l))
        call("b2f_modup_batch", self.handle, _ptr(ct), num_cts, l, _ptr(ext), _ptr(ws),
             ws.numel(), _stream())
        return ext

    def rotate_hoisted(self, ct: torch.Tensor, l: int, ext: torch.Tensor, galois, keys,
                       out: torch.Tensor | None = None, num_cts: int = 1) -> torch.Tensor:
        """Hoisted rotations: [count, 2, l, N] (one ciphertext) or
        [num_cts, count, 2, l, N]."""

        count = len(galois)
        if out is None:
            out = self.empty(count, 2, l) if num_cts == 1 else \
                self.empty(num_cts * count, 2, l).view(num_cts, count, 2, l, self.n)
        g = (ctypes.c_uint64 * max(count, 1))(*[int(v) for v in galois])
        kp = (ctypes.c_void_p * max(count, 1))(*[_ptr(k) if k is not None else None
                                                  for k in keys])
        ws = self.workspace(lib.b2f_rotate_hoisted_batch_workspace(self.handle, num_cts,
                                                                   count, l))
        call("b2f_rotate_hoisted_batch", self.handle, _ptr(ct), num_cts, l,
             _ptr(ext) if ext is not None else None, count, g, kp,
             _ptr(out), _ptr(ws), ws.numel(), _stream())
        return out

    def rotate_hoisted_ext(self, ct: torch.Tensor, l: int, ext: torch.Tensor | None, galois,
                           keys) -> torch.Tensor:
        count = len(galois)
        out = self.empty(count, 2, l + self.K)
        g = (ctypes.c_uint64 * max(count, 1))(*[int(v) for v in galois])
        kp = (ctypes.c_void_p * max(count, 1))(*[_ptr(k) if k is not None else None
                                                  for k in keys])
        ws = self.workspace(lib.b2f_rotate_hoisted_ext_workspace(self.handle, count, l))
        call("b2f_rotate_hoisted_ext", self.handle, _ptr(ct), l,
             _ptr(ext) if ext is not None else None, count, g, kp, _ptr(out), _ptr(ws),
             ws.numel(), _stream())
        return out

    def moddown_ext(self, data: torch.Tensor, num_cts: int, l: int) -> torch.Tensor:
        out = self.empty(num_cts, 2, l)
        ws = self.workspace(lib.b2f_moddown_ext_workspace(self.handle, num_cts, l))
        call("b2f_moddown_ext", self.handle, _ptr(data), num_cts, l, _ptr(out), _ptr(ws),
             ws.numel(), _stream())
        return out

    def giant_chain(self, sums: torch.Tensor, extended: bool, num_cts: int, giant_count: int,
                    l: int, giant_galois: int, giant_key: torch.Tensor | None) -> torch.Tensor:
        """Horner over the giant sums [num_cts, G, 2, l (+K if extended), N]
        with the giant rotation, kept in Q_l u P: [num_cts, 2, l, N]."""

        out = self.empty(num_cts, 2, l)
        ws = self.workspace(lib.b2f_giant_chain_workspace(self.handle, num_cts, l))
        call("b2f_giant_chain", self.handle, _ptr(sums), int(bool(extended)), num_cts,
             giant_count, l, int(giant_galois),
             _ptr(giant_key) if giant_key is not None else None, _ptr(out), _ptr(ws),
             ws.numel(), _stream())
        return out

    def pairwise_mac(self, cts: torch.Tensor, pts: torch.Tensor, count: int, groups: int,
                     q_limbs: int, p_limbs: int, pt_limb_stride: int) -> torch.Tensor:
        out = self.empty(groups, 2, q_limbs + p_limbs)
        call("b2f_pairwise_mac", self.handle, _ptr(cts), _ptr(pts), count, groups, q_limbs,
             p_limbs, pt_limb_stride, _ptr(out), _stream())
        return out

    def rescale(self, data: torch.Tensor, num_polys: int, l: int) -> torch.Tensor:
        out = self.empty(num_polys, l - 1)
        ws = self.workspace(lib.b2f_rescale_workspace(self.handle, num_polys, l))
        call("b2f_rescale", self.handle, _ptr(data), _ptr(out), num_polys, l, _ptr(ws),
             ws.numel(), _stream())
        return out

    def modraise(self, data: torch.Tensor, num_polys: int, l_out: int) -> torch.Tensor:
        out = self.empty(num_polys, l_out)
        call("b2f_modraise", self.handle, _ptr(data), num_polys, l_out, _ptr(out), _stream())
        return out

    def drop_limbs(self, data: torch.Tensor, num_polys: int, l_in: int,
                   l_out: int) -> torch.Tensor:
        out = self.empty(num_polys, l_out)
        call("b2f_drop_limbs", self.handle, _ptr(data), _ptr(out), num_polys, l_in, l_out,
             _stream())
        return out

    def elementwise(self, op: int, a: torch.Tensor, b: torch.Tensor, num_polys: int,
                    l: int, b_polys: int | None = None,
                    out: torch.Tensor | None = None) -> torch.Tensor:
        if out is None:
            out = self.empty(num_polys, l)
        call("b2f_elementwise", self.handle, op, _ptr(a), _ptr(b), _ptr(out), num_polys, l,
             num_polys if b_polys is None else b_polys, _stream())
        return out

    @property
    def arith(self) -> str:
        """Arithmetic of the NTT butterflies and the key inner product:
        "int64" or "f64"."""

        return "f64" if lib.b2f_context_arith(self.handle) == 2 else "int64"

    def set_arith(self, mode: str) -> None:
        """"auto" (binary64 when every prime is below 2^50), "int64" or "f64"."""

        codes = {"auto": 0, "int64": 1, "f64": 2}
        if mode not in codes:
            raise ValueError(f"ntt arithmetic {mode!r} not in {sorted(codes)}")
        call("b2f_context_set_arith", self.handle, codes[mode])

    def butterfly_peak(self, iters: int = 2000) -> float:
        """Lazy forward butterflies per second from registers alone, in the
        arithmetic the NTT kernels use (their roofline)."""

        out = ctypes.c_double(0.0)
        call("b2f_butterfly_peak", self.handle, int(iters), ctypes.byref(out), _stream())
        return float(out.value)

    CONV_PATHS = {"auto": 0, "mma_sync": 1, "tcgen05": 2}

    def set_conv_path(self, path: str) -> None:
        """Kernels of the key switch's fast base conversions (ModUp, ModDown):
        'auto' (the default: the faster, the ModDown conversion of 16+
        ciphertexts on tcgen05 with the accumulators in tensor memory, the
        rest on mma.sync), 'mma_sync' or 'tcgen05' for both.  All give
        identical residues."""

        if path not in self.CONV_PATHS:
            raise ValueError(f"conv path {path!r} not in {sorted(self.CONV_PATHS)}")
        call("b2f_set_conv_path", self.handle, self.CONV_PATHS[path])

    GIANT_CHAINS = {"extended": 0, "rotations": 1}

    def set_giant_chain(self, mode: str) -> None:
        """How bsgs_mac runs its Horner chain over the giants: 'extended'
        (the default: the chain stays in Q_l u P, each step ModDowns only
        the poly its key switch reads, one ModDown of both polys at the end)
        or 'rotations' (a full HRotate per giant).  Both decrypt to the same
        values; residues differ by the ModDown rounding."""

        if mode not in self.GIANT_CHAINS:
            raise ValueError(f"giant chain {mode!r} not in {sorted(self.GIANT_CHAINS)}")
        call("b2f_set_giant_chain", self.handle, self.GIANT_CHAINS[mode])
        self._giant_chain = mode

    @property
    def giant_chain_mode(self) -> str:
        return getattr(self, "_giant_chain", "extended")

    MAC_PATHS = {"auto": 0, "cuda_cores": 1}

    def set_mac_path(self, path: str) -> None:
        """'auto': BSGS multiply-accumulates on the u8 tensor cores wherever the
        byte-split sum is exact, else the CUDA cores; 'cuda_cores': always the
        CUDA-core kernel.  Both give identical residues."""

        if path not in self.MAC_PATHS:
            raise ValueError(f"mac path {path!r} not in {sorted(self.MAC_PATHS)}")
        call("b2f_set_mac_path", self.handle, self.MAC_PATHS[path])

    def mac_kernel(self, baby_count: int, q_limbs: int, p_limbs: int = 0,
                   num_cts: int = 2, giant_count: int = 8) -> str:
        """The kernel a MAC of this shape runs (its first launch of up to 8
        giants) under the current path: "mac_mma_kernel" (u8 tensor cores) or
        "mac_kernel" (CUDA cores)."""

        on_tc = lib.b2f_mac_uses_tensor_cores(self.handle, int(baby_count), int(giant_count),
                                              int(q_limbs), int(p_limbs), int(num_cts))
        return "mac_mma_kernel" if on_tc else "mac_kernel"

    def mac_peak(self, iters: int = 2000) -> float:
        """128-bit multiply-adds per second of mac_kernel's inner step from
        registers alone (its integer-multiply roofline)."""

        out = ctypes.c_double(0.0)
        call("b2f_mac_peak", self.handle, int(iters), ctypes.byref(out), _stream())
        return float(out.value)

    def mma_u8_peak(self, iters: int = 2000) -> float:
        """Byte multiply-adds per second of mma.sync m16n8k32 u8 from registers
        alone (the tensor-core MAC's compute roofline)."""

        out = ctypes.c_double(0.0)
        call("b2f_mma_u8_peak", self.handle, int(iters), ctypes.byref(out), _stream())
        return float(out.value)

    def linear_combination(self, terms, term_limbs, weights, num_cts: int, polys: int,
                           l: int) -> torch.Tensor:
        """sum_k weights[k] * terms[k] over num_cts x polys polynomials at l
        limbs; weights[k] is a sequence of l residues."""

        k = len(terms)
        out = self.empty(num_cts * polys, l)
        tp = (ctypes.c_void_p * k)(*[_ptr(t) for t in terms])
        tl = (ctypes.c_int * k)(*[int(v) for v in term_limbs])
        w = (ctypes.c_uint64 * (k * l))(*[int(v) for ws in weights for v in ws[:l]])
        call("b2f_linear_combination", self.handle, k, tp, tl, w, num_cts, polys, l,
             _ptr(out), _stream())
        return out

    def tensor(self, a: torch.Tensor, b: torch.Tensor, num_cts: int, l: int) -> torch.Tensor:
        out = self.empty(num_cts, 3, l)
        call("b2f_tensor", self.handle, _ptr(a), _ptr(b), _ptr(out), num_cts, l, _stream())
        return out

    def mul_i(self, a: torch.Tensor, num_polys: int, l: int, negative: bool = False) -> torch.Tensor:
        out = self.empty(num_polys, l)
        call("b2f_mul_i", self.handle, _ptr(a), _ptr(out), num_polys, l, int(negative),
             _stream())
        return out

    def scalar_op(self, a: torch.Tensor, num_polys: int, l: int, mul=None, add=None,
                  add_poly: int = 0) -> torch.Tensor:
        out = self.empty(num_polys, l)
        m = (ctypes.c_uint64 * l)(*[int(v) for v in mul]) if mul is not None else None
        ad = (ctypes.c_uint64 * l)(*[int(v) for v in add]) if add is not None else None
        call("b2f_scalar_op", self.handle, _ptr(a), _ptr(out), num_polys, l, m, ad, add_poly,
             _stream())
        return out

    def mac(self, babies: torch.Tensor, baby_count: int, pts: torch.Tensor,
            giant_count: int, l: int, num_cts: int = 1) -> torch.Tensor:
        out = self.empty(num_cts, giant_count, 2, l)
        call("b2f_mac", self.handle, _ptr(babies), baby_count, _ptr(pts), giant_count, l,
             _ptr(out), num_cts, _stream())
        return out

    def mac_ext(self, babies: torch.Tensor, baby_count: int, pts: torch.Tensor,
                giant_count: int, q_limbs: int, num_cts: int = 1) -> torch.Tensor:
        """[num_cts, G, 2, q_limbs + K, N] over the extended basis."""

        out = self.empty(num_cts, giant_count, 2, q_limbs + self.K)
        call("b2f_mac_ext", self.handle, _ptr(babies), baby_count, _ptr(pts), giant_count,
             q_limbs, self.K, _ptr(out), num_cts, _stream())
        return out

    def elementwise_ext(self, op: int, a: torch.Tensor, b: torch.Tensor, num_polys: int,
                        q_limbs: int, out: torch.Tensor | None = None) -> torch.Tensor:
        """Limb-wise op on polys over Q_{q_limbs} u P."""

        if out is None:
            out = torch.empty_like(a)
        call("b2f_elementwise_ext", self.handle, op, _ptr(a), _ptr(b), _ptr(out), num_polys,
             q_limbs, self.K, _stream())
        return out

    def bsgs_mac(self, babies: torch.Tensor, baby_count: int, pts: torch.Tensor,
                 giant_count: int, l: int, giant_galois: int,
                 giant_key: torch.Tensor | None, num_cts: int = 1) -> torch.Tensor:
        """[2, l, N] (one ciphertext) or [num_cts, 2, l, N]."""

        out = self.empty(2, l) if num_cts == 1 else \
            self.empty(num_cts * 2, l).view(num_cts, 2, l, self.n)
        ws = self.workspace(lib.b2f_bsgs_mac_batch_workspace(self.handle, num_cts,
                                                             giant_count, l))
        call("b2f_bsgs_mac_batch", self.handle, _ptr(babies), num_cts, baby_count, _ptr(pts),
             giant_count, l, int(giant_galois),
             _ptr(giant_key) if giant_key is not None else None, _ptr(out), _ptr(ws),
             ws.numel(), _stream())
        return out

    def pack_diagonals(self, weight: torch.Tensor, dimension: int, token_lanes: int,
                       baby_steps: int, giant_base: int, giant_count: int,
                       slots: int) -> torch.Tensor:
        w = weight.contiguous()
        if w.dtype == torch.complex128:
            dtype = 2
        elif w.dtype == torch.float32:
            dtype = 1
        else:
            w = w.to(torch.float64)
            dtype = 0
        rows = giant_count * baby_steps
        out = torch.empty(rows, slots, dtype=torch.complex128, device=self.device)
        call("b2f_pack_diagonals", self.handle, _ptr(w), dtype, dimension, token_lanes,
             baby_steps, giant_base, giant_count, slots, _ptr(out), _stream())
        return out

    _STRUCT_MAPS = ("real_source", "real_row", "real_scale", "imag_source", "imag_row",
                    "imag_scale", "column", "column_scale")

    def pack_structured(self, sources, maps: dict, dimension: int, token_lanes: int,
                        baby_steps: int, giant_base: int, giant_count: int,
                        slots: int) -> torch.Tensor:
        """BSGS diagonals read through a StructuredLinearWeight's maps
        (llama3fhe/operators/linear/structured_weight.py:1-20): 1-3 real
        source matrices (float32 or float64, one dtype), int64 index maps and
        float64 scales of length `dimension`.  Host arrays are uploaded."""

        import ctypes

        srcs = [torch.as_tensor(s) for s in sources]
        if not 1 <= len(srcs) <= 3:
            raise ValueError("structured packing takes one to three sources")
        want = torch.float32 if all(s.dtype == torch.float32 for s in srcs) else torch.float64
        srcs = [s.to(device=self.device, dtype=want) for s in srcs]
        if any(s.dim() != 2 for s in srcs):
            raise ValueError("structured sources must be matrices")
        dev = {}
        for name in self._STRUCT_MAPS:
            t = torch.as_tensor(maps[name])
            dt = torch.float64 if name.endswith("scale") else torch.int64
            t = t.to(device=self.device, dtype=dt).contiguous()
            if t.numel() != int(dimension):
                raise ValueError(f"structured map {name} has {t.numel()} entries, "
                                 f"expected {dimension}")
            dev[name] = t
        ptrs = (ctypes.c_void_p * 3)(*([s.data_ptr() for s in srcs] + [0] * (3 - len(srcs))))
        strides = (ctypes.c_int64 * 6)(*([v for s in srcs for v in s.stride()]
                                         + [0] * (6 - 2 * len(srcs))))
        rows = giant_count * baby_steps
        out = torch.empty(rows, slots, dtype=torch.complex128, device=self.device)
        call("b2f_pack_structured", self.handle, ptrs, strides, len(srcs),
             1 if want == torch.float32 else 0,
             *[dev[n].data_ptr() for n in self._STRUCT_MAPS], dimension, token_lanes,
             baby_steps, giant_base, giant_count, slots, _ptr(out), _stream())
        return out


def galois_element(rotation: int, log_n: int = LOG_N) -> int:
    return int(lib.b2f_galois_element(log_n, int(rotation)))


def sample_secret(seed: int, hamming: int, log_n: int = LOG_N) -> np.ndarray:
    s = np.zeros(1 << log_n, dtype=np.int8)
    call("b2f_sample_secret", log_n, int(seed), int(hamming), s.ctypes.data)
    return s


def to_numpy_u64(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().numpy().view(np.uint64)


def from_numpy_u64(a: np.ndarray, device) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.uint64).view(np.int64)).to(device)
