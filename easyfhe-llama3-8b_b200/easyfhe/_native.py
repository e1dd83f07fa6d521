"""ctypes binding of libb200fhe.so (the C ABI declared in include/b200fhe.h).

The library is required: there is no CPU fallback.  Importing this module
raises ImportError when the shared object has not been built, and every call
raises when the library reports an error (ValueError for argument, shape and
level errors, RuntimeError otherwise), mirroring the exception types the
reference's callers rely on (llama3fhe/operators/nonlinear/bootstrap.py:434
catches ValueError).
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libb200fhe.so"

B2F_OK = 0
B2F_ERR_ARG = 1
B2F_ERR_CUDA = 2
B2F_ERR_NOMEM = 3
B2F_ERR_UNSUPPORTED = 4

_vp = ctypes.c_void_p
_u64 = ctypes.c_uint64
_i64 = ctypes.c_int64
_int = ctypes.c_int
_u32 = ctypes.c_uint32
_dbl = ctypes.c_double
_size = ctypes.c_size_t
_u64p = ctypes.POINTER(ctypes.c_uint64)

# name -> (restype, argtypes)
_SIGS = {
    "b2f_last_error": (ctypes.c_char_p, []),
    "b2f_abi_version": (_int, []),
    "b2f_generate_primes": (_int, [_int, _int, _int, _int, _vp, _int, _vp]),
    "b2f_context_create": (_int, [_int, _vp, _int, _vp, _int, _int, _int, _vp]),
    "b2f_context_destroy": (_int, [_vp]),
    "b2f_context_info": (_int, [_vp, _vp]),
    "b2f_ntt": (_int, [_vp, _vp, _int, _int, _int, _int, _vp]),
    "b2f_automorphism": (_int, [_vp, _vp, _vp, _int, _int, _u64, _vp]),
    "b2f_galois_element": (_u64, [_int, _i64]),
    "b2f_rotate_workspace": (_size, [_vp, _int, _int]),
    "b2f_rotate": (_int, [_vp, _vp, _vp, _int, _int, _u64, _vp, _vp, _size, _vp]),
    "b2f_context_set_arith": (_int, [_vp, _int]),
    "b2f_context_arith": (_int, [_vp]),
    "b2f_relinearize_workspace": (_size, [_vp, _int, _int]),
    "b2f_relinearize": (_int, [_vp, _vp, _vp, _int, _int, _vp, _vp, _size, _vp]),
    "b2f_relinearize_rescale_workspace": (_size, [_vp, _int, _int]),
    "b2f_relinearize_rescale": (_int, [_vp, _vp, _vp, _int, _int, _vp, _vp, _size, _vp]),
    "b2f_relinearize_rescale_postop": (_int, [_vp, _vp, _vp, _int, _int, _vp, _int, _vp, _int,
                                              _vp, _vp, _size, _vp]),
    "b2f_modup_workspace": (_size, [_vp, _int]),
    "b2f_modup": (_int, [_vp, _vp, _int, _vp, _vp, _size, _vp]),
    "b2f_rotate_hoisted_workspace": (_size, [_vp, _int, _int]),
    "b2f_rotate_hoisted": (_int, [_vp, _vp, _int, _vp, _int, _vp, _vp, _vp, _vp, _size,
                                  _vp]),
    "b2f_rotate_hoisted_ext_workspace": (_size, [_vp, _int, _int]),
    "b2f_rotate_hoisted_ext": (_int, [_vp, _vp, _int, _vp, _int, _vp, _vp, _vp, _vp,
                                      _size, _vp]),
    "b2f_moddown_ext_workspace": (_size, [_vp, _int, _int]),
    "b2f_moddown_ext": (_int, [_vp, _vp, _int, _int, _vp, _vp, _size, _vp]),
    "b2f_giant_chain_workspace": (_size, [_vp, _int, _int]),
    "b2f_giant_chain": (_int, [_vp, _vp, _int, _int, _int, _int, _u64, _vp, _vp, _vp, _size,
                               _vp]),
    "b2f_pairwise_mac": (_int, [_vp, _vp, _vp, _int, _int, _int, _int, _int, _vp, _vp]),
    "b2f_rescale_workspace": (_size, [_vp, _int, _int]),
    "b2f_rescale": (_int, [_vp, _vp, _vp, _int, _int, _vp, _size, _vp]),
    "b2f_rescale_noalloc": (_int, [_vp, _vp, _vp, _int, _int, _vp]),
    "b2f_modraise": (_int, [_vp, _vp, _int, _int, _vp, _vp]),
    "b2f_drop_limbs": (_int, [_vp, _vp, _vp, _int, _int, _int, _vp]),
    "b2f_elementwise_ext": (_int, [_vp, _int, _vp, _vp, _vp, _int, _int, _int, _vp]),
    "b2f_elementwise": (_int, [_vp, _int, _vp, _vp, _vp, _int, _int, _int, _vp]),
    "b2f_mul_i": (_int, [_vp, _vp, _vp, _int, _int, _int, _vp]),
    "b2f_scalar_op": (_int, [_vp, _vp, _vp, _int, _int, _vp, _vp, _int, _vp]),
    "b2f_tensor": (_int, [_vp, _vp, _vp, _vp, _int, _int, _vp]),
    "b2f_linear_combination": (_int, [_vp, _int, _vp, _vp, _vp, _int, _int, _int, _vp,
                                      _vp]),
    "b2f_butterfly_peak": (_int, [_vp, _int, ctypes.POINTER(ctypes.c_double), _vp]),
    "b2f_mac_peak": (_int, [_vp, _int, ctypes.POINTER(ctypes.c_double), _vp]),
    "b2f_mma_u8_peak": (_int, [_vp, _int, ctypes.POINTER(ctypes.c_double), _vp]),
    "b2f_modup_batch_workspace": (_size, [_vp, _int, _int]),
    "b2f_modup_batch": (_int, [_vp, _vp, _int, _int, _vp, _vp, _size, _vp]),
    "b2f_rotate_hoisted_batch_workspace": (_size, [_vp, _int, _int, _int]),
    "b2f_rotate_hoisted_batch": (_int, [_vp, _vp, _int, _int, _vp, _int, _vp, _vp, _vp,
                                        _vp, _size, _vp]),
    "b2f_bsgs_mac_batch_workspace": (_size, [_vp, _int, _int, _int]),
    "b2f_bsgs_mac_batch": (_int, [_vp, _vp, _int, _int, _vp, _int, _int, _u64, _vp, _vp,
                                  _vp, _size, _vp]),
    "b2f_bsgs_mac_workspace": (_size, [_vp, _int]),
    "b2f_bsgs_mac": (_int, [_vp, _vp, _int, _vp, _int, _int, _u64, _vp, _vp, _vp, _size,
                            _vp]),
    "b2f_mac": (_int, [_vp, _vp, _int, _vp, _int, _int, _vp, _int, _vp]),
    "b2f_mac_ext": (_int, [_vp, _vp, _int, _vp, _int, _int, _int, _vp, _int, _vp]),
    "b2f_set_mac_path": (_int, [_vp, _int]),
    "b2f_mac_uses_tensor_cores": (_int, [_vp, _int, _int, _int, _int, _int]),
    "b2f_mac_wait_errors": (_int, []),
    "b2f_set_conv_path": (_int, [_vp, _int]),
    "b2f_conv_wait_errors": (_int, []),
    "b2f_set_giant_chain": (_int, [_vp, _int]),
    "b2f_encode": (_int, [_vp, _vp, _int, _int, _dbl, _int, _int, _vp, _vp, _size, _vp]),
    "b2f_encode_workspace": (_size, [_vp, _int, _int]),
    "b2f_decode": (_int, [_vp, _vp, _int, _int, _dbl, _vp, _vp, _size, _vp]),
    "b2f_decode_workspace": (_size, [_vp, _int]),
    "b2f_launch_count": (ctypes.c_ulonglong, []),
    "b2f_pack_diagonals": (_int, [_vp, _vp, _int, _int, _int, _int, _int, _int, _int, _vp,
                                  _vp]),
    "b2f_pack_structured": (_int, [_vp, _vp, _vp, _int, _int, _vp, _vp, _vp, _vp, _vp, _vp,
                                   _vp, _vp, _int, _int, _int, _int, _int, _int, _vp,
                                   _vp]),
    "b2f_secret_to_ntt": (_int, [_vp, _vp, _vp, _vp]),
    "b2f_keygen_switch": (_int, [_vp, _vp, _vp, _u64, _u32, _vp, _vp]),
    "b2f_keygen_rotation": (_int, [_vp, _vp, _u64, _u64, _vp, _vp]),
    "b2f_keygen_relin": (_int, [_vp, _vp, _u64, _vp, _vp]),
    "b2f_encrypt": (_int, [_vp, _vp, _int, _vp, _u64, _u64, _vp, _vp]),
    "b2f_decrypt": (_int, [_vp, _vp, _int, _vp, _vp, _vp]),
    "b2f_sample_secret": (_int, [_int, _u64, _int, _vp]),
}


def _load() -> ctypes.CDLL:
    override = os.environ.get("B200FHE_LIB")
    path = Path(override) if override else LIB_PATH
    if not path.exists():
        raise ImportError(
            f"libb200fhe.so not found at {path}; build it with "
            "`python easyfhe-llama3-8b_b200/build.py` (there is no CPU fallback)"
        )
    lib = ctypes.CDLL(str(path))
    for name, (res, args) in _SIGS.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


class NativeError(RuntimeError):
    pass


def check(rc: int, what: str = "") -> None:
    if rc == B2F_OK:
        return
    msg = (lib.b2f_last_error() or b"").decode(errors="replace")
    text = f"{what}: {msg}" if what else msg
    if rc == B2F_ERR_ARG:
        raise ValueError(text)
    if rc == B2F_ERR_UNSUPPORTED:
        raise NotImplementedError(text)
    if rc == B2F_ERR_NOMEM:
        raise MemoryError(text)
    raise NativeError(text)


def call(name: str, *args) -> None:
    check(getattr(lib, name)(*args), name)


def exported_symbols() -> list[str]:
    return sorted(_SIGS)
