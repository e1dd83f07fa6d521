"""The C-ABI library loads and exports every entry point include/b200fhe.h
declares; argument errors surface through b2f_last_error without touching a
GPU.  Runs on CPU."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def declared() -> set[str]:
    text = (ROOT / "include" / "b200fhe.h").read_text()
    return set(re.findall(r"\b(b2f_[a-z0-9_]+)\s*\(", text))


def test_library_exports_every_declared_symbol():
    from easyfhe import _native

    names = declared()
    assert len(names) >= 30
    for name in names:
        assert hasattr(_native.lib, name), name
    assert set(_native.exported_symbols()) == names


def test_abi_version_and_errors_without_gpu():
    from easyfhe import _native

    assert _native.lib.b2f_abi_version() == 1
    out = (ctypes.c_uint64 * 4)()
    rc = _native.lib.b2f_generate_primes(16, 70, 4, 0, None, 0, out)
    assert rc == _native.B2F_ERR_ARG
    assert b"bad arguments" in _native.lib.b2f_last_error()
    with pytest.raises(ValueError):
        _native.call("b2f_generate_primes", 16, 70, 4, 0, None, 0, out)
    h = ctypes.c_void_p()
    q = (ctypes.c_uint64 * 1)(12289)
    rc = _native.lib.b2f_context_create(12, q, 1, None, 0, 1, 0, ctypes.byref(h))
    assert rc == _native.B2F_ERR_UNSUPPORTED


def test_host_prime_generation_matches_oracle(oracle_mod):
    from easyfhe import core

    assert core.gen_primes(16, 50, 6, 0) == oracle_mod.gen_primes(16, 50, 6, 0)
    assert core.gen_primes(16, 59, 5, 1) == oracle_mod.gen_primes(16, 59, 5, 1)
