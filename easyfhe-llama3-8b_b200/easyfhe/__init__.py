"""easyfhe -- B200-native drop-in for the EasyFHE surface used by llama3fhe.

The reference imports this package three ways (llama3fhe/backend.py:18-20,
llama3fhe/graph.py:20, llama3fhe/operators/linear/gpu_packer.py:14): as
``easyfhe.fhe`` (CKKS evaluation), as ``easyfhe.bs.openfhe`` (bootstrapping)
and as a torch-like tensor module (``from_numpy``, ``cuda.synchronize``,
``cuda.Event``, ``get_device_module``, dtypes).  The tensor surface is torch
itself; the CKKS surface is implemented by libb200fhe (CUDA, sm_100a) through
``easyfhe.fhe``.
"""

from __future__ import annotations

import torch as _torch

from . import _native  # noqa: F401  (fails loudly when the library is missing)

# ---- tensor bridge (torch is the device-memory and stream plumbing) -------
Tensor = _torch.Tensor
from_numpy = _torch.from_numpy
is_tensor = _torch.is_tensor
cuda = _torch.cuda
float32 = _torch.float32
float64 = _torch.float64
complex64 = _torch.complex64
complex128 = _torch.complex128
int64 = _torch.int64
int32 = _torch.int32
uint8 = _torch.uint8
empty = _torch.empty
zeros = _torch.zeros
tensor = _torch.tensor
device = _torch.device


class _HostModule:
    @staticmethod
    def synchronize() -> None:
        return None

    @staticmethod
    def empty_cache() -> None:
        return None


def get_device_module(device: str = "cuda"):
    """Device module with synchronize()/empty_cache() (backend.py:361-390)."""

    return _torch.cuda if str(device).startswith("cuda") else _HostModule


def __getattr__(name):
    # fhe and bs import torch.cuda state lazily; keep `import easyfhe` cheap
    if name in ("fhe", "bs", "core"):
        import importlib

        return importlib.import_module(f"{__name__}.{name}")
    raise AttributeError(name)
