"""``easyfhe.bs`` -- bootstrapping (``easyfhe.bs.openfhe``, the module the
reference imports at llama3fhe/operators/nonlinear/bootstrap.py:16)."""

from . import openfhe  # noqa: F401
