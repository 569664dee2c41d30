"""Loading of the in-tree native extensions.

The CUDA kernels live in ``swarmllm_b200/_C*.so`` and the C++ runtime in
``swarmllm_b200/_native*.so``; both are built in place by
``python setup.py build_ext --inplace`` (see ``__graft_entry__.build``).
There is deliberately no pure-PyTorch fallback for a GPU op: if the extension
is missing on a machine with a GPU, importing an op raises.
"""
from __future__ import annotations

import importlib

_C = None
_NATIVE = None


class ExtensionMissing(ImportError):
    pass


def C():
    global _C
    if _C is None:
        try:
            _C = importlib.import_module("swarmllm_b200._C")
        except ImportError as e:  # pragma: no cover - exercised only without a build
            raise ExtensionMissing(
                "swarmllm_b200._C is not built; run `python setup.py build_ext --inplace`") from e
    return _C


def native():
    global _NATIVE
    if _NATIVE is None:
        try:
            _NATIVE = importlib.import_module("swarmllm_b200._native")
        except ImportError as e:  # pragma: no cover
            raise ExtensionMissing(
                "swarmllm_b200._native is not built; run `python setup.py build_ext --inplace`") from e
    return _NATIVE
