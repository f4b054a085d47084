"""FastFlowLM-derived operators (iron/operators/flm/__init__.py), lazily exported.

Only ``GEMM`` has a B200 counterpart; the q4nx-to-bfp16 ``DequantBFP`` and the
prebuilt NPU overlay ``MMPrebuilt`` are specific to the AIE2P block-float format
and the shipped NPU binary.
"""

import importlib

_OPERATOR_MODULES = {"GEMM": "gemm"}

__all__ = sorted(_OPERATOR_MODULES)


def __getattr__(name):
    module = _OPERATOR_MODULES.get(name)
    if module is None:
        raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
    return getattr(importlib.import_module(f".{module}.op", __name__), name)


def __dir__():
    return sorted(set(globals()) | set(_OPERATOR_MODULES))
