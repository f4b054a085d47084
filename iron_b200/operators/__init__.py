"""The operator library, re-exported lazily like iron/operators/__init__.py:13-43.

    from iron_b200.operators import GEMV  # imports iron_b200.operators.gemv.op only
"""

import importlib

_OPERATOR_MODULES = {
    "Dequant": "dequant",
    "ElementwiseAdd": "elementwise_add",
    "ElementwiseMul": "elementwise_mul",
    "GEMM": "gemm",
    "GEMV": "gemv",
    "MHA": "mha",
    "RMSNorm": "rms_norm",
    "RoPE": "rope",
    "SiLU": "silu",
    "Softmax": "softmax",
    "SwiGLUDecode": "swiglu_decode",
    "SwiGLUPrefill": "swiglu_prefill",
    "Transpose": "transpose",
    "StridedCopy": "strided_copy",
    "Repeat": "repeat",
    "DecodeAttention": "decode_attention",
}

_SUBPACKAGES = ("flm",)

__all__ = sorted(set(_OPERATOR_MODULES) | set(_SUBPACKAGES))


def __getattr__(name):
    if name in _SUBPACKAGES:
        return importlib.import_module(f".{name}", __name__)
    module = _OPERATOR_MODULES.get(name)
    if module is None:
        raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
    return getattr(importlib.import_module(f".{module}.op", __name__), name)


def __dir__():
    return sorted(set(globals()) | set(_OPERATOR_MODULES) | set(_SUBPACKAGES))
