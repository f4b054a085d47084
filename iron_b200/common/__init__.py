"""Common base classes and utilities, mirroring iron/common/__init__.py."""

from .base import (
    AIEOperatorBase,
    MLIROperator,
    CompositeOperator,
    AIERuntimeArgSpec,
    CUDAOperatorBase,
    CUDAOperator,
)
from .context import AIEContext
from .tensor import Tensor, XRTTensor
from .verify import Tolerance, compare, nearly_equal

__all__ = [
    "AIEOperatorBase",
    "MLIROperator",
    "CompositeOperator",
    "AIERuntimeArgSpec",
    "CUDAOperatorBase",
    "CUDAOperator",
    "AIEContext",
    "Tensor",
    "XRTTensor",
    "Tolerance",
    "compare",
    "nearly_equal",
]
