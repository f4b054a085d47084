"""ElementwiseMul on B200 -- iron/operators/elementwise_mul/op.py:12-24."""

from dataclasses import dataclass
from typing import ClassVar

from ...common.operator_bases import BinaryElementwiseOperator


@dataclass
class ElementwiseMul(BinaryElementwiseOperator):
    """a * b, element-wise."""

    _eltwise_op: ClassVar[int] = 1

    def reference(self, a, b):
        import torch

        return (a.float() * b.float()).to(torch.bfloat16)
