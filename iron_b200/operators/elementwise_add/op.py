"""ElementwiseAdd on B200 -- iron/operators/elementwise_add/op.py:12-24."""

from dataclasses import dataclass
from typing import ClassVar

from ...common.operator_bases import BinaryElementwiseOperator


@dataclass
class ElementwiseAdd(BinaryElementwiseOperator):
    """a + b, element-wise."""

    _eltwise_op: ClassVar[int] = 2

    def reference(self, a, b):
        import torch

        return (a.float() + b.float()).to(torch.bfloat16)
