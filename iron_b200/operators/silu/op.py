"""SiLU on B200 -- iron/operators/silu/op.py:12-26 (golden silu/reference.py:7-9)."""

from dataclasses import dataclass, field
from typing import ClassVar

from ...common.operator_bases import ChanneledUnaryOperator


@dataclass
class SiLU(ChanneledUnaryOperator):
    """x * sigmoid(x), element-wise."""

    num_channels: int = field(default=1, init=False, repr=False)
    _eltwise_op: ClassVar[int] = 0

    def reference(self, x):
        import torch

        return torch.nn.functional.silu(x.float()).to(torch.bfloat16)
