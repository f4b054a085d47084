"""Softmax on B200 -- iron/operators/softmax/op.py:21-97 (golden softmax/reference.py:9-11).

The row is masked to its first `valid` columns as the device's mask_bf16 does
(iron/operators/softmax/design.py:85-91): `rtp_vector_size` fixes it at
construction, `vector_size_parameter` names a runtime parameter that an
OperatorSequence binds to a device word (``bind_param``).
"""

from __future__ import annotations

from dataclasses import dataclass, field

from ...common.base import MLIROperator, AIERuntimeArgSpec
from ...common.verify import Tolerance
from ... import _lib


@dataclass
class Softmax(MLIROperator):
    """Row softmax, optionally masked to a runtime length."""

    rows: int
    cols: int
    num_aie_columns: int = 1
    num_channels: int = 1
    rtp_vector_size: int | None = None
    vector_size_parameter: str | None = None
    context: object = field(default=None, repr=False)

    _tolerance = Tolerance.relative(0.04, 1e-6)

    @property
    def size(self):
        return self.rows * self.cols

    def __post_init__(self):
        if self.rows % 16 != 0:
            raise ValueError(f"rows ({self.rows}) must be a multiple of 16")
        if self.cols % 16 != 0:
            raise ValueError(f"cols ({self.cols}) must be a multiple of 16")
        if self.rows % self.num_aie_columns != 0:
            raise ValueError(
                f"rows ({self.rows}) must be a multiple of num_aie_columns ({self.num_aie_columns})"
            )
        self._param_dev = None
        MLIROperator.__init__(self, context=self.context)

    def runtime_parameters(self) -> list[str]:
        return [self.vector_size_parameter] if self.vector_size_parameter else []

    def bind_param(self, name: str, device_word) -> None:
        """Read the mask length from `device_word` (an int32 CUDA tensor) at run time."""
        if name == self.vector_size_parameter:
            self._param_dev = device_word

    def get_arg_spec(self):
        return [AIERuntimeArgSpec("in", (self.size,)), AIERuntimeArgSpec("out", (self.size,))]

    def _launch(self, x, y, *, stream, flags=0):
        valid = self.rtp_vector_size if self.rtp_vector_size is not None else self.cols
        pdev = self._param_dev.data_ptr() if self._param_dev is not None else None
        _lib.call("iron_softmax", _lib.dptr(x), _lib.dptr(y), self.rows, self.cols, int(valid), pdev,
                  flags, stream)

    def reference(self, x):
        import torch

        return torch.softmax(x.reshape(self.rows, self.cols).float(), dim=-1).to(torch.bfloat16)
