"""RoPE on B200 -- iron/operators/rope/op.py:18-92 (golden rope/reference.py:69-102)."""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import ClassVar, Dict

from ...common.base import MLIROperator, AIERuntimeArgSpec
from ...common.verify import Tolerance
from ... import _lib


@dataclass
class RoPE(MLIROperator):
    """Rotary embedding from an interleaved cos/sin angle table."""

    rows: int
    cols: int
    angle_rows: int | None = None
    num_aie_columns: int = 1
    method_type: int = 0
    context: object = field(default=None, repr=False)

    _name_aliases: ClassVar[Dict[str, str]] = {
        **MLIROperator._name_aliases,
        "num_aie_columns": "col",
        "angle_rows": "arows",
        "method_type": "m",
    }
    _tolerance = Tolerance.relative(0.05)

    def __post_init__(self):
        if self.angle_rows is None:
            self.angle_rows = self.rows
        if not (self.cols % (16 * 2) == 0 and self.cols >= (16 * 2)):
            raise ValueError("cols must be multiple of 32 and >= 32")
        if self.rows % self.num_aie_columns != 0:
            raise ValueError("rows must be divisible by num_aie_columns")
        if not (self.angle_rows <= self.rows and self.rows % self.angle_rows == 0):
            raise ValueError("angle_rows must divide rows")
        if not (self.angle_rows >= self.num_aie_columns and self.angle_rows % self.num_aie_columns == 0):
            raise ValueError("angle_rows must be divisible by num_aie_columns")
        if self.method_type not in {0, 1}:
            raise ValueError(f"method_type must be 0 or 1, got {self.method_type}")
        MLIROperator.__init__(self, context=self.context)

    def get_arg_spec(self):
        return [
            AIERuntimeArgSpec("in", (self.rows, self.cols)),
            AIERuntimeArgSpec("in", (self.angle_rows, self.cols)),
            AIERuntimeArgSpec("out", (self.rows, self.cols)),
        ]

    def _launch(self, x, angles, y, *, stream, flags=0):
        p = _lib.dptr
        _lib.call("iron_rope", p(x), p(angles), None, p(y), self.rows, self.cols, self.angle_rows,
                  None, self.method_type, flags, stream)

    def reference(self, x, angles):
        import torch

        rep = self.rows // angles.shape[0]
        cos = angles[..., 0::2].float().repeat_interleave(rep, dim=0)
        sin = angles[..., 1::2].float().repeat_interleave(rep, dim=0)
        xf = x.float()
        if self.method_type == 0:
            h = x.shape[-1] // 2
            y = torch.cat([xf[..., :h] * cos - xf[..., h:] * sin, xf[..., h:] * cos + xf[..., :h] * sin], -1)
        else:
            y = torch.empty_like(xf)
            y[..., 0::2] = xf[..., 0::2] * cos - xf[..., 1::2] * sin
            y[..., 1::2] = xf[..., 0::2] * sin + xf[..., 1::2] * cos
        return y.to(torch.bfloat16)
