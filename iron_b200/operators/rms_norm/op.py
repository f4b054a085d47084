"""RMSNorm on B200 -- iron/operators/rms_norm/op.py:19-122 (golden rms_norm/reference.py:7-16)."""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import ClassVar, Dict

from ...common.base import MLIROperator, AIERuntimeArgSpec
from ...common.verify import Tolerance
from ... import _lib


@dataclass
class RMSNorm(MLIROperator):
    """Row-wise RMS normalization, optionally weighted; rows of `tile_size`."""

    size: int
    num_aie_columns: int
    num_channels: int
    tile_size: int
    weighted: bool = False
    epsilon: float = 1e-5
    context: object = field(default=None, repr=False)

    _name_aliases: ClassVar[Dict[str, str]] = {
        **MLIROperator._name_aliases,
        "weighted": "w",
        "epsilon": "eps",
    }
    _tolerance = Tolerance.relative(0.04, 1e-6)

    def __post_init__(self):
        max_multiple = self.num_aie_columns * self.num_channels * self.tile_size
        if self.size % max_multiple != 0:
            raise ValueError(
                f"size ({self.size}) must be a multiple of "
                f"num_aie_columns * num_channels * tile_size ({max_multiple})"
            )
        MLIROperator.__init__(self, context=self.context)

    def get_arg_spec(self):
        specs = [AIERuntimeArgSpec("in", (self.size // self.tile_size, self.tile_size))]
        if self.weighted:
            specs.append(AIERuntimeArgSpec("in", (self.tile_size,)))
        specs.append(AIERuntimeArgSpec("out", (self.size // self.tile_size, self.tile_size)))
        return specs

    def _launch(self, *bufs, stream, flags=0, residual=None, x_out=None):
        p = _lib.dptr
        if self.weighted:
            x, w, y = bufs
        else:
            (x, y), w = bufs, None
        _lib.call("iron_rmsnorm", p(x), p(residual) if residual is not None else None,
                  p(x_out) if x_out is not None else None, p(w) if w is not None else None, p(y),
                  self.size // self.tile_size, self.tile_size, float(self.epsilon), flags, stream)

    def reference(self, x, w=None):
        import torch

        xf = x.float()
        out = xf / torch.sqrt(torch.mean(xf * xf, dim=-1, keepdim=True) + self.epsilon)
        if self.weighted:
            out = out * w.float()
        return out.to(torch.bfloat16)
