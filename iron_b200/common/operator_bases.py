"""Unary / binary element-wise bases (iron/common/operator_bases.py:22-203).

The AIE column/channel/tile knobs keep IRON's divisibility checks (so shape errors
stay ValueErrors at construction); the CUDA kernels ignore them otherwise.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import ClassVar

from .base import MLIROperator, AIERuntimeArgSpec
from .context import AIEContext
from .verify import Tolerance
from .. import _lib


@dataclass
class ChanneledUnaryOperator(MLIROperator):
    size: int
    num_aie_columns: int
    num_channels: int
    tile_size: int
    context: AIEContext | None = field(default=None, repr=False)

    _eltwise_op: ClassVar[int] = -1
    _tolerance = Tolerance.relative(0.04, 1e-6)

    def __post_init__(self) -> None:
        max_multiple = self.num_aie_columns * self.tile_size
        if self.size % max_multiple != 0:
            raise ValueError(
                f"size ({self.size}) must be a multiple of "
                f"num_aie_columns * tile_size ({max_multiple})"
            )
        super().__init__(context=self.context)

    def get_arg_spec(self):
        return [AIERuntimeArgSpec("in", (self.size,)), AIERuntimeArgSpec("out", (self.size,))]

    def _launch(self, x, y, *, stream, flags=0):
        _lib.call("iron_eltwise", _lib.dptr(x), None, _lib.dptr(y), self.size, self._eltwise_op,
                  flags, stream)


@dataclass
class BinaryElementwiseOperator(MLIROperator):
    size: int
    tile_size: int
    num_aie_columns: int = 8
    context: AIEContext | None = field(default=None, repr=False)

    _name_aliases: ClassVar[dict[str, str]] = {
        **MLIROperator._name_aliases,
        "num_aie_columns": "col",
    }
    _eltwise_op: ClassVar[int] = -1
    _tolerance = Tolerance.relative(0.04, 1e-6)

    def __post_init__(self) -> None:
        if self.size % (self.num_aie_columns * self.tile_size) != 0:
            raise ValueError(
                f"size ({self.size}) must be a multiple of "
                f"num_aie_columns * tile_size ({self.num_aie_columns * self.tile_size})"
            )
        super().__init__(context=self.context)

    def get_arg_spec(self):
        return [
            AIERuntimeArgSpec("in", (self.size,)),
            AIERuntimeArgSpec("in", (self.size,)),
            AIERuntimeArgSpec("out", (self.size,)),
        ]

    def _launch(self, a, b, y, *, stream, flags=0):
        _lib.call("iron_eltwise", _lib.dptr(a), _lib.dptr(b), _lib.dptr(y), self.size,
                  self._eltwise_op, flags, stream)
