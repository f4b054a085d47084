"""uint4 Dequant on B200 -- iron/operators/dequant/op.py:20-81.

Payload per tile: ``tile_size/2`` code bytes (element 2k = low nibble, unsigned),
then ``tile_size/group_size`` bf16 scales; output ``bf16(code * scale)``, exact.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from ...common.base import MLIROperator, AIERuntimeArgSpec
from ...common.verify import Tolerance
from ... import _lib

try:
    from ml_dtypes import bfloat16
except ImportError:  # pragma: no cover
    bfloat16 = np.uint16


@dataclass
class Dequant(MLIROperator):
    """Tile-wise uint4 x bf16-scale dequantization."""

    size: int
    num_aie_columns: int
    num_channels: int
    tile_size: int
    group_size: int = field(default=32, repr=False)
    context: object = field(default=None, repr=False)

    _tolerance = Tolerance.exact()

    def __post_init__(self):
        self.input_size = (self.size // 2) + (self.size // self.group_size) * 2
        self.output_size = self.size
        total_cores = self.num_aie_columns * self.num_channels
        if self.size % total_cores != 0:
            raise ValueError(f"size ({self.size}) must be divisible by total cores ({total_cores})")
        if total_cores > 16:
            raise ValueError(f"total cores ({total_cores}) must be <= 16")
        if self.group_size % 2 or self.tile_size % self.group_size or self.size % self.tile_size:
            raise ValueError("size must be a multiple of tile_size, tile_size of an even group_size")
        MLIROperator.__init__(self, context=self.context)

    def get_arg_spec(self):
        return [
            AIERuntimeArgSpec("in", (self.input_size,), dtype=np.uint8),
            AIERuntimeArgSpec("out", (self.output_size,), dtype=bfloat16),
        ]

    def _launch(self, payload, out, *, stream):
        _lib.call("iron_dequant_u4", _lib.dptr(payload), _lib.dptr(out), self.size,
                  self.tile_size, self.group_size, stream)

    def reference(self, payload):
        from .reference import reference

        return reference(payload, self.tile_size, self.group_size)
