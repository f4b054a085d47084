"""Repeat on B200 -- iron/operators/repeat/op.py:17-69 (golden repeat/reference.py:7-9)."""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import ClassVar, Dict

import numpy as np

from ...common.base import MLIROperator, AIERuntimeArgSpec
from ...common.tensor import np_dtype
from ...common.verify import Tolerance
from ... import _lib

try:
    from ml_dtypes import bfloat16
except ImportError:  # pragma: no cover
    bfloat16 = np.uint16


@dataclass
class Repeat(MLIROperator):
    """repeat_interleave along the leading dimension."""

    rows: int
    cols: int
    repeat: int
    transfer_size: int | None = None
    dtype: object = field(default=bfloat16, repr=False)
    context: object = field(default=None, repr=False)

    _name_aliases: ClassVar[Dict[str, str]] = {
        **MLIROperator._name_aliases,
        "repeat": "by",
        "transfer_size": "ts",
    }
    _tolerance = Tolerance.exact()

    def __post_init__(self):
        MLIROperator.__init__(self, context=self.context)

    def get_arg_spec(self):
        return [
            AIERuntimeArgSpec("in", (self.rows, self.cols), dtype=self.dtype),
            AIERuntimeArgSpec("out", (self.rows * self.repeat, self.cols), dtype=self.dtype),
        ]

    def _launch(self, x, y, *, stream, flags=0):
        row_bytes = self.cols * np_dtype(self.dtype).itemsize
        if row_bytes % 16 == 0:
            _lib.call("iron_repeat_interleave", _lib.dptr(x), _lib.dptr(y), self.rows, row_bytes,
                      self.repeat, flags, stream)
            return
        # rows that are not a whole number of 16-byte vectors: a strided copy per repeat
        import ctypes

        item = np_dtype(self.dtype).itemsize
        for r in range(self.repeat):
            ins = (ctypes.c_int64 * 2)(self.rows, self.cols)
            ist = (ctypes.c_int64 * 2)(self.cols, 1)
            ost = (ctypes.c_int64 * 2)(self.repeat * self.cols, 1)
            _lib.call("iron_strided_copy", _lib.dptr(x), _lib.dptr(y), item, 2, ins, ist, 0, 2, ins,
                      ost, r * self.cols, 1, None, None, self.rows * self.cols,
                      self.rows * self.repeat * self.cols, flags, stream)

    def reference(self, x):
        return x.repeat_interleave(self.repeat, dim=0)
