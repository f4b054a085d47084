"""StridedCopy on B200 -- iron/operators/strided_copy/op.py:18-100
(golden strided_copy/reference.py:37-75). Decode uses it as the KV-cache append,
with the output offset supplied at run time (``output_offset_parameter``)."""

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
class StridedCopy(MLIROperator):
    """Gather by one access pattern, scatter by another (channel-split innermost dim)."""

    input_sizes: list
    input_strides: list
    input_offset: int
    output_sizes: list
    output_strides: list
    output_offset: int
    input_buffer_size: int = field(repr=False)
    output_buffer_size: int = field(repr=False)
    dtype: object = field(default=bfloat16, repr=False)
    transfer_size: int | None = None
    num_aie_channels: int = 1
    input_offset_parameter: str | None = None
    output_offset_parameter: str | None = None
    kwargs: dict = field(default_factory=dict, repr=False)
    context: object = field(default=None, repr=False)

    _name_aliases: ClassVar[Dict[str, str]] = {
        **MLIROperator._name_aliases,
        "input_sizes": "isz",
        "input_strides": "ist",
        "input_offset": "ioff",
        "output_sizes": "osz",
        "output_strides": "ost",
        "output_offset": "ooff",
        "transfer_size": "tr",
        "num_aie_channels": "ch",
        "input_offset_parameter": "ipar",
        "output_offset_parameter": "opar",
    }
    _tolerance = Tolerance.exact()

    def __post_init__(self):
        if len(self.input_sizes) != len(self.input_strides):
            raise ValueError(
                f"input_sizes and input_strides must have the same length "
                f"({len(self.input_sizes)} vs {len(self.input_strides)})"
            )
        if len(self.output_sizes) != len(self.output_strides):
            raise ValueError(
                f"output_sizes and output_strides must have the same length "
                f"({len(self.output_sizes)} vs {len(self.output_strides)})"
            )
        if len(self.input_sizes) > 4 or len(self.output_sizes) > 4:
            raise ValueError("access patterns have at most 4 dimensions")
        self._params = {}
        MLIROperator.__init__(self, context=self.context)

    def runtime_parameters(self) -> list[str]:
        return [n for n in (self.input_offset_parameter, self.output_offset_parameter) if n]

    def bind_param(self, name: str, device_word) -> None:
        """Read an offset addend (elements) from `device_word` (int32 CUDA tensor) at run time."""
        if name in (self.input_offset_parameter, self.output_offset_parameter):
            self._params[name] = device_word

    def get_arg_spec(self):
        return [
            AIERuntimeArgSpec("in", (int(self.input_buffer_size),), dtype=self.dtype),
            AIERuntimeArgSpec("out", (int(self.output_buffer_size),), dtype=self.dtype),
        ]

    def _launch(self, src, dst, *, stream, flags=0):
        import ctypes

        def arr(v):
            return (ctypes.c_int64 * len(v))(*[int(a) for a in v])

        ia = self._params.get(self.input_offset_parameter)
        oa = self._params.get(self.output_offset_parameter)
        _lib.call("iron_strided_copy", _lib.dptr(src), _lib.dptr(dst), np_dtype(self.dtype).itemsize,
                  len(self.input_sizes), arr(self.input_sizes), arr(self.input_strides),
                  int(self.input_offset), len(self.output_sizes), arr(self.output_sizes),
                  arr(self.output_strides), int(self.output_offset), int(self.num_aie_channels),
                  ia.data_ptr() if ia is not None else None, oa.data_ptr() if oa is not None else None,
                  int(self.input_buffer_size), int(self.output_buffer_size), flags, stream)

    def reference(self, x):
        """Scatter into a zero buffer (the IRON golden's convention)."""
        import torch

        from .reference import reference

        return reference(x.reshape(-1), self.input_sizes, self.input_strides, self.input_offset,
                         self.output_buffer_size, self.output_sizes, self.output_strides,
                         self.output_offset, self.num_aie_channels)
