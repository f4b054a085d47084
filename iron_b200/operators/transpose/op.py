"""Transpose on B200 -- iron/operators/transpose/op.py:18-120 (golden transpose/reference.py:7-10)."""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import ClassVar, Dict

from ...common.base import MLIROperator, AIERuntimeArgSpec
from ...common.verify import Tolerance
from ... import _lib


@dataclass
class Transpose(MLIROperator):
    """`num_batches` independent (M, N) -> (N, M) transposes, back to back."""

    M: int
    N: int
    num_aie_columns: int
    num_channels: int
    m: int
    n: int
    s: int
    num_batches: int = 1
    context: object = field(default=None, repr=False)

    _name_aliases: ClassVar[Dict[str, str]] = {
        **MLIROperator._name_aliases,
        "num_batches": "batch",
    }
    _tolerance = Tolerance.exact()

    def __post_init__(self):
        if self.M % self.m != 0:
            raise ValueError(f"Matrix rows ({self.M}) must be a multiple of {self.m}")
        if self.N % self.n != 0:
            raise ValueError(f"Matrix columns ({self.N}) must be a multiple of {self.n}")
        if self.m % self.s != 0:
            raise ValueError(f"AIE tile rows ({self.m}) must be a multiple of {self.s}")
        if self.n % self.s != 0:
            raise ValueError(f"AIE tile columns ({self.n}) must be a multiple of {self.s}")
        if self.M * self.N % (self.m * self.n * self.num_aie_columns * self.num_channels) != 0:
            raise ValueError("Transfer size must be divisible by m*n*num_columns*num_channels")
        if self.N // self.num_aie_columns // self.n < 1:
            raise ValueError(f"num_aie_columns ({self.num_aie_columns}) exceeds N/n ({self.N // self.n})")
        if self.M // self.num_channels // self.m < 1:
            raise ValueError(f"num_channels ({self.num_channels}) exceeds M/m ({self.M // self.m})")
        MLIROperator.__init__(self, context=self.context)

    def get_arg_spec(self):
        batch_dim = (self.num_batches,) if self.num_batches > 1 else ()
        return [
            AIERuntimeArgSpec("in", batch_dim + (self.M * self.N,)),
            AIERuntimeArgSpec("out", batch_dim + (self.N * self.M,)),
        ]

    def _launch(self, x, y, *, stream, flags=0):
        _lib.call("iron_transpose", _lib.dptr(x), _lib.dptr(y), self.M, self.N, self.num_batches, 2,
                  flags, stream)

    def reference(self, x):
        return x.reshape(-1, self.M, self.N).transpose(-2, -1)
