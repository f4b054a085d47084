"""GEMM on B200 -- constructor and buffers of iron/operators/gemm/op.py:21-231.

``C = A @ B`` with bf16 inputs/outputs and fp32 accumulation on the tcgen05
tensor cores (``iron_gemm_bf16``). ``b_col_maj`` / ``c_col_maj`` keep IRON's
storage conventions: B stored (N, K) is the kernel's native K-major operand; B
stored (K, N) is transposed into an operator-owned workspace first (one
``iron_transpose`` launch); C stored (N, M) is produced by swapping the operand
roles (C^T = B A^T), at no extra cost. The AIE tile knobs keep IRON's
divisibility checks (``ValueError`` at construction) and are otherwise ignored.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import ClassVar, Dict

import numpy as np

from ... import _lib
from ...common.base import AIERuntimeArgSpec, MLIROperator
from ...common.verify import Tolerance


@dataclass
class GEMM(MLIROperator):
    """General matrix multiplication on the B200 tensor cores."""

    M: int
    K: int
    N: int
    tile_m: int = 64
    tile_k: int = 64
    tile_n: int = 64
    b_col_maj: bool = False
    c_col_maj: bool = False
    num_aie_columns: int = field(default=8)
    emulate_bf16_mmul_with_bfp16: bool = field(default=True, repr=False)
    prio_accuracy: bool = field(default=False, repr=False)
    round_conv_even: bool = field(default=True, repr=False)
    dtype_in: str = field(default="bf16", repr=False)
    dtype_out: str = field(default="bf16", repr=False)
    use_scalar: bool = field(default=False, repr=False)
    separate_c_tiles: bool = field(default=False, repr=False)
    context: object = field(default=None, repr=False)

    _name_aliases: ClassVar[Dict[str, str]] = {
        **MLIROperator._name_aliases,
        "tile_m": "tm",
        "tile_k": "tk",
        "tile_n": "tn",
        "b_col_maj": "bc",
        "c_col_maj": "cc",
    }
    _tolerance = Tolerance.relative(0.005, 0.005)

    def __post_init__(self):
        rows = 4  # IRON's compute rows; the divisibility contract is kept as is
        for name, value, unit in (("M", self.M, self.tile_m * rows), ("K", self.K, self.tile_k),
                                  ("N", self.N, self.tile_n * self.num_aie_columns)):
            if value % unit != 0:
                raise ValueError(f"{name} ({value}) must be a multiple of {unit}")
        r, s, t = (8, 8, 8) if self.emulate_bf16_mmul_with_bfp16 else (4, 8, 8)
        for name, value, unit in (("tile_m", self.tile_m, 2 * r), ("tile_k", self.tile_k, s),
                                  ("tile_n", self.tile_n, 2 * t)):
            if value % unit != 0:
                raise ValueError(f"{name} ({value}) must be a multiple of {unit}")
        if self.dtype_in != "bf16" or self.dtype_out != "bf16":
            raise ValueError("the B200 GEMM computes bf16 x bf16 -> bf16 (fp32 accumulation)")
        if self.K % 8 or self.N % 8 or self.M % 8:
            raise ValueError("M, K and N must be multiples of 8 (16-byte rows)")
        self._bt = None
        MLIROperator.__init__(self, context=self.context)

    def get_arg_spec(self):
        return [
            AIERuntimeArgSpec("in", (self.M, self.K)),
            AIERuntimeArgSpec("in", (self.N, self.K) if self.b_col_maj else (self.K, self.N)),
            AIERuntimeArgSpec("out", (self.N, self.M) if self.c_col_maj else (self.M, self.N)),
        ]

    def prepare(self):
        if not self.b_col_maj and self._bt is None:
            import torch

            self._bt = torch.empty(self.N, self.K, dtype=torch.bfloat16, device="cuda")

    def _launch(self, A, B, C, *, stream, flags=0):
        p = _lib.dptr
        if self.b_col_maj:
            bk = p(B)
        else:
            self.prepare()
            _lib.call("iron_transpose", p(B), self._bt.data_ptr(), self.K, self.N, 1, 2, flags, stream)
            bk = self._bt.data_ptr()
        M, N, K = self.M, self.N, self.K
        if self.c_col_maj:  # C^T [N, M] = B [N, K] . A [M, K]^T
            _lib.call("iron_gemm_bf16", bk, p(A), p(C), N, M, K, K, K, M, None, 0, 0, 0, 0.0, 0.0, 0, flags, stream)
        else:
            _lib.call("iron_gemm_bf16", p(A), bk, p(C), M, N, K, K, K, N, None, 0, 0, 0, 0.0, 0.0, 0, flags, stream)

    def reference(self, A, B):
        from .reference import reference

        return reference(A.reshape(self.M, self.K), B.reshape(self.get_arg_spec()[1].shape), self.b_col_maj,
                         self.c_col_maj)

    # -- host-side helpers of IRON's operator (op.py:179-231) ----------------------
    def pad_A(self, A_np):
        M, K = A_np.shape
        if M > self.M:
            raise ValueError(f"A rows ({M}) exceeds operator M ({self.M})")
        if M == self.M and K == self.K:
            return A_np
        out = np.zeros((-(-M // self.M) * self.M, self.K), dtype=A_np.dtype)
        out[:M, :K] = A_np
        return out

    def pad_B(self, B_np):
        if self.b_col_maj:
            N, K = B_np.shape
            if N > self.N or K > self.K:
                raise ValueError(f"B (col-major) shape ({N}, {K}) exceeds operator N ({self.N}), K ({self.K})")
            shape = (self.N, self.K)
        else:
            K, N = B_np.shape
            if N > self.N or K > self.K:
                raise ValueError(f"B (row-major) shape ({K}, {N}) exceeds operator K ({self.K}), N ({self.N})")
            shape = (self.K, self.N)
        if B_np.shape == shape:
            return B_np
        out = np.zeros(shape, dtype=B_np.dtype)
        out[: B_np.shape[0], : B_np.shape[1]] = B_np
        return out

    def partition_B(self, B, partition_N):
        """Split B into `partition_N` column blocks of this operator's N, padded."""
        if B is None:
            return [None] * partition_N
        parts = []
        for i in range(partition_N):
            sl = slice(i * self.N, (i + 1) * self.N)
            parts.append(self.pad_B(B[sl, :] if self.b_col_maj else B[:, sl]))
        return parts
