"""GEMV on B200 -- constructor and buffers of iron/operators/gemv/op.py:22-159.

``C = A @ B`` per batch, bf16 in/out, fp32 accumulation (golden
iron/operators/gemv/reference.py:9-11). The AIE tiling knobs
(``num_aie_columns``, ``tile_size_*``, ``kernel_vector_size``) are validated as
IRON validates them and otherwise ignored: the CUDA kernel picks its own tiling.

Two optional fields extend the operator without changing existing calls:
``weight_dtype="int4g32"`` selects the fused int4-unpack + group-scale GEMV
(buffers: packed weights, vector, output; ``GEMV.pack_int4g32`` turns natural
codes + scales into the packed buffer once, as IRON's flm.GEMM ``pack_B`` does)
and ``n_vec`` multiplies one matrix by ``n_vec`` vectors (a decode batch).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import ClassVar, Dict

import numpy as np

from ...common.base import MLIROperator, AIERuntimeArgSpec
from ...common.verify import Tolerance
from ... import _lib


@dataclass
class GEMV(MLIROperator):
    """General matrix-vector product on the B200."""

    M: int
    K: int
    num_aie_columns: int = 1
    tile_size_input: int = 2
    tile_size_output: int | None = None
    num_batches: int = 1
    kernel_vector_size: int = field(default=64, repr=False)
    epilogue: str = field(default="none", repr=False)
    context: object = field(default=None, repr=False)
    weight_dtype: str = field(default="bf16", repr=False)
    n_vec: int = field(default=1, repr=False)

    _name_aliases: ClassVar[Dict[str, str]] = {
        **MLIROperator._name_aliases,
        "num_aie_columns": "col",
        "tile_size_input": "tsi",
        "tile_size_output": "tso",
        "num_batches": "batch",
    }
    _tolerance = Tolerance.relative(0.04, 1e-3)

    def __post_init__(self):
        if self.tile_size_output is None:
            self.tile_size_output = self.tile_size_input
        if not (
            self.tile_size_output % self.tile_size_input == 0
            and self.tile_size_output >= self.tile_size_input
        ):
            raise ValueError("tile_size_output must be a multiple of tile_size_input")
        while self.kernel_vector_size > 16 and self.K < 2 * self.kernel_vector_size:
            self.kernel_vector_size //= 2
        if self.K % self.kernel_vector_size or self.K < 2 * self.kernel_vector_size:
            raise ValueError(
                f"K ({self.K}) must be a multiple of kernel_vector_size "
                f"({self.kernel_vector_size}) and at least twice as large"
            )
        if self.epilogue not in ("none", "gelu"):
            raise ValueError(f"unknown epilogue {self.epilogue!r} (expected 'none' or 'gelu')")
        if self.epilogue == "gelu" and self.tile_size_output % 16 != 0:
            raise ValueError(
                f"gelu epilogue needs tile_size_output % 16 == 0 (got {self.tile_size_output})"
            )
        if self.weight_dtype not in ("bf16", "int4g32", "q4nx"):
            raise ValueError(f"weight_dtype must be 'bf16', 'int4g32' or 'q4nx', got {self.weight_dtype!r}")
        if not 1 <= self.n_vec <= 64:
            raise ValueError(f"n_vec must be in [1, 64], got {self.n_vec}")
        if self.weight_dtype == "q4nx":
            if self.K % 512 or self.M % 64:
                raise ValueError("q4nx GEMV needs K % 512 == 0 and M % 64 == 0")
            if self.n_vec > 8:
                raise ValueError("q4nx GEMV takes at most 8 vectors")
        if self.weight_dtype in ("int4g32", "q4nx"):
            if self.K % 128 or self.M % 16:
                raise ValueError("int4g32 GEMV needs K % 128 == 0 and M % 16 == 0")
            if self.num_batches != 1:
                raise ValueError("int4g32 GEMV takes one matrix (num_batches=1)")
            if self.epilogue != "none":
                raise ValueError("int4g32 GEMV has no activation epilogue")
        MLIROperator.__init__(self, context=self.context)

    @property
    def name(self) -> str:
        base = super().name
        if self.epilogue != "none":
            base = f"{base}_epi{self.epilogue}"
        if self.weight_dtype != "bf16":
            base = f"{base}_w{self.weight_dtype}"
        if self.n_vec != 1:
            base = f"{base}_nv{self.n_vec}"
        return base

    def get_arg_spec(self):
        vec = (self.n_vec,) if self.n_vec > 1 else ()
        if self.weight_dtype in ("int4g32", "q4nx"):
            nbytes = self.packed_bytes(self.M, self.K) * (1280 if self.weight_dtype == "q4nx" else 1152) // 1152
            return [
                AIERuntimeArgSpec("in", (nbytes,), dtype=np.uint8),
                AIERuntimeArgSpec("in", vec + (self.K,)),  # vector(s)
                AIERuntimeArgSpec("out", vec + (self.M,)),  # output
            ]
        batch_dim = (self.num_batches,) if self.num_batches > 1 else ()
        return [
            AIERuntimeArgSpec("in", batch_dim + (self.M, self.K)),  # matrix
            AIERuntimeArgSpec("in", batch_dim + vec + (self.K,)),  # vector(s)
            AIERuntimeArgSpec("out", batch_dim + vec + (self.M,)),  # output
        ]

    # -- int4g32 weights ----------------------------------------------------------
    @staticmethod
    def packed_bytes(M: int, K: int) -> int:
        return (M // 16) * (K // 128) * 1152

    @staticmethod
    def pack_int4g32(codes, scales):
        """Natural codes uint8 [M, K/2] + bf16 scales [M, K/32] (CUDA tensors) ->
        the packed uint8 buffer the int4g32 GEMV streams."""
        import torch

        M, K = codes.shape[0], codes.shape[1] * 2
        out = torch.empty(GEMV.packed_bytes(M, K), dtype=torch.uint8, device=codes.device)
        _lib.call("iron_pack_int4g32", _lib.dptr(codes), _lib.dptr(scales), _lib.dptr(out), M, K,
                  _lib.current_stream())
        return out

    @staticmethod
    def pack_q4nx(blob, K: int, N: int):
        """A q4nx blob (IRON's asymmetric int4: min + scale * code; CUDA uint8) for an
        N x K matrix -> the packed uint8 buffer the q4nx GEMV streams (1280 B units)."""
        import torch

        from .q4nx import q4nx_natural

        codes, scales, mins = q4nx_natural(blob, K, N)
        out = torch.empty((N // 16) * (K // 128) * 1280, dtype=torch.uint8, device=blob.device)
        _lib.call("iron_pack_q4g32", _lib.dptr(codes), _lib.dptr(scales), _lib.dptr(mins), _lib.dptr(out), N, K,
                  _lib.current_stream())
        return out

    def _launch(self, *bufs, stream, residual=None, flags=0):
        p = _lib.dptr
        res = p(residual) if residual is not None else None
        if self.weight_dtype == "q4nx":
            w, x, y = bufs
            _lib.call("iron_gemv_q4g32", p(w), p(x), p(y), self.M, self.K, self.n_vec, res, flags, stream)
            return
        if self.weight_dtype == "int4g32":
            w, x, y = bufs
            _lib.call("iron_gemv_int4g32", p(w), p(x), p(y), self.M, self.K, self.n_vec, res,
                      flags, stream)
            return
        A, x, y = bufs
        epi = _lib.IRON_EPI_GELU if self.epilogue == "gelu" else _lib.IRON_EPI_NONE
        _lib.call("iron_gemv_bf16", p(A), p(x), p(y), self.M, self.K, self.K,
                  self.num_batches, self.M * self.K, self.n_vec * self.K, self.n_vec * self.M,
                  self.n_vec, res, epi, flags, stream)

    def reference(self, *inputs):
        """CPU golden model: (batched) ``A @ B`` (gemv/reference.py:9-11)."""
        from .reference import reference

        return reference(self, *inputs)
