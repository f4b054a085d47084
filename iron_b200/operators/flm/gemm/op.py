"""flm.GEMM on B200 -- constructor, ``pack_B`` and buffers of
iron/operators/flm/gemm/op.py:64-499.

``C = clamp(activation(bf16(A @ B)))`` on the tcgen05 tensor cores with the
epilogue fused into the TMEM drain (``iron_gemm_bf16``). ``pack_B`` reorders a
row-major (K, N) weight matrix into the kernel's consumption order, as IRON's
does for its NPU: here that is K-major (N, K), the layout the tensor-core B
operand reads through a 128-byte-swizzled TMA tile, so no per-call transpose
runs. Tile knobs are resolved and validated as IRON does on NPU2 and do not
steer the B200 kernel.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import ClassVar, Dict

import numpy as np

from .... import _lib
from ....common.base import AIERuntimeArgSpec, MLIROperator
from ....common.verify import Tolerance
from .design import CT_MAX_K_FOR_N, COMPUTE_ROWS, K_TILE, M_CHUNK_FOR_N, M_TILE, Epilogue, Rounding


@dataclass
class GEMM(MLIROperator):
    """bf16 GEMM with a fused activation / clamp epilogue."""

    M: int
    K: int
    N: int
    epilogue: Epilogue = Epilogue.NONE
    epilogue_modes: tuple = tuple(Epilogue)
    clamp: tuple | None = None
    tile_n: int | None = None
    k_tile: int = K_TILE
    tile_ma: int | None = None
    m_chunk: int | None = None
    rounding: Rounding = Rounding.CONV_EVEN
    context: object = field(default=None, repr=False)

    _name_aliases: ClassVar[Dict[str, str]] = {
        **MLIROperator._name_aliases,
        "epilogue": "epi",
        "tile_n": "tn",
        "k_tile": "kt",
        "tile_ma": "ma",
        "m_chunk": "mc",
        "rounding": "rnd",
    }
    _tolerance = Tolerance.relative(0.04, 1e-2)

    def __post_init__(self):
        if self.tile_n is None:
            self.tile_n = 128 if self.K // self.k_tile <= 1 else 64
        elif self.tile_n not in CT_MAX_K_FOR_N:
            raise ValueError(f"tile_n must be one of {sorted(CT_MAX_K_FOR_N)}, got {self.tile_n}")
        if self.m_chunk is None:
            want = M_CHUNK_FOR_N[self.tile_n]
            rows = M_TILE * COMPUTE_ROWS
            blocks = self.M // rows if self.M % rows == 0 else 0
            self.m_chunk = want if blocks and blocks % want == 0 else 1
        if self.tile_ma is None:
            self.tile_ma = M_TILE
        ct_max_k = CT_MAX_K_FOR_N[self.tile_n]
        if self.k_tile % ct_max_k != 0:
            raise ValueError(f"k_tile ({self.k_tile}) must be a multiple of ct_max_k ({ct_max_k}) "
                             f"for tile_n={self.tile_n}")
        for name, value, unit in (("M", self.M, M_TILE * COMPUTE_ROWS), ("K", self.K, self.k_tile),
                                  ("N", self.N, self.tile_n)):
            if value % unit != 0:
                raise ValueError(f"{name} ({value}) must be a multiple of {unit}")
        self.epilogue = Epilogue(self.epilogue)
        self.rounding = Rounding(self.rounding)
        self.epilogue_modes = tuple(dict.fromkeys(Epilogue(m) for m in self.epilogue_modes))
        if self.epilogue is not Epilogue.NONE and self.epilogue not in self.epilogue_modes:
            raise ValueError(f"epilogue {self.epilogue} is not in epilogue_modes "
                             f"{tuple(str(m) for m in self.epilogue_modes)}")
        if self.clamp is not None:
            lo, hi = self.clamp
            if lo > hi:
                raise ValueError(f"clamp min ({lo}) must be <= max ({hi})")
        MLIROperator.__init__(self, context=self.context)

    @property
    def name(self) -> str:
        base = f"FLM_GEMM_tn{self.tile_n}_kt{self.k_tile}_M{self.M}_K{self.K}_N{self.N}_{self.rounding}_b200"
        if self.epilogue != Epilogue.NONE:
            base += f"_epi{self.epilogue}"
        if self.clamp is not None:
            lo, hi = (int(np.float32(v).view(np.int32)) & 0xFFFFFFFF for v in self.clamp)
            base += f"_cl{lo:08x}{hi:08x}"
        return base

    def pack_B(self, B):
        """(K, N) row-major weights -> the kernel's consumption order, K-major (N, K), flat."""
        import torch

        if isinstance(B, np.ndarray):
            B = torch.from_numpy(np.ascontiguousarray(B).view(np.uint16)).view(torch.bfloat16)
        if tuple(B.shape) != (self.K, self.N):
            raise ValueError(f"pack_B expects a ({self.K}, {self.N}) matrix, got {tuple(B.shape)}")
        return B.T.contiguous().reshape(-1)

    def packed_B_size(self, K, N):
        return K * N

    def get_arg_spec(self):
        return [
            AIERuntimeArgSpec("in", (self.M, self.K)),
            AIERuntimeArgSpec("in", (self.K, self.N)),  # holds pack_B's (N, K) order
            AIERuntimeArgSpec("out", (self.M, self.N)),
        ]

    def _launch(self, A, B, C, *, stream, flags=0):
        p = _lib.dptr
        epi = self.epilogue.mode | (_lib.IRON_GEMM_ROUND_FLOOR if self.rounding is Rounding.FLOOR else 0)
        lo, hi = self.clamp if self.clamp is not None else (0.0, 0.0)
        _lib.call("iron_gemm_bf16", p(A), p(B), p(C), self.M, self.N, self.K, self.K, self.K, self.N, None, 0, epi,
                  int(self.clamp is not None), float(lo), float(hi), 0, flags, stream)

    def reference(self, A, B):
        """C = epilogue(A @ B) from the UNPACKED (K, N) B."""
        from .reference import reference

        return reference(A.reshape(self.M, self.K), B.reshape(self.K, self.N), self.epilogue, self.clamp)
