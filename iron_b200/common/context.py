"""Operator context (iron/common/context.py:12-67).

IRON's context selects an MLIR-AIE compiler and build directory. On B200 there is
one prebuilt CUDA library, so the context only keeps the fields callers pass.
"""

from __future__ import annotations

import os
from dataclasses import dataclass, field
from pathlib import Path


@dataclass
class AIEContext:
    build_dir: Path = field(default_factory=lambda: Path(os.getcwd()) / "build")
    mlir_verbose: bool = False
    compiler: str = "nvcc"

    def __post_init__(self) -> None:
        self.build_dir = Path(self.build_dir)
        if self.compiler not in ("nvcc", "peano", "chess"):
            raise ValueError(f"unknown compiler {self.compiler!r}")

    @property
    def compilation_rules(self):
        return []


CUDAContext = AIEContext
