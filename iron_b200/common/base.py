"""Operator base classes with IRON's method surface (iron/common/base.py:33-231).

IRON's operators generate an MLIR-AIE design, compile it to an xclbin and
dispatch it through XRT. On B200 every operator is a thin host wrapper over one
or more entry points of libiron_b200.so: ``compile()`` loads the library (there
is nothing to generate), ``get_arg_spec()`` keeps IRON's buffer contract, and
``get_callable()`` returns ``call(*buffers)`` that launches on the current CUDA
stream. Names keep IRON's mangling, with the device suffix ``b200``.
"""

from __future__ import annotations

import dataclasses
from abc import ABC, abstractmethod
from dataclasses import dataclass
from typing import Any, Callable, ClassVar

import numpy as np

from .context import AIEContext
from .tensor import np_dtype
from .utils import DEVICE_NAME, float_to_name
from .verify import Tolerance

try:
    from ml_dtypes import bfloat16
except ImportError:  # pragma: no cover
    bfloat16 = np.uint16


class AIEOperatorBase(ABC):
    """Root of every operator (iron/common/base.py:33-91)."""

    _default_context: ClassVar[AIEContext | None] = None

    def __init__(self, context: AIEContext | None = None) -> None:
        if context is None:
            context = self.get_default_context()
        self.context = context

    @classmethod
    def get_default_context(cls) -> AIEContext:
        if AIEOperatorBase._default_context is None:
            AIEOperatorBase._default_context = AIEContext()
        return AIEOperatorBase._default_context

    def set_up_artifacts(self) -> None:
        """Nothing to declare: the kernels ship prebuilt in libiron_b200.so."""

    def compile(self, dry_run: bool = False) -> "AIEOperatorBase":
        """Load the CUDA library (IRON compiles the design here, base.py:72-86)."""
        self.set_up_artifacts()
        if not dry_run:
            from .. import _lib

            _lib.load()
        return self

    @abstractmethod
    def get_arg_spec(self) -> list["AIERuntimeArgSpec"]: ...

    @abstractmethod
    def get_callable(self) -> Callable[..., Any]: ...


def _serialize_param(v: object) -> str:
    if isinstance(v, bool):
        return str(int(v))
    if isinstance(v, float):
        return float_to_name(v)
    if isinstance(v, (list, tuple)):
        return "x".join(str(x) for x in v)
    return str(v)


class MLIROperator(AIEOperatorBase):
    """Single-kernel operator (iron/common/base.py:104-209).

    The class keeps IRON's name so ``isinstance`` checks in callers hold.
    Subclasses implement ``_launch(*buffers, stream)``; ``get_callable`` checks
    the buffers against the arg spec and launches.
    """

    _name_aliases: ClassVar[dict[str, str]] = {
        "num_aie_columns": "c",
        "num_channels": "ch",
        "tile_size": "t",
        "size": "sz",
        "scalar_factor": "sf",
        "rows": "r",
        "cols": "n",
    }

    def design_key(self) -> str | None:
        return None

    @property
    def name(self) -> str:
        if not dataclasses.is_dataclass(self):
            raise NotImplementedError(f"{type(self).__name__} must be a @dataclass or override name")
        aliases = type(self)._name_aliases
        parts = (
            f"{aliases.get(f.name, f.name)}{_serialize_param(getattr(self, f.name))}"
            for f in dataclasses.fields(self)
            if f.repr and getattr(self, f.name) is not None
        )
        return f"{type(self).__name__}_{'_'.join(parts)}_{DEVICE_NAME}"

    def runtime_parameters(self) -> list[str]:
        """Names of the int32 runtime parameters this operator reads at launch
        (an OperatorSequence binds each to a device word with ``bind_param``)."""
        return []

    def bind_param(self, name: str, device_word) -> None:
        raise KeyError(f"{type(self).__name__} has no runtime parameter {name!r}")

    def prepare(self) -> None:
        """Allocate whatever the launch needs (workspaces) ahead of a CUDA-graph capture."""

    def reference_tolerance(self) -> Tolerance | None:
        """The tolerance the kernel's output is held to against ``reference()``."""
        return getattr(self, "_tolerance", None)

    # -- dispatch --------------------------------------------------------------
    def _launch(self, *bufs, stream: int) -> None:  # pragma: no cover - abstract
        raise NotImplementedError

    def _check_buffers(self, bufs) -> None:
        specs = self.get_arg_spec()
        if len(bufs) != len(specs):
            raise ValueError(f"{type(self).__name__} takes {len(specs)} buffers, got {len(bufs)}")
        for i, (b, s) in enumerate(zip(bufs, specs)):
            t = getattr(b, "device_tensor", b)
            need = int(np.prod(s.shape, dtype=np.int64)) * np_dtype(s.dtype).itemsize
            have = t.numel() * t.element_size()
            if have < need:
                raise ValueError(f"buffer {i} of {type(self).__name__} holds {have} B, needs {need} B")

    def get_callable(self) -> Callable[..., Any]:
        from .. import _lib

        _lib.load()

        def call(*bufs):
            self._check_buffers(bufs)
            self._launch(*bufs, stream=_lib.current_stream())
            # the kernel rewrote its outputs in HBM: their device copies are now the
            # authoritative ones (a later to("cpu") / to_torch() pulls them)
            for b, spec in zip(bufs, self.get_arg_spec()):
                if spec.direction in ("out", "inout") and hasattr(b, "mark_device_written"):
                    b.mark_device_written()

        return call


class CompositeOperator(AIEOperatorBase):
    """Operator that chains sub-operators (iron/common/base.py:212-216)."""


@dataclass(frozen=True)
class AIERuntimeArgSpec:
    """One runtime buffer of an operator (iron/common/base.py:219-231)."""

    direction: str
    shape: tuple[int, ...]
    dtype: Any = dataclasses.field(default_factory=lambda: bfloat16)

    def __post_init__(self) -> None:
        if self.direction not in {"in", "out", "inout"}:
            raise ValueError(
                f"Invalid direction {self.direction!r}: must be one of 'in', 'out', 'inout'"
            )


# B200-flavoured aliases; the IRON names above stay the public surface.
CUDAOperatorBase = AIEOperatorBase
CUDAOperator = MLIROperator
RuntimeArgSpec = AIERuntimeArgSpec
