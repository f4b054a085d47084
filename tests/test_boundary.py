"""The C-ABI boundary and the host-side operator surface, CPU only.

- libiron_b200.so loads and exports every entry point include/*.h declares, and
  the ctypes table binds exactly those (no compute call is made without a GPU).
- Operators keep IRON's constructor validation (ValueError at construction) and
  arg-spec contract (iron/tests/common/arg_spec_dtype.py:33-127).
"""

import re
from pathlib import Path

import numpy as np
import pytest

from iron_b200 import _lib
from iron_b200.common.base import AIERuntimeArgSpec

REPO = Path(__file__).resolve().parent.parent


def _declared():
    names = set()
    for h in (REPO / "include").glob("*.h"):
        text = h.read_text()
        names |= set(re.findall(r"^\s*(?:int|size_t|const char \*)\s*(iron_\w+)\s*\(", text, re.M))
    return names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    declared = _declared()
    assert declared, "no declarations found"
    for name in sorted(declared):
        assert hasattr(lib, name), f"libiron_b200.so lacks {name}"


def test_ctypes_table_matches_header():
    assert _declared() == set(_lib.SIGNATURES), (
        sorted(_declared() ^ set(_lib.SIGNATURES)))


def test_strerror_and_version():
    assert _lib.strerror(0) == "ok"
    for code in range(-1, -9, -1):
        assert _lib.strerror(code) != "unknown status"
    assert _lib.strerror(-99) == "unknown status"
    assert _lib.load().iron_abi_version() >> 16 == 1


def test_null_pointer_rejected_without_launch():
    # Host-side validation runs before any CUDA call, so this is safe on a CPU box.
    st = _lib.load().iron_gemv_bf16(None, None, None, 16, 16, 16, 1, 0, 0, 0, 1, None, 0, 0, None)
    assert st == -1
    st = _lib.load().iron_gemv_int4g32(16, 32, 16, 16, 100, 1, None, 0, None)  # K % 128
    assert st == -2
    st = _lib.load().iron_gemv_int4g32(16, 32, 16, 24, 128, 1, None, 0, None)  # N % 16
    assert st == -2
    st = _lib.load().iron_dequant_u4(16, 32, 2048, 1024, 33, None)  # odd group
    assert st == -2


def test_gemv_constructor_validation_matches_iron():
    from iron_b200.operators import GEMV

    with pytest.raises(ValueError, match="tile_size_output must be a multiple"):
        GEMV(M=128, K=128, tile_size_input=4, tile_size_output=6)
    with pytest.raises(ValueError, match="kernel_vector_size"):
        GEMV(M=128, K=40)
    with pytest.raises(ValueError, match="unknown epilogue"):
        GEMV(M=128, K=128, epilogue="relu")
    g = GEMV(M=2048, K=64, num_batches=32)  # llama attention-scores shape narrows the vector
    assert g.kernel_vector_size == 32
    assert [s.shape for s in g.get_arg_spec()] == [(32, 2048, 64), (32, 64), (32, 2048)]
    with pytest.raises(ValueError):
        GEMV(M=8192, K=2048, weight_dtype="int4g32", num_batches=2)


def test_operator_names_are_stable():
    from iron_b200.operators import GEMV

    assert GEMV(M=2048, K=8192).name == "GEMV_M2048_K8192_col1_tsi2_tso2_batch1_b200"
    assert GEMV(M=128, K=128, epilogue="gelu", tile_size_output=16,
                tile_size_input=16).name.endswith("_epigelu")


def test_dequant_arg_spec_bytes():
    from iron_b200.operators import Dequant

    op = Dequant(size=2048, num_aie_columns=1, num_channels=2, tile_size=1024)
    (inp, out) = op.get_arg_spec()
    assert inp.shape == (2048 // 2 + 2048 // 32 * 2,) and inp.dtype == np.uint8
    assert out.shape == (2048,)
    with pytest.raises(ValueError):
        Dequant(size=2048, num_aie_columns=8, num_channels=3, tile_size=1024)


def test_arg_spec_direction_validated():
    with pytest.raises(ValueError):
        AIERuntimeArgSpec("sideways", (1,))


def test_lazy_operator_import():
    import importlib
    import sys

    for m in [m for m in sys.modules if m.startswith("iron_b200.operators.")]:
        del sys.modules[m]
    ops = importlib.import_module("iron_b200.operators")
    _ = ops.GEMV
    assert "iron_b200.operators.gemv.op" in sys.modules
    assert "iron_b200.operators.dequant.op" not in sys.modules
