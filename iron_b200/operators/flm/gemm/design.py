"""Configuration vocabulary of the flm GEMM (iron/operators/flm/gemm/design.py:51-178):
the epilogue and rounding enums (declaration order is the wire format) and the
tile constants IRON's constructor validates against. Nothing here drives the
B200 kernel's own tiling."""

from enum import StrEnum

M_TILE, K_TILE = 64, 512
N_TILE_DEFAULT = 64
CT_MAX_K_FOR_N = {16: 16, 32: 32, 64: 128, 128: 32}
M_CHUNK_FOR_N = {16: 1, 32: 1, 64: 1, 128: 1}
R, S, T = 8, 8, 8
COMPUTE_ROWS = 4  # IRON's NPU2 compute-tile rows; kept for its divisibility contract


class Epilogue(StrEnum):
    """Activation folded into the C drain."""

    NONE = "none"
    GELU = "gelu"
    SILU = "silu"
    SIGMOID = "sigmoid"

    @property
    def mode(self) -> int:
        return list(Epilogue).index(self)


class Rounding(StrEnum):
    """Rounding of every fp32 -> bf16 conversion."""

    CONV_EVEN = "conv_even"
    FLOOR = "floor"
