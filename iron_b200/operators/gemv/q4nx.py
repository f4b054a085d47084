"""q4nx weights (IRON's asymmetric int4 format: min + scale * code) for the q4 GEMV.

IRON keeps FastFlowLM's q4nx blobs as the input of its flm.DequantBFP operator
(iron/operators/flm/dequant/README.md, input layers 1-9; op iron/operators/flm/dequant/
op.py). Blocks of 32 out-features x 256 in-features hold 512 B of bf16 group scales
[8 groups][32 n], 512 B of bf16 group mins and 4096 B of codes (byte = the codes of two
adjacent n at one k, even n in the low nibble; 16 n per 8-byte slice); block i sits at
column block cb, k tile kb, k half, n half with i = ((cb * K/512 + kb) * 2 + k_half) * 2 +
n_half (iron/operators/flm/dequant/reference.py:40-77 walks the same order).

`q4nx_natural` turns a blob (a CUDA uint8 tensor) into natural arrays with torch index
arithmetic on the device -- codes [N, K/2] (two k per byte, even k low), scales and
mins bf16 [N, K/32] -- which `iron_pack_q4g32` repacks into the GEMV's streaming units.
The GEMV multiplies bf16(min + scale * code), the fp32 value of IRON's dequantization
rounded once to bf16 (the bfp16 conversion of IRON's AIE path is out of scope here).
"""

from __future__ import annotations

import torch

M_TILE, K_TILE, GROUP, K_TILE_B, PAR = 32, 256, 32, 512, 16
BLOCK_BYTES = M_TILE * K_TILE * 5 // 8


def q4nx_bytes(K: int, N: int) -> int:
    return N * K * 5 // 8


def q4nx_natural(blob: torch.Tensor, K: int, N: int):
    """q4nx blob (uint8, CUDA) -> (codes uint8 [N, K/2], scales bf16 [N, K/32], mins bf16
    [N, K/32]); K % 512 == 0, N % 64 == 0."""
    if K % K_TILE_B or N % (2 * M_TILE):
        raise ValueError(f"q4nx needs K % {K_TILE_B} == 0 and N % {2 * M_TILE} == 0, got K={K}, N={N}")
    if blob.numel() != q4nx_bytes(K, N):
        raise ValueError(f"q4nx blob of {blob.numel()} bytes, expected {q4nx_bytes(K, N)} for K={K}, N={N}")
    ng = K_TILE // GROUP
    cbs, kts = N // (2 * M_TILE), K // K_TILE_B
    b = blob.reshape(cbs, kts, 2, 2, BLOCK_BYTES)  # cb, kb, k_half, n_half, bytes
    sm = ng * M_TILE * 2

    def groups(part):  # [cb, kb, kh, nh, g, n] bf16 -> [N, K/32]
        t = part.contiguous().view(torch.bfloat16).reshape(cbs, kts, 2, 2, ng, M_TILE)
        return t.permute(0, 3, 5, 1, 2, 4).reshape(N, K // GROUP).contiguous()

    scales, mins = groups(b[..., :sm]), groups(b[..., sm:2 * sm])
    qs = b[..., 2 * sm:].reshape(cbs, kts, 2, 2, M_TILE // PAR, K_TILE, PAR // 2)
    lo, hi = qs & 0xF, qs >> 4                      # n even / odd within a byte
    q = torch.stack([lo, hi], -1).reshape(cbs, kts, 2, 2, M_TILE // PAR, K_TILE, PAR)
    # -> [cb, n_half, n_slice, n_in_slice, kb, k_half, k]
    q = q.permute(0, 3, 4, 6, 1, 2, 5).reshape(N, K)
    codes = (q[:, 0::2] | (q[:, 1::2] << 4)).contiguous()
    return codes, scales, mins
