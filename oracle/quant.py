"""Integer/byte work of the hot path, restated in numpy (test oracle).

- ``dequant_u4_tiles``: IRON Dequant, contract iron/operators/dequant/reference.py:8-18
  (per tile: tile/2 code bytes, element 2k = low nibble, unsigned; then tile/group
  bf16 scales; out = bf16(code * scale), the fp32 product rounded once).
- ``pack_u4_tiles``: the payload layout written by IRON's packer
  iron/operators/dequant/reference.py:68-92.
- ``dequant_s4g32`` / ``pack_s4g32``: the int4 group-32 GEMV weight format of the
  north star (signed int4 in [-8, 7], two per byte along K, low nibble = even k,
  one bf16 scale per 32 k).
"""

from __future__ import annotations

import numpy as np


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bit patterns (NaN stays NaN)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    out = rounded.astype(np.uint16)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    out[nan] = 0x7FC0
    return out


def dequant_u4_tiles(payload: np.ndarray, tile_size: int, group_size: int) -> np.ndarray:
    """bf16 bits of code * scale for IRON's Dequant payload."""
    payload = np.asarray(payload, dtype=np.uint8)
    tile_bytes = tile_size // 2 + 2 * (tile_size // group_size)
    tiles = payload.reshape(-1, tile_bytes)
    codes = tiles[:, : tile_size // 2]
    q = np.stack([codes & 0xF, codes >> 4], axis=-1).reshape(len(tiles), tile_size)
    sb = tiles[:, tile_size // 2 :].reshape(len(tiles), -1, 2)
    sbits = sb[..., 0].astype(np.uint16) | (sb[..., 1].astype(np.uint16) << 8)
    s = np.repeat(bf16_bits_to_f32(sbits), group_size, axis=1)
    return f32_to_bf16_bits(q.astype(np.float32) * s).reshape(-1)


def pack_u4_tiles(codes: np.ndarray, scale_bits: np.ndarray, tile_size: int, group_size: int) -> np.ndarray:
    """codes: uint8 [size] in 0..15; scale_bits: uint16 [size/group] -> payload bytes."""
    codes = np.asarray(codes, dtype=np.uint8).reshape(-1, tile_size)
    sbits = np.asarray(scale_bits, dtype=np.uint16).reshape(len(codes), tile_size // group_size)
    packed = (codes[:, 0::2] & 0xF) | ((codes[:, 1::2] & 0xF) << 4)
    sbytes = np.stack([sbits & 0xFF, sbits >> 8], axis=-1).astype(np.uint8).reshape(len(codes), -1)
    return np.concatenate([packed.astype(np.uint8), sbytes], axis=1).reshape(-1)


def pack_s4g32(q: np.ndarray) -> np.ndarray:
    """q: int [N, K] in [-8, 7] -> uint8 [N, K/2], even k in the low nibble."""
    u = (np.asarray(q).astype(np.int16) & 0xF).astype(np.uint8)
    return (u[:, 0::2] | (u[:, 1::2] << 4)).astype(np.uint8)


def unpack_s4(codes: np.ndarray) -> np.ndarray:
    """uint8 [N, K/2] -> int8 [N, K], two's-complement nibbles."""
    c = np.asarray(codes, dtype=np.uint8)
    lo = (c & 0xF).astype(np.int8)
    hi = (c >> 4).astype(np.int8)
    lo = np.where(lo >= 8, lo - 16, lo)
    hi = np.where(hi >= 8, hi - 16, hi)
    return np.stack([lo, hi], axis=-1).reshape(c.shape[0], -1).astype(np.int8)


def dequant_s4g32(codes: np.ndarray, scale_bits: np.ndarray, group: int = 32) -> np.ndarray:
    """bf16 bits [N, K] of bf16(q * scale) for the int4g32 GEMV weights."""
    q = unpack_s4(codes).astype(np.float32)
    s = np.repeat(bf16_bits_to_f32(np.asarray(scale_bits, dtype=np.uint16)), group, axis=1)
    return f32_to_bf16_bits(q * s)


def make_s4g32(n: int, k: int, seed: int = 42, smin: float = 0.005, smax: float = 0.02):
    """BASELINE config-2 weights: q ~ U{-8..7}, scales ~ U[smin, smax] rounded to bf16."""
    rng = np.random.default_rng(seed)
    q = rng.integers(-8, 8, size=(n, k), dtype=np.int16)
    s = rng.uniform(smin, smax, size=(n, k // 32)).astype(np.float32)
    return pack_s4g32(q), f32_to_bf16_bits(s), q


def pack_s4g32_units(codes: np.ndarray, scale_bits: np.ndarray) -> np.ndarray:
    """Streaming layout of the int4g32 GEMV (the unit format iron_pack_int4g32 writes).

    Unit (t, c) covers rows 16t..16t+15 and k 128c..128c+127 and is 1152 bytes:
    the 32-bit word at bytes [h*512 + lane*16 + 4j, +4) holds the 8 codes of row
    16t + gid + 8h (lane = 4*gid + tid) at k (4c+j)*32 + 8*tid + i, i = 0..7, the
    code of k_i at bits 4*(i//2) for even i and 16 + 4*(i//2) for odd i (pairs of
    consecutive k share a bf16x2 after dequantization); bytes [1024 + 16*gid, +16) =
    the bf16 scales of groups 4c..4c+3 of row 16t+gid, then of row 16t+gid+8.
    """
    codes = np.asarray(codes, dtype=np.uint8)
    sb = np.asarray(scale_bits, dtype=np.uint16)
    M, Kh = codes.shape
    K = Kh * 2
    T, C = M // 16, K // 128
    # codes: row = 16t + gid + 8h ; byte = (4c + j)*16 + 4*tid + b
    cc = codes.reshape(T, 2, 8, C, 4, 4, 4)  # t, h, gid, c, j, tid, b
    cc = cc.transpose(0, 3, 1, 2, 5, 4, 6)  # t, c, h, gid, tid, j, b
    # the word's nibble order: low nibbles of the 4 natural bytes into bits 0-15, high
    # nibbles into bits 16-31 (byte 0 = lo(b0) | lo(b1) << 4, byte 2 = hi(b0) | hi(b1) << 4)
    lo, hi = cc & 0x0F, cc >> 4
    cc = np.stack([lo[..., 0] | (lo[..., 1] << 4), lo[..., 2] | (lo[..., 3] << 4),
                   hi[..., 0] | (hi[..., 1] << 4), hi[..., 2] | (hi[..., 3] << 4)], axis=-1)
    cc = cc.astype(np.uint8).reshape(T, C, 1024)
    ss = sb.reshape(T, 2, 8, C, 4).transpose(0, 3, 2, 1, 4).reshape(T, C, 64)  # t,c,gid,h,j
    units = np.concatenate([cc, ss.view(np.uint8).reshape(T, C, 128)], axis=2)
    return units.reshape(-1)


def unpack_s4g32_units(units: np.ndarray, M: int, K: int):
    """Inverse of pack_s4g32_units: natural codes [M, K/2] and scale bits [M, K/32]."""
    T, C = M // 16, K // 128
    u = np.asarray(units, dtype=np.uint8).reshape(T, C, 1152)
    cc = u[:, :, :1024].reshape(T, C, 2, 8, 4, 4, 4)  # t, c, h, gid, tid, j, packed byte
    p0, p1, p2, p3 = (cc[..., i] for i in range(4))
    lo = np.stack([p0 & 0x0F, p0 >> 4, p1 & 0x0F, p1 >> 4], axis=-1)  # low nibbles of natural bytes 0..3
    hi = np.stack([p2 & 0x0F, p2 >> 4, p3 & 0x0F, p3 >> 4], axis=-1)
    nat = (lo | (hi << 4)).astype(np.uint8)  # t, c, h, gid, tid, j, b
    codes = nat.transpose(0, 2, 3, 1, 5, 4, 6).reshape(M, K // 2)  # t, h, gid, c, j, tid, b
    ss = u[:, :, 1024:].copy().view(np.uint16).reshape(T, C, 8, 2, 4)  # t, c, gid, h, j
    scales = ss.transpose(0, 3, 2, 1, 4).reshape(M, K // 32)
    return codes, scales


# ---- q4nx: asymmetric int4, min + scale * code ---------------------------------------
# The input format of IRON's flm.DequantBFP (iron/operators/flm/dequant/README.md, input
# layers 1-9; reference iron/operators/flm/dequant/reference.py:40-77): blocks of 32
# out-features x 256 in-features -- 512 B of bf16 scales [8 groups][32 n], 512 B of bf16
# mins, 4096 B of codes (two n per byte: even n in the low nibble) -- ordered, for block
# i, as cb, kb, k_half, n_half (i = ((cb * K/512 + kb) * 2 + k_half) * 2 + n_half).
Q4NX_M, Q4NX_K, Q4NX_G, Q4NX_KB, Q4NX_PAR = 32, 256, 32, 512, 16
Q4NX_BLOCK = Q4NX_M * Q4NX_K * 5 // 8


def q4nx_to_natural(blob: np.ndarray, K: int, N: int):
    """q4nx blob -> (codes uint8 [N, K] in 0..15, scale bits uint16 [N, K/32], min bits
    uint16 [N, K/32]): the block walk of reference.py:40-77, per block."""
    b = np.asarray(blob, dtype=np.uint8).reshape(-1, Q4NX_BLOCK)
    n_blocks = b.shape[0]
    ng = Q4NX_K // Q4NX_G
    sm = ng * Q4NX_M * 2
    sc = b[:, :sm].copy().view(np.uint16).reshape(n_blocks, ng, Q4NX_M)
    mn = b[:, sm:2 * sm].copy().view(np.uint16).reshape(n_blocks, ng, Q4NX_M)
    qs = b[:, 2 * sm:].reshape(n_blocks, Q4NX_M // Q4NX_PAR, Q4NX_K, Q4NX_PAR // 2)
    q = np.empty((n_blocks, Q4NX_M // Q4NX_PAR, Q4NX_K, Q4NX_PAR), dtype=np.uint8)
    q[..., 0::2] = qs & 0xF
    q[..., 1::2] = qs >> 4
    q = q.transpose(0, 1, 3, 2).reshape(n_blocks, Q4NX_M, Q4NX_K)
    k_tiles = K // Q4NX_KB
    codes = np.zeros((N, K), dtype=np.uint8)
    sbits = np.zeros((N, K // Q4NX_G), dtype=np.uint16)
    mbits = np.zeros_like(sbits)
    for i in range(n_blocks):
        cb, rest = divmod(i, 4 * k_tiles)
        kb, rest = divmod(rest, 4)
        k_half, n_half = divmod(rest, 2)
        r0, c0 = (2 * cb + n_half) * Q4NX_M, (2 * kb + k_half) * Q4NX_K
        codes[r0:r0 + Q4NX_M, c0:c0 + Q4NX_K] = q[i]
        sbits[r0:r0 + Q4NX_M, c0 // Q4NX_G:c0 // Q4NX_G + ng] = sc[i].T
        mbits[r0:r0 + Q4NX_M, c0 // Q4NX_G:c0 // Q4NX_G + ng] = mn[i].T
    return codes, sbits, mbits


def q4nx_dequant(codes: np.ndarray, sbits: np.ndarray, mbits: np.ndarray) -> np.ndarray:
    """fp32 [N, K] = min + scale * code, as reference.py computes it."""
    s = np.repeat(bf16_bits_to_f32(sbits), Q4NX_G, axis=1)
    m = np.repeat(bf16_bits_to_f32(mbits), Q4NX_G, axis=1)
    return (m + s * codes.astype(np.float32)).astype(np.float32)


def q4nx_from_natural(codes: np.ndarray, sbits: np.ndarray, mbits: np.ndarray) -> np.ndarray:
    """Inverse of q4nx_to_natural (builds blobs for tests)."""
    N, K = codes.shape
    k_tiles = K // Q4NX_KB
    n_blocks = (N // Q4NX_M) * (K // Q4NX_K)
    ng = Q4NX_K // Q4NX_G
    out = np.empty((n_blocks, Q4NX_BLOCK), dtype=np.uint8)
    for i in range(n_blocks):
        cb, rest = divmod(i, 4 * k_tiles)
        kb, rest = divmod(rest, 4)
        k_half, n_half = divmod(rest, 2)
        r0, c0 = (2 * cb + n_half) * Q4NX_M, (2 * kb + k_half) * Q4NX_K
        q = codes[r0:r0 + Q4NX_M, c0:c0 + Q4NX_K].reshape(Q4NX_M // Q4NX_PAR, Q4NX_PAR, Q4NX_K).transpose(0, 2, 1)
        qs = (q[..., 0::2] & 0xF) | ((q[..., 1::2] & 0xF) << 4)
        s = np.ascontiguousarray(sbits[r0:r0 + Q4NX_M, c0 // Q4NX_G:c0 // Q4NX_G + ng].T).view(np.uint8)
        m = np.ascontiguousarray(mbits[r0:r0 + Q4NX_M, c0 // Q4NX_G:c0 // Q4NX_G + ng].T).view(np.uint8)
        out[i] = np.concatenate([s.reshape(-1), m.reshape(-1), qs.astype(np.uint8).reshape(-1)])
    return out.reshape(-1)
