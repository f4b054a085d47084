"""Tensor-parallel partition of one Llama-3-8B decoder block (Megatron form).

Column-parallel: the q / k / v projections by heads (32 / tp query heads and
8 / tp kv heads per rank; the GQA group of 4 stays on one rank) and the gate / up
projections by FFN rows (14336 / tp). Row-parallel: o_proj over the local heads'
input columns and down_proj over the local FFN columns; each rank's partial
output is summed by one all-reduce after o_proj and one after down_proj. The KV
cache is split by kv head with no exchange; RMSNorm runs replicated.

Weights are int4 with one bf16 scale per 32 inputs, in their natural layout:
``codes`` uint8 [rows, in / 2] (element 2k in the low nibble), ``scales`` bf16
[rows, in / 32]. Column slices stay on 128-element boundaries, so groups never
straddle ranks.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class BlockShape:
    """Llama-3-8B decoder block (hidden 4096, 32 / 8 heads of 128, FFN 14336)."""

    hidden: int = 4096
    n_heads: int = 32
    n_kv: int = 8
    head_dim: int = 128
    ffn: int = 14336
    eps: float = 1e-5
    rope_base: float = 500000.0

    def params(self) -> int:
        q, kv = self.n_heads * self.head_dim, self.n_kv * self.head_dim
        return (q + 2 * kv) * self.hidden + self.hidden * q + 3 * self.ffn * self.hidden


@dataclass(frozen=True)
class Shard:
    tp: int
    rank: int
    h0: int  # query heads [h0, h1)
    h1: int
    k0: int  # kv heads [k0, k1)
    k1: int
    f0: int  # FFN rows [f0, f1)
    f1: int


def shard_of(shape: BlockShape, tp: int, rank: int) -> Shard:
    if shape.n_kv % tp or shape.n_heads % tp or shape.ffn % tp:
        raise ValueError(f"tp={tp} does not divide heads ({shape.n_heads}/{shape.n_kv}) and FFN ({shape.ffn})")
    if (shape.ffn // tp) % 128:
        raise ValueError("the FFN slice must be a multiple of 128 (int4 groups and GEMV units)")
    hq, hk, f = shape.n_heads // tp, shape.n_kv // tp, shape.ffn // tp
    return Shard(tp, rank, rank * hq, (rank + 1) * hq, rank * hk, (rank + 1) * hk, rank * f, (rank + 1) * f)


def _rows(t: torch.Tensor, r0: int, r1: int) -> torch.Tensor:
    return t[r0:r1]


def _cols(codes: torch.Tensor, scales: torch.Tensor, c0: int, c1: int):
    return codes[:, c0 // 2 : c1 // 2].contiguous(), scales[:, c0 // 32 : c1 // 32].contiguous()


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """Rows in tiles of 16: 8 gate rows, then the matching 8 up rows."""
    n = gate.shape[0]
    g = gate.reshape(n // 8, 8, *gate.shape[1:])
    u = up.reshape(n // 8, 8, *up.shape[1:])
    return torch.cat([g, u], dim=1).reshape(2 * n, *gate.shape[1:])


def shard_weights(W: dict, shape: BlockShape, sh: Shard) -> dict:
    """This rank's int4 weights from the full block's natural codes / scales.

    W maps "q", "k", "v", "o", "g", "u", "d" to (codes, scales) pairs in the
    natural layout ([out, in] rows); "n1" / "n2" are the bf16 norm weights.
    Returns "qkv" (local q rows, then local k, then local v), "o" (all rows, the
    local heads' input columns), "gu" (local gate/up rows, interleaved per 8),
    "d" (all rows, the local FFN columns), "n1", "n2".
    """
    hd = shape.head_dim
    q = [_rows(x, sh.h0 * hd, sh.h1 * hd) for x in W["q"]]
    k = [_rows(x, sh.k0 * hd, sh.k1 * hd) for x in W["k"]]
    v = [_rows(x, sh.k0 * hd, sh.k1 * hd) for x in W["v"]]
    qkv = tuple(torch.cat([a, b, c]).contiguous() for a, b, c in zip(q, k, v))
    o = _cols(*W["o"], sh.h0 * hd, sh.h1 * hd)
    g = [_rows(x, sh.f0, sh.f1) for x in W["g"]]
    u = [_rows(x, sh.f0, sh.f1) for x in W["u"]]
    gu = tuple(interleave_gate_up(a, b).contiguous() for a, b in zip(g, u))
    d = _cols(*W["d"], sh.f0, sh.f1)
    return {"qkv": qkv, "o": o, "gu": gu, "d": d, "n1": W["n1"], "n2": W["n2"]}


def random_block_weights(shape: BlockShape, seed: int, device) -> dict:
    """Seeded random int4 weights of the whole block (identical on every rank):
    codes ~ U{0..255} bytes, scales ~ U[0.001, 0.004] (down: U[0.0005, 0.002])."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    E, F = shape.hidden, shape.ffn
    q, kv = shape.n_heads * shape.head_dim, shape.n_kv * shape.head_dim

    def mat(rows, cols, smin, smax):
        codes = torch.randint(0, 256, (rows, cols // 2), dtype=torch.uint8, device=device, generator=g)
        scales = (torch.rand(rows, cols // 32, device=device, generator=g) * (smax - smin) + smin).to(torch.bfloat16)
        return codes, scales

    W = {"n1": (1 + 0.02 * torch.randn(E, device=device, generator=g)).to(torch.bfloat16),
         "n2": (1 + 0.02 * torch.randn(E, device=device, generator=g)).to(torch.bfloat16)}
    W["q"] = mat(q, E, 0.001, 0.004)
    W["k"] = mat(kv, E, 0.001, 0.004)
    W["v"] = mat(kv, E, 0.001, 0.004)
    W["o"] = mat(E, q, 0.001, 0.004)
    W["g"] = mat(F, E, 0.001, 0.004)
    W["u"] = mat(F, E, 0.001, 0.004)
    W["d"] = mat(E, F, 0.0005, 0.002)
    return W
