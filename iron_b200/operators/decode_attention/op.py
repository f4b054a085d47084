"""GQA decode attention on B200 (split-KV flash-decoding).

IRON runs decode attention as a chain of operators over the whole padded cache
(iron/applications/llama_3.2_1b/llama_npu.py:495-529: Repeat x2, scores GEMV,
scale, masked Softmax, 32x Transpose, context GEMV; CPU truth
iron/applications/llama_3.2_1b/llama_cpu.py:118-140). This operator computes the
same softmax(q K^T / sqrt(d)) V for a batch of sequences with ragged lengths in
one pass over each sequence's valid cache rows.

Buffers: q bf16 [B, Hq, D]; k_cache, v_cache bf16 [B, Hkv, max_seq_len, D];
lens int32 [B] (valid tokens, read on the device); out bf16 [B, Hq, D].
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

from ...common.base import MLIROperator, AIERuntimeArgSpec
from ...common.verify import Tolerance
from ... import _lib


@dataclass
class DecodeAttention(MLIROperator):
    batch: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    max_seq_len: int
    context: object = field(default=None, repr=False)

    _tolerance = Tolerance.relative(2e-2, 1e-2)

    def __post_init__(self):
        if self.head_dim != 64:
            raise ValueError(f"Only d=64 is supported in this version, got d={self.head_dim}")
        if self.num_heads % self.num_kv_heads or self.num_heads // self.num_kv_heads > 16:
            raise ValueError("num_heads must be a multiple of num_kv_heads (group <= 16)")
        self._ws = None
        MLIROperator.__init__(self, context=self.context)

    def get_arg_spec(self):
        B, H, Hkv, D, L = self.batch, self.num_heads, self.num_kv_heads, self.head_dim, self.max_seq_len
        return [
            AIERuntimeArgSpec("in", (B, H, D)),
            AIERuntimeArgSpec("in", (B, Hkv, L, D)),
            AIERuntimeArgSpec("in", (B, Hkv, L, D)),
            AIERuntimeArgSpec("in", (B,), dtype=np.int32),
            AIERuntimeArgSpec("out", (B, H, D)),
        ]

    def workspace(self):
        import torch

        nbytes = _lib.load().iron_attn_decode_workspace_bytes(self.batch, self.num_heads,
                                                              self.num_kv_heads, self.max_seq_len)
        if self._ws is None or self._ws.numel() < nbytes:
            self._ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device="cuda")
        return self._ws

    def prepare(self):
        self.workspace()

    def _launch(self, q, k, v, lens, out, *, stream, flags=0):
        p = _lib.dptr
        ws = self.workspace()
        L, D = self.max_seq_len, self.head_dim
        _lib.call("iron_attn_decode", p(q), p(k), p(v), p(lens), p(out), self.batch, self.num_heads,
                  self.num_kv_heads, D, L, self.num_kv_heads * L * D, L * D,
                  1.0 / math.sqrt(D), ws.data_ptr(), ws.numel(), flags, stream)

    def reference(self, q, k, v, lens):
        import torch

        g = self.num_heads // self.num_kv_heads
        out = torch.empty_like(q)
        for b in range(self.batch):
            n = int(lens[b])
            K = k[b, :, :n].float().repeat_interleave(g, dim=0)
            V = v[b, :, :n].float().repeat_interleave(g, dim=0)
            s = torch.einsum("hd,hld->hl", q[b].float(), K) / math.sqrt(self.head_dim)
            out[b] = torch.einsum("hl,hld->hd", torch.softmax(s, -1), V).to(q.dtype)
        return out
