"""MHA on B200 -- constructor and buffers of iron/operators/mha/op.py:21-135.

Causal multi-head / grouped-query attention over a whole sequence (prefill):
``O = softmax(Q K^T / sqrt(d), causal) V`` with K/V heads shared by
``num_heads / num_KV_heads`` query heads (golden mha/reference.py:27-94). Buffers
keep IRON's padded layout: Q and O ``(heads, S_pad, d)``, K and V
``(kv_heads, S_pad, d)``, S_pad the sequence rounded up to 64 * pipelines; output
rows past ``seq_len`` are zero. ``num_of_pipelines`` only sets that padding.
"""

from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass, field
from typing import ClassVar, Dict

import numpy as np

from ... import _lib
from ...common.base import AIERuntimeArgSpec, MLIROperator
from ...common.verify import Tolerance


@dataclass
class MHA(MLIROperator):
    """Causal (GQA) attention over a sequence on the B200."""

    num_heads: int
    seq_len: int
    d: int
    num_KV_heads: int
    num_of_pipelines: int = field(default=1, repr=False)
    context: object = field(default=None, repr=False)

    _name_aliases: ClassVar[Dict[str, str]] = {
        **MLIROperator._name_aliases,
        "num_heads": "h",
        "num_KV_heads": "kv",
        "seq_len": "s",
    }
    _tolerance = Tolerance.relative(4.0e-2, 1.5e-1, max_mismatch_frac=0.005)

    def __post_init__(self):
        self.B_q = 64
        self.B_kv = 64
        if self.d != 64:
            raise ValueError(f"Only d=64 is supported in this version, got d={self.d}")
        kv = self.num_KV_heads if self.num_KV_heads else self.num_heads
        if self.num_heads % kv:
            raise ValueError("num_heads must be a multiple of num_KV_heads")
        MLIROperator.__init__(self, context=self.context)

    @property
    def kv_heads(self) -> int:
        return self.num_KV_heads if self.num_KV_heads else self.num_heads

    def _calculate_seq_padding(self, seq_len, num_pipeline=1):
        return ((seq_len + 63 * num_pipeline) // (64 * num_pipeline)) * (64 * num_pipeline)

    def _pad_to_multiple_of_64(self, tensor, seq_dim, num_pipeline=1):
        seq_len = tensor.shape[seq_dim]
        padded = self._calculate_seq_padding(seq_len, num_pipeline)
        if padded == seq_len:
            return tensor
        width = [(0, 0)] * tensor.ndim
        width[seq_dim] = (0, padded - seq_len)
        return np.pad(tensor, width)

    def _pack_compact_to_padded(self, src, H, S, S_pad, D):
        if S == S_pad:
            return src
        dst = np.zeros((H, S_pad, D), dtype=src.dtype)
        dst[:H, :S, :D] = src
        return dst

    def _unpack_padded_to_compact(self, src, H, S, S_pad, D):
        return src[:H, :S, :D] if S < S_pad else src

    def get_arg_spec(self):
        pad = self._calculate_seq_padding(self.seq_len, self.num_of_pipelines)
        q = self.num_heads * self.d * pad
        kv = self.kv_heads * self.d * pad
        return [AIERuntimeArgSpec("in", (q,)), AIERuntimeArgSpec("in", (kv,)), AIERuntimeArgSpec("in", (kv,)),
                AIERuntimeArgSpec("out", (q,))]

    def _launch(self, Q, K, V, O, *, stream, flags=0):
        pad = self._calculate_seq_padding(self.seq_len, self.num_of_pipelines)
        st = (ctypes.c_int64 * 3)(0, pad * self.d, self.d)
        p = _lib.dptr
        # the kernel pads its work to 64-row blocks; IRON's S_pad is a multiple of 64
        _lib.call("iron_attn_prefill", p(Q), p(K), p(V), p(O), 1, self.num_heads, self.kv_heads, self.d,
                  self.seq_len, pad, self.seq_len, st, st, st, 1.0 / math.sqrt(self.d), 1, flags, stream)

    def reference(self, Q, K, V):
        import torch

        pad = self._calculate_seq_padding(self.seq_len, self.num_of_pipelines)
        H, Hk, S, D = self.num_heads, self.kv_heads, self.seq_len, self.d
        q = Q.reshape(H, pad, D)[:, :S].float()
        k = K.reshape(Hk, pad, D)[:, :S].float().repeat_interleave(H // Hk, dim=0)
        v = V.reshape(Hk, pad, D)[:, :S].float().repeat_interleave(H // Hk, dim=0)
        o = torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True, scale=1 / math.sqrt(D))
        out = torch.zeros(H, pad, D, dtype=torch.bfloat16)
        out[:, :S] = o.to(torch.bfloat16)
        return out.reshape(-1)
