"""One Llama-3-8B decoder block, tensor-parallel over the GPUs of one node.

Each rank holds the int4 shard of ``sharding.shard_weights`` and runs the decode
step of a batch of sequences:

    RMSNorm -> QKV GEMV (local heads) -> RoPE + KV append -> GQA attention (local
    heads, head_dim 128) -> o_proj GEMV (local input columns; rank 0 adds the
    residual) -> all-reduce -> RMSNorm -> gate/up GEMV + SwiGLU (local FFN rows)
    -> down_proj GEMV (local FFN columns; rank 0 adds the residual) -> all-reduce

so the all-reduced o_proj output is the residual stream h and the all-reduced
down_proj output the block output. The two all-reduces (bf16 sums over NCCL,
NVLink / NVSwitch) are the only exchange; with tp = 1 they vanish. The kernels are
the ones of the Llama-3.2-1B decode engine (llama_cpu.py:170-218 semantics).
"""

from __future__ import annotations

import math

import torch

from ... import _lib
from ...operators.gemv.op import GEMV
from ..llama_3_2_1b.decode import rope_table
from .sharding import BlockShape, random_block_weights, shard_of, shard_weights


class TPDecoderBlock:
    def __init__(self, shape: BlockShape, tp: int, rank: int, batch: int, max_seq: int, seed: int = 0,
                 group=None, pdl: bool = True, keep_full: bool = False):
        self.s, self.tp, self.rank, self.B, self.L = shape, tp, rank, batch, max_seq
        self.group = group
        self.dev = torch.device("cuda", torch.cuda.current_device())
        self.flags = _lib.IRON_FLAG_PDL if pdl else 0
        self.sh = shard_of(shape, tp, rank)
        W = random_block_weights(shape, seed, self.dev)
        self.full = W if keep_full else None
        S = shard_weights(W, shape, self.sh)
        self.w = {k: GEMV.pack_int4g32(*S[k]) for k in ("qkv", "o", "gu", "d")}
        self.dims = {"qkv": (S["qkv"][0].shape[0], shape.hidden), "o": (shape.hidden, S["o"][0].shape[1] * 2),
                     "gu": (S["gu"][0].shape[0], shape.hidden), "d": (shape.hidden, S["d"][0].shape[1] * 2)}
        self.n1, self.n2 = W["n1"], W["n2"]
        del S
        if not keep_full:
            del W
        hd = shape.head_dim
        self.hq, self.hk = self.sh.h1 - self.sh.h0, self.sh.k1 - self.sh.k0
        self.ffn_local = self.sh.f1 - self.sh.f0
        B, dev = batch, self.dev
        bf = dict(dtype=torch.bfloat16, device=dev)
        self.kc = torch.zeros(B, self.hk, max_seq, hd, **bf)
        self.vc = torch.zeros_like(self.kc)
        self.x = torch.zeros(B, shape.hidden, **bf)
        self.xn = torch.zeros_like(self.x)
        self.h = torch.zeros_like(self.x)
        self.qkv = torch.zeros(B, self.dims["qkv"][0], **bf)
        self.q = torch.zeros(B, self.hq, hd, **bf)
        self.attn = torch.zeros(B, self.hq * hd, **bf)
        self.act = torch.zeros(B, self.ffn_local, **bf)
        self.pos = torch.zeros(B, dtype=torch.int32, device=dev)
        self.lens = torch.zeros(B, dtype=torch.int32, device=dev)
        self.lut = rope_table(hd, max_seq, shape.rope_base, dev)
        wsb = _lib.load().iron_attn_decode_workspace_bytes_d(B, self.hq, self.hk, max_seq, hd)
        self.ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device=dev)
        self.graph = None

    # -- bytes / launches ---------------------------------------------------------------
    def weight_bytes(self) -> int:
        return sum(r * c * 9 // 16 for r, c in self.dims.values())

    def kv_bytes(self, positions) -> int:
        return int(sum(int(p) + 1 for p in positions)) * self.hk * self.s.head_dim * 2 * 2

    def _allreduce(self, t: torch.Tensor):
        if self.tp > 1:
            import torch.distributed as dist

            dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)

    def _launch(self, stream: int):
        s, B, f = self.s, self.B, self.flags
        call, p = _lib.call, (lambda t: t.data_ptr())
        hd, E = s.head_dim, s.hidden
        lead = self.rank == 0
        call("iron_rmsnorm", p(self.x), None, None, p(self.n1), p(self.xn), B, E, s.eps, f, stream)
        call("iron_gemv_int4g32", p(self.w["qkv"]), p(self.xn), p(self.qkv), self.dims["qkv"][0], E, B, None, f,
             stream)
        kv_b, kv_h = self.hk * self.L * hd, self.L * hd
        call("iron_rope_kv_append", p(self.qkv), p(self.pos), p(self.lut), p(self.q), p(self.kc), p(self.vc),
             p(self.lens), B, self.hq, self.hk, hd, kv_b, kv_h, f, stream)
        call("iron_attn_decode", p(self.q), p(self.kc), p(self.vc), p(self.lens), p(self.attn), B, self.hq,
             self.hk, hd, self.L, kv_b, kv_h, 1.0 / math.sqrt(hd), p(self.ws), self.ws.numel(), f, stream)
        call("iron_gemv_int4g32", p(self.w["o"]), p(self.attn), p(self.h), E, self.dims["o"][1], B,
             p(self.x) if lead else None, f, stream)
        self._allreduce(self.h)
        call("iron_rmsnorm", p(self.h), None, None, p(self.n2), p(self.xn), B, E, s.eps, f, stream)
        call("iron_gemv_int4g32", p(self.w["gu"]), p(self.xn), p(self.act), self.dims["gu"][0], E, B, None,
             f | _lib.IRON_FLAG_SWIGLU, stream)
        call("iron_gemv_int4g32", p(self.w["d"]), p(self.act), p(self.x), E, self.dims["d"][1], B,
             p(self.h) if lead else None, f, stream)
        self._allreduce(self.x)

    def step(self):
        """x <- block(x) for every sequence at its position pos[b] (caches updated)."""
        if self.graph is not None:
            self.graph.replay()
        else:
            self._launch(torch.cuda.current_stream().cuda_stream)

    def capture(self):
        """Capture one step (kernels and NCCL all-reduces) as a CUDA graph."""
        st = torch.cuda.Stream()
        st.wait_stream(torch.cuda.current_stream())
        saved = self.x.clone()
        with torch.cuda.stream(st):
            self._launch(st.cuda_stream)  # warm-up outside capture
        torch.cuda.current_stream().wait_stream(st)
        torch.cuda.synchronize()
        self.x.copy_(saved)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=st):
            self._launch(st.cuda_stream)
        torch.cuda.synchronize()
        self.x.copy_(saved)
        torch.cuda.synchronize()

    def release(self):
        """Drop the captured graph (it holds NCCL work; release before destroying the group)."""
        self.graph = None
        torch.cuda.synchronize()
