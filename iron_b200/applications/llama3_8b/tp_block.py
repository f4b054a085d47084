"""One Llama-3-8B decoder block, tensor-parallel over the GPUs of one node.

Each rank holds the int4 shard of ``sharding.shard_weights`` and runs the decode
step of a batch of sequences:

    RMSNorm -> QKV GEMV (local heads) -> GQA attention with RoPE + KV append (local
    heads, head_dim 128) -> o_proj GEMV (local input columns; rank 0 adds the
    residual) -> all-reduce -> RMSNorm -> gate/up GEMV + SwiGLU (local FFN rows)
    -> down_proj GEMV (local FFN columns; rank 0 adds the residual) -> all-reduce

so the all-reduced o_proj output is the residual stream h and the all-reduced
down_proj output the block output. The two all-reduces are the only exchange; with
tp = 1 they vanish. Either NCCL runs them (bf16 sums over NVLink / NVSwitch, rank 0
adding the residual), or -- fused_allreduce -- the o_proj / down_proj GEMVs do: each
finished tile's fp32 partial is stored into every rank's receive buffer over NVLink
(CUDA IPC mappings) and every rank sums the partials in rank order and adds the
residual, so no collective call runs at all. The kernels are the ones of the
Llama-3.2-1B decode engine (llama_cpu.py:170-218 semantics).
"""

from __future__ import annotations

import ctypes
import math

import torch

from ... import _lib
from ...operators.gemv.op import GEMV
from ..llama_3_2_1b.decode import rope_table
from .sharding import BlockShape, random_block_weights, shard_of, shard_weights


class AllReducePeers(ctypes.Structure):
    """iron_allreduce_peers (include/iron_b200.h)."""

    _fields_ = [("world", ctypes.c_int), ("rank", ctypes.c_int), ("recv", ctypes.c_void_p * 8),
                ("status", ctypes.c_void_p), ("wait_us", ctypes.c_uint)]


class _DeviceBuffer:
    """A zero-filled allocation of its own (an IPC handle maps an allocation's start),
    viewed by torch through __cuda_array_interface__."""

    def __init__(self, shape, typestr: str, itemsize: int):
        n = 1
        for d in shape:
            n *= d
        out = ctypes.c_void_p()
        _lib.call("iron_ipc_alloc", n * itemsize, ctypes.byref(out))
        self.ptr = out.value
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (self.ptr, False),
                                         "version": 3}
        self.tensor = torch.as_tensor(self, device="cuda")

    def free(self):
        if self.ptr:
            _lib.call("iron_ipc_free", self.ptr)
            self.ptr = None


class _PeerSite:
    """Receive buffer ((value, flag) slots) of one fused all-reduce site, mapped on every rank."""

    def __init__(self, rows: int, n_vec: int, tp: int, rank: int, group):
        import torch.distributed as dist

        # (fp32 value, flag) 8-byte slots per (source, row, vector)
        self._bufs = [_DeviceBuffer((tp, rows, n_vec), "<u8", 8)]
        self.recv = self._bufs[0].tensor
        self.status = torch.zeros(4, dtype=torch.int32, device=torch.device("cuda", torch.cuda.current_device()))
        lib = _lib.load()
        hs = []
        for b in self._bufs:
            h = (ctypes.c_char * 64)()
            _lib.call("iron_ipc_handle", b.ptr, h)
            hs.append(bytes(h))
        everyone = [None] * tp
        dist.all_gather_object(everyone, hs, group=group)
        self.opened = []
        self.peers = AllReducePeers()
        self.peers.world, self.peers.rank = tp, rank
        for r in range(tp):
            if r == rank:
                self.peers.recv[r] = self._bufs[0].ptr
                continue
            ptrs = []
            for hb in everyone[r]:
                out = ctypes.c_void_p()
                _lib.call("iron_ipc_open", (ctypes.c_char * 64).from_buffer_copy(hb), ctypes.byref(out))
                ptrs.append(out.value)
                self.opened.append(out.value)
            self.peers.recv[r] = ptrs[0]
        self.peers.status = self.status.data_ptr()
        del lib

    def close(self):
        for p in self.opened:
            _lib.call("iron_ipc_close", p)
        self.opened = []
        self.recv = None
        for b in self._bufs:
            b.tensor = None
            b.free()


class TPDecoderBlock:
    def __init__(self, shape: BlockShape, tp: int, rank: int, batch: int, max_seq: int, seed: int = 0,
                 group=None, pdl: bool = True, keep_full: bool = False, fused_allreduce: bool = False):
        self.s, self.tp, self.rank, self.B, self.L = shape, tp, rank, batch, max_seq
        self.group = group
        self.dev = torch.device("cuda", torch.cuda.current_device())
        self.flags = _lib.IRON_FLAG_PDL if pdl else 0
        # GEMVs read activations through the read-only path: the block keeps the PDL
        # windows that needs (o_proj / down_proj add residuals and bound them; with NCCL
        # the all-reduce kernels, which start only after their predecessor ends, do)
        self.gflags = self.flags | _lib.IRON_FLAG_X_READONLY
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
        self.attn = torch.zeros(B, self.hq * hd, **bf)
        self.act = torch.zeros(B, self.ffn_local, **bf)
        self.pos = torch.zeros(B, dtype=torch.int32, device=dev)
        self.lut = rope_table(hd, max_seq, shape.rope_base, dev)
        wsb = _lib.load().iron_attn_decode_workspace_bytes_d(B, self.hq, self.hk, max_seq, hd)
        self.ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device=dev)
        self.graph = None
        # the two all-reduces inside the o_proj / down_proj GEMVs (peer stores over
        # NVLink) instead of NCCL calls
        self.fused = bool(fused_allreduce) and tp > 1
        if self.fused:
            if B > 8:
                raise ValueError("the fused all-reduce GEMV serves batch <= 8")
            self.site_o = _PeerSite(shape.hidden, B, tp, rank, group)
            self.site_d = _PeerSite(shape.hidden, B, tp, rank, group)

    # -- bytes / launches ---------------------------------------------------------------
    def weight_bytes(self) -> int:
        return sum(r * c * 9 // 16 for r, c in self.dims.values())

    def kernels_per_step(self) -> int:
        """Launches of one step: 2 RMSNorm, 4 GEMVs, attention (+ a split combine)."""
        return 6 + _lib.load().iron_attn_decode_kernels(self.B, self.hq, self.hk, self.L)

    def kv_bytes(self, positions) -> int:
        return int(sum(int(p) + 1 for p in positions)) * self.hk * self.s.head_dim * 2 * 2

    def _allreduce(self, t: torch.Tensor):
        if self.tp > 1:
            import torch.distributed as dist

            dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)

    def _launch(self, stream: int):
        self._attention_half(stream)
        if not self.fused:
            self._allreduce(self.h)
        self._mlp_half(stream)
        if not self.fused:
            self._allreduce(self.x)

    def _attention_half(self, stream: int):
        """RMSNorm -> QKV -> RoPE + KV append -> attention -> o_proj: h (this rank's
        partial, rank 0's holding the residual; the sum over ranks when fused)."""
        s, B, f = self.s, self.B, self.flags
        call, p = _lib.call, (lambda t: t.data_ptr())
        hd, E = s.head_dim, s.hidden
        call("iron_rmsnorm", p(self.x), None, None, p(self.n1), p(self.xn), B, E, s.eps, f, stream)
        call("iron_gemv_int4g32", p(self.w["qkv"]), p(self.xn), p(self.qkv), self.dims["qkv"][0], E, B, None,
             self.gflags, stream)
        kv_b, kv_h = self.hk * self.L * hd, self.L * hd
        # RoPE + KV append inside the attention kernel (q, k, v of the local heads)
        call("iron_attn_decode_qkv", p(self.qkv), p(self.pos), p(self.lut), p(self.kc), p(self.vc), p(self.attn), B,
             self.hq, self.hk, hd, self.L, kv_b, kv_h, 1.0 / math.sqrt(hd), p(self.ws), self.ws.numel(), f, stream)
        if self.fused:
            call("iron_gemv_int4g32_allreduce", p(self.w["o"]), p(self.attn), p(self.h), E, self.dims["o"][1], B,
                 p(self.x), ctypes.addressof(self.site_o.peers), self.gflags, stream)
        else:
            call("iron_gemv_int4g32", p(self.w["o"]), p(self.attn), p(self.h), E, self.dims["o"][1], B,
                 p(self.x) if self.rank == 0 else None, self.gflags, stream)

    def _mlp_half(self, stream: int):
        """RMSNorm -> gate/up + SwiGLU -> down_proj: x (partial / sum as above)."""
        s, B, f = self.s, self.B, self.flags
        call, p = _lib.call, (lambda t: t.data_ptr())
        E = s.hidden
        call("iron_rmsnorm", p(self.h), None, None, p(self.n2), p(self.xn), B, E, s.eps, f, stream)
        call("iron_gemv_int4g32", p(self.w["gu"]), p(self.xn), p(self.act), self.dims["gu"][0], E, B, None,
             self.gflags | _lib.IRON_FLAG_SWIGLU, stream)
        if self.fused:
            call("iron_gemv_int4g32_allreduce", p(self.w["d"]), p(self.act), p(self.x), E, self.dims["d"][1], B,
                 p(self.h), ctypes.addressof(self.site_d.peers), self.gflags, stream)
        else:
            call("iron_gemv_int4g32", p(self.w["d"]), p(self.act), p(self.x), E, self.dims["d"][1], B,
                 p(self.h) if self.rank == 0 else None, self.gflags, stream)

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

    def check_status(self):
        if self.fused and int(self.site_o.status[0] | self.site_d.status[0]) != 0:
            raise RuntimeError("fused all-reduce: a wait for a peer's tile timed out")

    def release(self):
        """Drop the captured graph (it may hold NCCL work; release before destroying the
        group) and unmap the peers' buffers."""
        self.graph = None
        torch.cuda.synchronize()
        if self.fused:
            self.site_o.close()
            self.site_d.close()
