"""One Llama-3.2-1B decoder block at decode with bf16 weights, on one B200.

Two forms:

- the operator chain of BASELINE config 3 -- weighted RMSNorm, the QKV GEMV, RoPE,
  the KV-cache append and the SwiGLU MLP on the normed input -- i.e. the decode
  runlist of iron/applications/llama_3.2_1b/llama_npu.py:459-495 (norm, q/k/v
  GEMVs, RoPE of q and k, the two StridedCopy appends at cache_offset) followed
  by IRON's SwiGLUDecode (iron/operators/swiglu_decode/op.py:56-62);
- the full block (``full=True``; llama_cpu.py:170-207): the same plus GQA
  attention over each sequence's cache, o_proj with the residual, the second
  RMSNorm, and the SwiGLU MLP on it with the second residual.

Every step is a chain of the library's kernels with programmatic dependent
launch -- GEMVs stream their weights while their predecessor finishes -- and is
captured once as a CUDA graph. The gate and up projections are two GEMVs over
the same input, as in IRON's SwiGLUDecode (one GEMV object run on w_gate and
w_up), followed by one silu(gate) * up kernel.

Weights are random (seeded): linear weights ~ N(0, 0.02), norm weights
~ N(1, 0.02), in IRON's GEMV layout (out rows x in columns).
"""

from __future__ import annotations

import math

import torch

from ... import _lib
from .decode import LlamaShape, rope_table


class DecoderBlockBF16:
    """Decoder block with bf16 weights for a batch of sequences at their own positions."""

    def __init__(self, shape: LlamaShape | None = None, batch: int = 1, max_seq: int = 4096, seed: int = 0,
                 full: bool = False, pdl: bool = True):
        s = self.s = shape if shape is not None else LlamaShape()
        self.B, self.L, self.full = batch, max_seq, full
        self.dev = dev = torch.device("cuda", torch.cuda.current_device())
        self.flags = _lib.IRON_FLAG_PDL if pdl else 0
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        E, H, Hd, Q = s.emb_dim, s.hidden_dim, s.head_dim, s.qkv_dim

        def lin(rows, cols):
            return (0.02 * torch.randn(rows, cols, device=dev, generator=g)).to(torch.bfloat16)

        def norm_w():
            return (1 + 0.02 * torch.randn(E, device=dev, generator=g)).to(torch.bfloat16)

        # q rows, then k rows, then v rows: one GEMV for the three projections
        self.W = {"n1": norm_w(), "qkv": lin(Q, E), "o": lin(E, s.n_heads * Hd), "n2": norm_w(),
                  "g": lin(H, E), "u": lin(H, E), "d": lin(E, H)}
        self.lut = rope_table(Hd, max_seq, s.rope_base, dev)
        B = batch
        self.kc = torch.zeros(B, s.n_kv_groups, max_seq, Hd, dtype=torch.bfloat16, device=dev)
        self.vc = torch.zeros_like(self.kc)
        bf = dict(dtype=torch.bfloat16, device=dev)
        self.x = torch.zeros(B, E, **bf)      # block input
        self.out = torch.zeros(B, E, **bf)    # block output (MLP output in the config-3 form)
        self.xn = torch.zeros(B, E, **bf)
        self.qkv = torch.zeros(B, Q, **bf)
        self.q = torch.zeros(B, s.n_heads, Hd, **bf)
        self.attn = torch.zeros(B, s.n_heads * Hd, **bf)
        self.h = torch.zeros(B, E, **bf)
        self.gate = torch.zeros(B, H, **bf)
        self.up = torch.zeros(B, H, **bf)
        self.act = torch.zeros(B, H, **bf)
        self.pos = torch.zeros(B, dtype=torch.int32, device=dev)
        self.lens = torch.zeros(B, dtype=torch.int32, device=dev)
        lib = _lib.load()
        wsb = lib.iron_attn_decode_qkv_workspace_bytes(B, s.n_heads, s.n_kv_groups, max_seq, Hd) if full else 0
        self.attn_ws = torch.zeros(max(wsb, 16), dtype=torch.uint8, device=dev)
        self.graph = None

    # -- bytes moved per step (the roofline numerator) ---------------------------------
    def weight_bytes(self) -> int:
        keys = ("n1", "qkv", "o", "n2", "g", "u", "d") if self.full else ("n1", "qkv", "g", "u", "d")
        return sum(self.W[k].numel() * 2 for k in keys)

    def step_bytes(self, positions) -> int:
        """Algorithmic HBM bytes of one step: every weight once, the block input and
        output rows, the K/V rows appended and (full form) the cached K/V rows the
        attention reads."""
        s, B = self.s, self.B
        row_kv = 2 * s.n_kv_groups * s.head_dim * 2  # one position's K and V rows
        b = self.weight_bytes() + 2 * B * s.emb_dim * 2 + B * row_kv
        if self.full:
            b += sum(int(p) for p in positions) * row_kv
        return b

    def kernels_per_step(self) -> int:
        if not self.full:
            return 7
        s = self.s
        return 8 + _lib.load().iron_attn_decode_kernels(self.B, s.n_heads, s.n_kv_groups, self.L)

    # -- one step -------------------------------------------------------------------------
    def _gemv(self, name, x, y, residual=None, stream=0):
        W = self.W[name]
        M, K = W.shape
        _lib.call("iron_gemv_bf16", W.data_ptr(), x.data_ptr(), y.data_ptr(), M, K, K, 1, 0, 0, 0, self.B,
                  residual.data_ptr() if residual is not None else None, 0, self.flags, stream)

    def _launch(self, stream: int):
        s, B, f, W = self.s, self.B, self.flags, self.W
        call, p = _lib.call, (lambda t: t.data_ptr())
        E, H, Hd, L = s.emb_dim, s.hidden_dim, s.head_dim, self.L
        kv_b, kv_h = s.n_kv_groups * L * Hd, L * Hd
        call("iron_rmsnorm", p(self.x), None, None, p(W["n1"]), p(self.xn), B, E, s.eps, f, stream)
        self._gemv("qkv", self.xn, self.qkv, stream=stream)
        if self.full:
            # RoPE of q and the new k, the append at pos[b], and attention over pos[b] + 1 rows
            call("iron_attn_decode_qkv", p(self.qkv), p(self.pos), p(self.lut), p(self.kc), p(self.vc),
                 p(self.attn), B, s.n_heads, s.n_kv_groups, Hd, L, kv_b, kv_h, 1.0 / math.sqrt(Hd),
                 p(self.attn_ws), self.attn_ws.numel(), f, stream)
            self._gemv("o", self.attn, self.h, residual=self.x, stream=stream)
            call("iron_rmsnorm", p(self.h), None, None, p(W["n2"]), p(self.xn), B, E, s.eps, f, stream)
        else:
            call("iron_rope_kv_append", p(self.qkv), p(self.pos), p(self.lut), p(self.q), p(self.kc), p(self.vc),
                 p(self.lens), B, s.n_heads, s.n_kv_groups, Hd, kv_b, kv_h, f, stream)
        self._gemv("g", self.xn, self.gate, stream=stream)
        self._gemv("u", self.xn, self.up, stream=stream)
        call("iron_eltwise", p(self.gate), p(self.up), p(self.act), B * H, 3, f, stream)  # silu(gate) * up
        self._gemv("d", self.act, self.out, residual=self.h if self.full else None, stream=stream)

    def step(self):
        """One block step (graph replay once captured)."""
        if self.graph is not None:
            self.graph.replay()
        else:
            self._launch(torch.cuda.current_stream().cuda_stream)

    def capture(self):
        """Capture one step as a CUDA graph (the caches' slot pos[b] is rewritten by
        every replay with the same values)."""
        st = torch.cuda.Stream()
        st.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(st):
            self._launch(st.cuda_stream)  # outside capture: first-call attribute setup
        torch.cuda.current_stream().wait_stream(st)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=st):
            self._launch(st.cuda_stream)
        torch.cuda.synchronize()
