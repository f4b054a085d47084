"""Llama-3.2-1B decode on one B200: the fused int4 decode step of IRON's pipeline.

IRON's decode step (iron/applications/llama_3.2_1b/llama_npu.py:459-584, driven
by llama_forward_pass_decode :1156-1195) is one fused OperatorSequence of ~40
operators per layer. Here the same computation -- RMSNorm, q/k/v projections,
RoPE, KV-cache append, GQA attention, o projection, residual, RMSNorm, SwiGLU
MLP, residual; final norm and tied lm-head (llama_cpu.py:170-285) -- runs as
five kernels per layer up to batch 8 (the RMSNorms folded into the GEMVs around
them) and seven from batch 9 on, with int4 group-32 weights, for a batch of sequences at
their own positions, captured once as a CUDA graph whose kernels are launched
with programmatic dependent launch (each GEMV streams its weights while its
predecessor finishes). Greedy argmax picks the next token on the device and
advances every sequence's position, so graph replays chain decode steps.

Weights are random (seeded): int4 codes ~ U{-8..7} and bf16 group scales, the
embedding table being the exact dequantization of the tied lm-head weights.
"""

from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import torch

from ... import _lib
from ...operators.gemv.op import GEMV


@dataclass
class LlamaShape:
    """Model dimensions (iron/applications/llama_3.2_1b/llama_inference_harness.py:28-48)."""

    vocab_size: int = 128256
    emb_dim: int = 2048
    n_layers: int = 16
    n_heads: int = 32
    n_kv_groups: int = 8
    head_dim: int = 64
    hidden_dim: int = 8192
    rope_base: float = 500000.0
    eps: float = 1e-5

    @property
    def qkv_dim(self) -> int:
        return (self.n_heads + 2 * self.n_kv_groups) * self.head_dim

    def weight_params(self) -> int:
        E, H, Q = self.emb_dim, self.hidden_dim, self.qkv_dim
        per_layer = Q * E + E * self.n_heads * self.head_dim + 2 * H * E + E * H
        return self.n_layers * per_layer + self.vocab_size * E


def rope_table(head_dim: int, positions: int, base: float, device) -> torch.Tensor:
    """fp32 [positions, head_dim] interleaved cos/sin
    (iron/applications/llama_3.2_1b/llama_inference_harness.py:109-123)."""
    inv = 1.0 / (base ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
    f = torch.outer(torch.arange(positions, dtype=torch.float32), inv)
    t = torch.empty(positions, head_dim, dtype=torch.float32)
    t[:, 0::2] = torch.cos(f)
    t[:, 1::2] = torch.sin(f)
    return t.to(device)


class Int4Matrix:
    """int4 group-32 weights: natural codes/scales (for checks) and the packed GEMV layout."""

    def __init__(self, rows: int, cols: int, gen: torch.Generator, smin: float, smax: float,
                 keep_natural: bool = False):
        dev = gen.device
        codes = torch.randint(0, 256, (rows, cols // 2), dtype=torch.uint8, device=dev, generator=gen)
        scales = (torch.rand(rows, cols // 32, device=dev, generator=gen) * (smax - smin) + smin).to(torch.bfloat16)
        self.rows, self.cols = rows, cols
        self.packed = GEMV.pack_int4g32(codes, scales)
        self.codes = codes if keep_natural else None
        self.scales = scales if keep_natural else None
        if not keep_natural:
            del codes, scales

    @classmethod
    def from_dense(cls, w: torch.Tensor, keep_natural: bool = False) -> "Int4Matrix":
        """Quantize bf16 / fp32 weights [rows, cols] (weights.quantize_int4g32) and pack them."""
        from .weights import quantize_int4g32

        m = cls.__new__(cls)
        codes, scales = quantize_int4g32(w)
        m.rows, m.cols = w.shape
        m.packed = GEMV.pack_int4g32(codes, scales)
        m.codes = codes if keep_natural else None
        m.scales = scales if keep_natural else None
        return m

    def dequant(self) -> torch.Tensor:
        """Exact bf16 weights [rows, cols] (needs keep_natural)."""
        out = torch.empty(self.rows, self.cols, dtype=torch.bfloat16, device=self.codes.device)
        _lib.call("iron_dequant_s4g32_rows", self.codes.data_ptr(), self.scales.data_ptr(),
                  out.data_ptr(), self.rows, self.cols, _lib.current_stream())
        return out


def interleave_gate_up(gate_rows: int) -> torch.Tensor:
    """Row permutation placing 8 gate rows then the 8 matching up rows in each
    16-row tile (the layout the SwiGLU epilogue of the int4 GEMV expects)."""
    t = torch.arange(gate_rows // 8)
    idx = torch.stack([t * 8 + i for i in range(8)] + [gate_rows + t * 8 + i for i in range(8)], 1)
    return idx.reshape(-1)


@dataclass
class SamplingConfig:
    """Next-token sampling of IRON's harness (llama_inference_harness.py:44-45 defaults,
    :146-169 steps): logits / temperature, top-k filter, softmax, multinomial draw.
    Runs on the device; the draw is a function of (seed, sequence, position)."""

    temperature: float = 0.7
    top_k: int = 50
    seed: int = 0


class LlamaDecodeEngine:
    """Batched greedy decode of a random-init int4 Llama-3.2-1B-shape model."""

    def __init__(self, shape: LlamaShape, batch: int, max_seq: int, seed: int = 0,
                 keep_natural: bool = False, pdl: bool = True, fuse_norm: str | None = None,
                 fuse_rope: bool | None = None, l2_prefetch: bool | None = None,
                 sampling: "SamplingConfig | None" = None, weights: dict | None = None):
        """weights: a checkpoint's tensors by Hugging Face name (weights.load_checkpoint),
        quantized here to int4 group-32; None: random weights from `seed`."""
        self.s, self.B, self.L = shape, batch, max_seq
        # None: greedy argmax fused into the lm-head GEMV; else temperature / top-k /
        # multinomial on the device (iron_sample_topk)
        self.sampling = sampling
        self.dev = torch.device("cuda", torch.cuda.current_device())
        self.flags = _lib.IRON_FLAG_PDL if pdl else 0
        s, dev = shape, self.dev
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        E, Hd = s.emb_dim, s.head_dim
        self.layers = []
        if weights is not None:
            self._load_weights(weights, keep_natural)
        for _ in range(s.n_layers if weights is None else 0):
            lay = {
                "n1": (1 + 0.02 * torch.randn(E, device=dev, generator=g)).to(torch.bfloat16),
                "n2": (1 + 0.02 * torch.randn(E, device=dev, generator=g)).to(torch.bfloat16),
                "qkv": Int4Matrix(s.qkv_dim, E, g, 0.001, 0.004, keep_natural),
                "o": Int4Matrix(E, s.n_heads * Hd, g, 0.001, 0.004, keep_natural),
                # gate rows then up rows, interleaved per 8 rows (see interleave_gate_up)
                "gu": Int4Matrix(2 * s.hidden_dim, E, g, 0.001, 0.004, keep_natural),
                "d": Int4Matrix(E, s.hidden_dim, g, 0.0005, 0.002, keep_natural),
            }
            self.layers.append(lay)
        if weights is None:
            self.nf = (1 + 0.02 * torch.randn(E, device=dev, generator=g)).to(torch.bfloat16)
            self.lm = Int4Matrix(s.vocab_size, E, g, 0.001, 0.004, keep_natural=True)
            self.embed_table = self.lm.dequant()  # tied: the embedding is the dequantized lm-head
            if not keep_natural:
                self.lm.codes = self.lm.scales = None
        self.lut = rope_table(Hd, max_seq, s.rope_base, dev)
        B = batch
        self.kc = torch.zeros(s.n_layers, B, s.n_kv_groups, max_seq, Hd, dtype=torch.bfloat16, device=dev)
        self.vc = torch.zeros_like(self.kc)
        bf = dict(dtype=torch.bfloat16, device=dev)
        self.x = torch.zeros(B, E, **bf)
        self.xn = torch.zeros(B, E, **bf)
        self.h = torch.zeros(B, E, **bf)
        self.qkv = torch.zeros(B, s.qkv_dim, **bf)
        self.q = torch.zeros(B, s.n_heads, Hd, **bf)
        self.attn = torch.zeros(B, s.n_heads * Hd, **bf)
        self.act = torch.zeros(B, s.hidden_dim, **bf)
        self.logits = torch.zeros(B, s.vocab_size, **bf)
        self.tokens = torch.zeros(B, dtype=torch.int32, device=dev)
        self.pos = torch.zeros(B, dtype=torch.int32, device=dev)
        self.lens = torch.zeros(B, dtype=torch.int32, device=dev)
        wsb = max(_lib.load().iron_attn_decode_workspace_bytes(B, s.n_heads, s.n_kv_groups, max_seq),
                  _lib.load().iron_attn_decode_qkv_workspace_bytes(B, s.n_heads, s.n_kv_groups, max_seq, s.head_dim))
        self.attn_ws = torch.zeros(max(wsb, 16), dtype=torch.uint8, device=dev)
        self.amax = torch.zeros(B * 32, dtype=torch.int64, device=dev)  # fused argmax key slots
        self.graph = None
        self.graph_io = None  # capture_host_io
        # where the RMSNorms run: "chain" (B <= 8) folds them into the GEMVs around them
        # (iron_gemv_int4g32_chain: the residual GEMVs write bf16(h * w) and per-16-row
        # sums of squares, the next GEMV scales its output by 1 / rms -- no norm kernels);
        # "none": RMSNorm kernels; "layers" / "all": RMSNorm recomputed in the QKV and
        # gate/up (and lm-head) GEMVs' prologue. RoPE inside attention (whose cached K / V
        # rows are then requested before the wait for the QKV projection) saves 44 us per
        # step at B = 1, 62 us at B = 8 and 305 us at B = 64 (B200).
        self.fuse_norm = fuse_norm if fuse_norm is not None else ("chain" if B <= 8 else "none")
        if self.fuse_norm not in ("chain", "none", "layers", "all"):
            raise ValueError(f"unknown fuse_norm {self.fuse_norm!r}")
        if self.fuse_norm != "none" and B > 8:
            raise ValueError("the fused RMSNorm forms serve B <= 8")
        if self.fuse_norm == "chain":
            self.xw = torch.zeros(B, E, dtype=torch.bfloat16, device=dev)  # bf16(x * w) inputs
            self.hw = torch.zeros(B, E, dtype=torch.bfloat16, device=dev)
            self.ss_x = torch.zeros(B, E // 16, dtype=torch.float32, device=dev)  # their sums of squares
            self.ss_h = torch.zeros(B, E // 16, dtype=torch.float32, device=dev)
        # RoPE + KV append inside the attention kernel (else the rope_kv_append kernel)
        self.fuse_rope = fuse_rope if fuse_rope is not None else True
        # each layer's gate/up and down weights requested into L2 on a side branch of
        # the step (off the dependent chain) when the layer starts
        self.l2_prefetch = bool(l2_prefetch) if l2_prefetch is not None else False
        self._side = torch.cuda.Stream() if self.l2_prefetch else None

    def _load_weights(self, state: dict, keep_natural: bool):
        """Bind a checkpoint's tensors (IRON's names, llama_npu.py:588-639) and quantize the
        projections: q / k / v stacked into the QKV matrix, gate and up interleaved per 8
        rows (interleave_gate_up), the head from lm_head.weight or the tied embedding."""
        from . import weights as W

        s, dev = self.s, self.dev
        W.check_checkpoint(state, s)

        def dense(name):
            return state[name].to(device=dev, dtype=torch.bfloat16)

        perm = interleave_gate_up(s.hidden_dim).to(dev)
        for i in range(s.n_layers):
            qkv = torch.cat([dense(W.layer_name(i, k)) for k in ("q", "k", "v")])
            gu = torch.cat([dense(W.layer_name(i, "g")), dense(W.layer_name(i, "u"))])[perm]
            self.layers.append({
                "n1": dense(W.layer_name(i, "n1")), "n2": dense(W.layer_name(i, "n2")),
                "qkv": Int4Matrix.from_dense(qkv, keep_natural),
                "o": Int4Matrix.from_dense(dense(W.layer_name(i, "o")), keep_natural),
                "gu": Int4Matrix.from_dense(gu, keep_natural),
                "d": Int4Matrix.from_dense(dense(W.layer_name(i, "d")), keep_natural),
            })
        self.nf = dense(W.FINAL_NORM)
        self.embed_table = dense(W.EMBED).contiguous()
        self.lm = Int4Matrix.from_dense(dense(W.LM_HEAD if W.LM_HEAD in state else W.EMBED), keep_natural)

    # -- bytes moved per step (the roofline numerator) ---------------------------------
    def weight_bytes(self) -> int:
        return self.s.weight_params() * 9 // 16  # 0.5 B codes + 2 B / 32 scales per weight

    def kv_bytes(self, positions) -> int:
        """K and V bytes the attention reads for sequences at the given positions."""
        s = self.s
        return int(sum(int(p) + 1 for p in positions)) * s.n_layers * 2 * s.n_kv_groups * s.head_dim * 2

    # -- one decode step ----------------------------------------------------------------
    def _launch_step(self, stream: int):
        self._launch_step_graph_kernels(stream)

    def check_status(self):
        """The step's kernels have no device-side waits to report on (kept for callers
        that check every engine after a step)."""

    def _launch_step_graph_kernels(self, stream: int):
        """The step as a chain of kernels: per layer QKV GEMV (RMSNorm fused for
        B <= 8), fused RoPE + KV append + attention (+ split merge), O GEMV +
        residual, gate/up GEMV (RMSNorm fused) + SwiGLU, down GEMV + residual; then
        the lm-head GEMV with the final RMSNorm and the argmax fused, and the token
        update."""
        if self.fuse_norm == "chain":
            return self._launch_step_chain(stream)
        s, B, f = self.s, self.B, self.flags
        # the step keeps the PDL windows the read-only activation path needs (its o_proj
        # and down_proj GEMVs add residuals and so bound each layer's two windows)
        fg = f | _lib.IRON_FLAG_X_READONLY
        call, p = _lib.call, (lambda t: t.data_ptr())
        E, Hd, L = s.emb_dim, s.head_dim, self.L
        kv_b, kv_h = s.n_kv_groups * L * Hd, L * Hd
        fuse_norm = self.fuse_norm != "none"
        main = torch.cuda.ExternalStream(stream) if self.l2_prefetch else None
        call("iron_embed", p(self.tokens), p(self.embed_table), p(self.x), B, E, s.vocab_size, f, stream)
        for li, lay in enumerate(self.layers):
            kc, vc = self.kc[li], self.vc[li]
            if self.l2_prefetch:
                fork = torch.cuda.Event()
                fork.record(main)
                self._side.wait_event(fork)
                for m in ("gu", "d"):
                    call("iron_l2_prefetch", p(lay[m].packed), lay[m].packed.numel(), 0, self._side.cuda_stream)
            if fuse_norm:
                call("iron_gemv_int4g32_ex", p(lay["qkv"].packed), p(self.x), p(self.qkv), s.qkv_dim, E, B, None,
                     p(lay["n1"]), s.eps, None, fg, stream)
            else:
                call("iron_rmsnorm", p(self.x), None, None, p(lay["n1"]), p(self.xn), B, E, s.eps, f, stream)
                call("iron_gemv_int4g32", p(lay["qkv"].packed), p(self.xn), p(self.qkv), s.qkv_dim, E, B,
                     None, fg, stream)
            if self.fuse_rope:
                call("iron_attn_decode_qkv", p(self.qkv), p(self.pos), p(self.lut), p(kc), p(vc), p(self.attn), B,
                     s.n_heads, s.n_kv_groups, Hd, L, kv_b, kv_h, 1.0 / math.sqrt(Hd), p(self.attn_ws),
                     self.attn_ws.numel(), f, stream)
            else:
                call("iron_rope_kv_append", p(self.qkv), p(self.pos), p(self.lut), p(self.q), p(kc), p(vc),
                     p(self.lens), B, s.n_heads, s.n_kv_groups, Hd, kv_b, kv_h, f, stream)
                call("iron_attn_decode", p(self.q), p(kc), p(vc), p(self.lens), p(self.attn), B, s.n_heads,
                     s.n_kv_groups, Hd, L, kv_b, kv_h, 1.0 / math.sqrt(Hd), p(self.attn_ws),
                     self.attn_ws.numel(), f, stream)
            call("iron_gemv_int4g32", p(lay["o"].packed), p(self.attn), p(self.h), E, s.n_heads * Hd, B,
                 p(self.x), fg, stream)
            if fuse_norm:
                call("iron_gemv_int4g32_ex", p(lay["gu"].packed), p(self.h), p(self.act), 2 * s.hidden_dim, E, B,
                     None, p(lay["n2"]), s.eps, None, fg | _lib.IRON_FLAG_SWIGLU, stream)
            else:
                call("iron_rmsnorm", p(self.h), None, None, p(lay["n2"]), p(self.xn), B, E, s.eps, f, stream)
                call("iron_gemv_int4g32", p(lay["gu"].packed), p(self.xn), p(self.act), 2 * s.hidden_dim, E,
                     B, None, fg | _lib.IRON_FLAG_SWIGLU, stream)
            call("iron_gemv_int4g32", p(lay["d"].packed), p(self.act), p(self.x), E, s.hidden_dim, B,
                 p(self.h), fg, stream)
        amax = None if self.sampling is not None else p(self.amax)
        if self.fuse_norm == "all":
            call("iron_gemv_int4g32_ex", p(self.lm.packed), p(self.x), p(self.logits), s.vocab_size, E, B, None,
                 p(self.nf), s.eps, amax, fg, stream)
        else:
            call("iron_rmsnorm", p(self.x), None, None, p(self.nf), p(self.xn), B, E, s.eps, f, stream)
            call("iron_gemv_int4g32_ex", p(self.lm.packed), p(self.xn), p(self.logits), s.vocab_size, E, B, None,
                 None, 0.0, amax, fg, stream)
        if self.sampling is None:
            call("iron_argmax_finalize", p(self.amax), p(self.tokens), p(self.pos), B, f, stream)
        else:
            sp = self.sampling
            call("iron_sample_topk", p(self.logits), B, s.vocab_size, sp.temperature, sp.top_k, sp.seed,
                 p(self.tokens), p(self.pos), f, stream)
        if self.l2_prefetch:
            join = torch.cuda.Event()
            join.record(self._side)
            main.wait_event(join)

    def _launch_step_chain(self, stream: int):
        """The step with the RMSNorms folded into the GEMVs (5 kernels per layer at batch 1
        and 2): the embedding gather writes x, bf16(x * n1) and x's sums of squares; per
        layer the QKV GEMV scales by 1 / rms(x), attention (RoPE + append + splits), the O
        GEMV adds the residual and writes h, bf16(h * n2) and h's sums of squares, the
        gate/up GEMV scales by 1 / rms(h) before SwiGLU, the down GEMV adds the residual and
        writes the next layer's inputs (with n1 of the next layer, or the final norm's
        weights); the lm-head scales by 1 / rms and picks the token."""
        s, B, f = self.s, self.B, self.flags
        fg = f | _lib.IRON_FLAG_X_READONLY  # the windows hold as in _launch_step_graph_kernels
        call, p = _lib.call, (lambda t: t.data_ptr())
        E, Hd, L = s.emb_dim, s.head_dim, self.L
        kv_b, kv_h = s.n_kv_groups * L * Hd, L * Hd
        C = _lib.GemvChain

        def chain(packed, x, y, N, K, c, flags):
            call("iron_gemv_int4g32_chain", p(packed), p(x), p(y), N, K, B, ctypes.byref(c), flags, stream)

        call("iron_embed_chain", p(self.tokens), p(self.embed_table), p(self.x), p(self.xw),
             p(self.layers[0]["n1"]), p(self.ss_x), B, E, s.vocab_size, f, stream)
        for li, lay in enumerate(self.layers):
            kc, vc = self.kc[li], self.vc[li]
            nxt = self.layers[li + 1]["n1"] if li + 1 < len(self.layers) else self.nf
            chain(lay["qkv"].packed, self.xw, self.qkv, s.qkv_dim, E, C(ss_in=p(self.ss_x), eps=s.eps), fg)
            call("iron_attn_decode_qkv", p(self.qkv), p(self.pos), p(self.lut), p(kc), p(vc), p(self.attn), B,
                 s.n_heads, s.n_kv_groups, Hd, L, kv_b, kv_h, 1.0 / math.sqrt(Hd), p(self.attn_ws),
                 self.attn_ws.numel(), f, stream)
            chain(lay["o"].packed, self.attn, self.h, E, s.n_heads * Hd,
                  C(residual=p(self.x), ss_out=p(self.ss_h), y_weighted=p(self.hw), weight=p(lay["n2"])), fg)
            chain(lay["gu"].packed, self.hw, self.act, 2 * s.hidden_dim, E, C(ss_in=p(self.ss_h), eps=s.eps),
                  fg | _lib.IRON_FLAG_SWIGLU)
            chain(lay["d"].packed, self.act, self.x, E, s.hidden_dim,
                  C(residual=p(self.h), ss_out=p(self.ss_x), y_weighted=p(self.xw), weight=p(nxt)), fg)
        amax = p(self.amax) if self.sampling is None else None
        chain(self.lm.packed, self.xw, self.logits, s.vocab_size, E,
              C(ss_in=p(self.ss_x), eps=s.eps, argmax_keys=amax), fg)
        if self.sampling is None:
            call("iron_argmax_finalize", p(self.amax), p(self.tokens), p(self.pos), B, f, stream)
        else:
            sp = self.sampling
            call("iron_sample_topk", p(self.logits), B, s.vocab_size, sp.temperature, sp.top_k, sp.seed,
                 p(self.tokens), p(self.pos), f, stream)

    # -- prefill: a whole prompt through the tensor-core GEMMs -----------------------------
    def _prefill_buffers(self, S: int):
        S = -(-S // 64) * 64  # the attention writes its padded rows (zeros) too
        if getattr(self, "_pf_S", 0) >= S:
            return
        s, dev = self.s, self.dev
        bf = dict(dtype=torch.bfloat16, device=dev)
        E, H = s.emb_dim, s.hidden_dim
        self._pf = {
            "x": torch.empty(S, E, **bf), "xn": torch.empty(S, E, **bf), "h": torch.empty(S, E, **bf),
            "qkv": torch.empty(S, s.qkv_dim, **bf), "q": torch.empty(S, s.n_heads, s.head_dim, **bf),
            "attn": torch.empty(S, s.n_heads * s.head_dim, **bf), "act": torch.empty(S, H, **bf),
            "w": torch.empty(2 * H * E, **bf),  # one layer matrix, dequantized
            "pos": torch.arange(S, dtype=torch.int32, device=dev), "lens": torch.empty(S, dtype=torch.int32, device=dev),
            "tok": torch.empty(S, dtype=torch.int32, device=dev),
        }
        self._pf_S = S

    def _gemm(self, A, mat, C, M, residual=None, swiglu=False, stream=0):
        """C = A . dequant(mat)^T (+ residual | SwiGLU) on the tcgen05 tensor cores."""
        p, w = (lambda t: t.data_ptr()), self._pf["w"]
        _lib.call("iron_unpack_int4g32", p(mat.packed), p(w), mat.rows, mat.cols, stream)
        N, K = mat.rows, mat.cols
        _lib.call("iron_gemm_bf16", p(A), p(w), p(C), M, N, K, K, K, N // 2 if swiglu else N,
                  p(residual) if residual is not None else None, N if residual is not None else 0,
                  _lib.IRON_GEMM_EPI_SWIGLU if swiglu else 0, 0, 0.0, 0.0, 0, self.flags, stream)

    def _launch_prefill(self, S: int, seq: int, stream: int):
        s, f, pf = self.s, self.flags, self._pf
        call, p = _lib.call, (lambda t: t.data_ptr())
        E, Hd, L = s.emb_dim, s.head_dim, self.L
        Hq, Hk = s.n_heads, s.n_kv_groups
        kv_h = L * Hd
        qst = (ctypes.c_int64 * 3)(0, Hd, Hq * Hd)
        kvst = (ctypes.c_int64 * 3)(0, kv_h, Hd)
        call("iron_embed", p(pf["tok"]), p(self.embed_table), p(pf["x"]), S, E, s.vocab_size, f, stream)
        for li, lay in enumerate(self.layers):
            kc = self.kc[li, seq]
            vc = self.vc[li, seq]
            call("iron_rmsnorm", p(pf["x"]), None, None, p(lay["n1"]), p(pf["xn"]), S, E, s.eps, f, stream)
            self._gemm(pf["xn"], lay["qkv"], pf["qkv"], S, stream=stream)
            # every prompt token is a "sequence" of the RoPE + cache-append kernel at position t
            call("iron_rope_kv_append", p(pf["qkv"]), p(pf["pos"]), p(self.lut), p(pf["q"]), p(kc), p(vc),
                 p(pf["lens"]), S, Hq, Hk, Hd, 0, kv_h, f, stream)
            call("iron_attn_prefill", p(pf["q"]), p(kc), p(vc), p(pf["attn"]), 1, Hq, Hk, Hd, S,
                 -(-S // 64) * 64, S, qst, kvst, qst, 1.0 / math.sqrt(Hd), 1, f, stream)
            self._gemm(pf["attn"], lay["o"], pf["h"], S, residual=pf["x"], stream=stream)
            call("iron_rmsnorm", p(pf["h"]), None, None, p(lay["n2"]), p(pf["xn"]), S, E, s.eps, f, stream)
            self._gemm(pf["xn"], lay["gu"], pf["act"], S, swiglu=True, stream=stream)
            self._gemm(pf["act"], lay["d"], pf["x"], S, residual=pf["h"], stream=stream)
        # next token from the last position only
        last = pf["x"][S - 1 : S]
        xn1 = self.xn[seq : seq + 1]
        call("iron_rmsnorm", p(last), None, None, p(self.nf), p(xn1), 1, E, s.eps, f, stream)
        call("iron_gemv_int4g32", p(self.lm.packed), p(xn1), p(self.logits[seq : seq + 1]), s.vocab_size, E, 1,
             None, f, stream)
        if self.sampling is None:
            call("iron_argmax", p(self.logits[seq : seq + 1]), p(self.tokens[seq : seq + 1]), 1, s.vocab_size,
                 None, f, stream)
        else:  # the draw for the prompt's last position S - 1 (the word is advanced, then dropped)
            self._pf_draw_pos = torch.full((1,), S - 1, dtype=torch.int32, device=self.dev)
            sp = self.sampling
            call("iron_sample_topk", p(self.logits[seq : seq + 1]), 1, s.vocab_size, sp.temperature, sp.top_k,
                 sp.seed, p(self.tokens[seq : seq + 1]), p(self._pf_draw_pos), f, stream)

    def prefill(self, tokens, seq: int = 0):
        """Run a prompt through the model for sequence `seq`: fills its KV cache at
        positions 0..S-1, leaves the greedy next token in tokens[seq] and sets
        pos[seq] = S (so decode steps continue from there)."""
        toks = torch.as_tensor(tokens, dtype=torch.int32).reshape(-1)
        S = int(toks.numel())
        if S < 1 or S > self.L:
            raise ValueError(f"prompt of {S} tokens does not fit the cache ({self.L})")
        self._prefill_buffers(S)
        self._pf["tok"][:S].copy_(toks)
        self._launch_prefill(S, seq, torch.cuda.current_stream().cuda_stream)
        self.pos[seq] = S
        self.lens[seq] = S

    def prefill_flops(self, S: int) -> int:
        """Tensor-core FLOPs of the prefill GEMMs and attention for an S-token prompt."""
        s = self.s
        E, H, Q, Hd = s.emb_dim, s.hidden_dim, s.qkv_dim, s.head_dim
        gemm = 2 * S * (Q * E + E * s.n_heads * Hd + 2 * H * E + E * H)
        attn = 4 * s.n_heads * Hd * S * (S + 1) // 2
        return s.n_layers * (gemm + attn)

    def kernels_per_step(self) -> int:
        attn = _lib.load().iron_attn_decode_kernels(self.B, self.s.n_heads, self.s.n_kv_groups, self.L)
        if self.fuse_norm == "chain":
            return 1 + self.s.n_layers * (4 + attn) + 2
        per_layer = ((4 if self.fuse_norm != "none" else 6) + attn + (0 if self.fuse_rope else 1)
                     + (2 if self.l2_prefetch else 0))
        return 1 + self.s.n_layers * per_layer + (2 if self.fuse_norm == "all" else 3)

    def set_state(self, tokens, positions):
        self.tokens.copy_(torch.as_tensor(tokens, dtype=torch.int32))
        self.pos.copy_(torch.as_tensor(positions, dtype=torch.int32))

    def step(self):
        """One decode step (graph replay once captured)."""
        if self.graph is not None:
            self.graph.replay()
        else:
            self._launch_step(torch.cuda.current_stream().cuda_stream)

    def capture_host_io(self):
        """Capture a second decode step whose graph also moves the token ids between host
        and device: it copies `host_tokens_in` (pinned, [B] int32) into the device before
        the step and the step's tokens into `host_tokens_out` (pinned) after it, so a host
        loop that feeds and reads token ids every step -- IRON's decode loop reads the
        result back every token (iron/common/sequence.py:721-730) -- launches one graph
        per token. `step_host` replays it; host_tokens_out is valid once the stream has
        synchronised."""
        B = self.B
        self.host_tokens_in = torch.zeros(B, dtype=torch.int32).pin_memory()
        self.host_tokens_out = torch.zeros(B, dtype=torch.int32).pin_memory()
        self.host_tokens_in.copy_(self.tokens.cpu())
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        saved_tok, saved_pos = self.tokens.clone(), self.pos.clone()
        torch.cuda.synchronize()
        self.graph_io = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph_io, stream=s):
            self.tokens.copy_(self.host_tokens_in, non_blocking=True)
            self._launch_step(s.cuda_stream)
            self.host_tokens_out.copy_(self.tokens, non_blocking=True)
        torch.cuda.synchronize()
        self.tokens.copy_(saved_tok)
        self.pos.copy_(saved_pos)
        torch.cuda.synchronize()

    def step_host(self):
        """One decode step of the host-I/O graph (capture_host_io): reads host_tokens_in,
        writes host_tokens_out."""
        self.graph_io.replay()

    def capture(self):
        """Capture one decode step as a CUDA graph (positions/tokens are device state)."""
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        saved_tok, saved_pos = self.tokens.clone(), self.pos.clone()
        with torch.cuda.stream(s):
            self._launch_step(s.cuda_stream)  # warm-up outside capture
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        self.tokens.copy_(saved_tok)
        self.pos.copy_(saved_pos)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=s):
            self._launch_step(s.cuda_stream)
        torch.cuda.synchronize()
        self.tokens.copy_(saved_tok)
        self.pos.copy_(saved_pos)
        torch.cuda.synchronize()
