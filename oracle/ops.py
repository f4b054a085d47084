"""Floating-point goldens of the hot path, restated on the CPU (test oracle).

Every function follows IRON's own torch golden for the operator (cited per
function), computing in fp32 and rounding to bf16 once at the end, which is what
those goldens do or tolerate. Inputs and outputs are torch CPU tensors.
"""

from __future__ import annotations

import contextlib
import math

import numpy as np
import torch

BF16 = torch.bfloat16

# The arithmetic type of the restated goldens: fp32, as IRON's goldens compute. A test
# may rerun the oracle in fp64 (same bf16 rounding points) to measure how sensitive a
# result is to the precision of its sums -- the spread a correct fp32 implementation
# with another summation order can show.
_ACC = [torch.float32]
# The type every restated operator rounds its output to: bf16 (the operators' buffers).
# IRON's accuracy reference is the CPU model run in fp32 throughout
# (iron/applications/llama_3.2_1b/llama_npu.py:1239-1241): fp32 here, no bf16 rounding.
_OUT = [BF16]


@contextlib.contextmanager
def accumulate(dtype):
    """Run the oracle's arithmetic in `dtype` inside the block (rounding points unchanged)."""
    old, _ACC[0] = _ACC[0], dtype
    try:
        yield
    finally:
        _ACC[0] = old


@contextlib.contextmanager
def fp32_reference():
    """Inside the block every operator keeps fp32 outputs (IRON's fp32 CPU reference)."""
    old, _OUT[0] = _OUT[0], torch.float32
    try:
        yield
    finally:
        _OUT[0] = old


def _f(t: torch.Tensor) -> torch.Tensor:
    return t.to(_ACC[0])


def gemv(A: torch.Tensor, B: torch.Tensor) -> torch.Tensor:
    """C = A @ B, fp32 accumulate, bf16 out (iron/operators/gemv/reference.py:9-11).
    A [M, K] or [b, M, K]; B [K] or [b, K]."""
    Af, Bf = _f(A), _f(B)
    if A.dim() == 3:
        return torch.einsum("bmk,bk->bm", Af, Bf).to(_OUT[0])
    return (Af @ Bf).to(_OUT[0])


def gemv_multi(A: torch.Tensor, X: torch.Tensor) -> torch.Tensor:
    """One matrix, a batch of vectors: Y[v] = A @ X[v] (decode batch)."""
    return (_f(X) @ _f(A).T).to(_OUT[0])


def gelu_tanh(x: torch.Tensor) -> torch.Tensor:
    """Tanh-approximation GELU (iron/operators/gemv/reference.py:59-66)."""
    xf = _f(x)
    return 0.5 * xf * (1.0 + torch.tanh(0.7978845608028654 * (xf + 0.044715 * xf**3)))


def rms_norm(x: torch.Tensor, w: torch.Tensor | None = None, eps: float = 1e-5) -> torch.Tensor:
    """x / sqrt(mean(x^2) + eps) [* w] row-wise (iron/operators/rms_norm/reference.py:7-16)."""
    xf = _f(x)
    out = xf / torch.sqrt(torch.mean(xf * xf, dim=-1, keepdim=True) + eps)
    if w is not None:
        out = out * _f(w)
    return out.to(_OUT[0])


def rope(x: torch.Tensor, angles: torch.Tensor, method_type: int = 0) -> torch.Tensor:
    """Rotary embedding from the interleaved [cos, sin, ...] table; angle row
    r // (rows / angle_rows) for row r; fp32, rounded once
    (iron/operators/rope/reference.py:69-102)."""
    rows = x.shape[0]
    rep = rows // angles.shape[0]
    cos = _f(angles[..., 0::2]).repeat_interleave(rep, dim=0)
    sin = _f(angles[..., 1::2]).repeat_interleave(rep, dim=0)
    xf = _f(x)
    if method_type == 0:
        half = x.shape[-1] // 2
        x1, x2 = xf[..., :half], xf[..., half:]
        y = torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1)
    else:
        xe, xo = xf[..., 0::2], xf[..., 1::2]
        y = torch.empty_like(xf)
        y[..., 0::2] = xe * cos - xo * sin
        y[..., 1::2] = xe * sin + xo * cos
    return y.to(_OUT[0])


def softmax(x: torch.Tensor, valid: int | None = None) -> torch.Tensor:
    """Row softmax in fp32 (iron/operators/softmax/reference.py:9-11). With
    ``valid``, columns >= valid are first set to -inf as the device's mask_bf16
    does (iron/operators/softmax/design.py:85-91)."""
    xf = _f(x)
    if valid is not None:
        xf = xf.clone()
        xf[..., valid:] = -math.inf
    return torch.softmax(xf, dim=-1).to(_OUT[0])


def silu(x: torch.Tensor) -> torch.Tensor:
    """iron/operators/silu/reference.py:7-9."""
    return torch.nn.functional.silu(_f(x)).to(_OUT[0])


def mul(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """iron/operators/elementwise_mul/reference.py:7-9."""
    return (_f(a) * _f(b)).to(_OUT[0])


def add(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """iron/operators/elementwise_add/reference.py:7-9."""
    return (_f(a) + _f(b)).to(_OUT[0])


def swiglu_act(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """silu(gate) * up, the SiLU + ElementwiseMul steps of SwiGLUDecode
    (iron/operators/swiglu_decode/op.py:56-62), fused."""
    g = _f(gate)
    return (g * torch.sigmoid(g) * _f(up)).to(_OUT[0])


def repeat_interleave(x: torch.Tensor, repeat: int) -> torch.Tensor:
    """iron/operators/repeat/reference.py:7-9."""
    return x.repeat_interleave(repeat, dim=0)


def transpose(x: torch.Tensor) -> torch.Tensor:
    """Per-matrix transpose (iron/operators/transpose/reference.py:7-10)."""
    return x.transpose(-2, -1).contiguous()


# ---- StridedCopy (exact index arithmetic) ---------------------------------
def _pad4(sizes, strides):
    return [1] * (4 - len(sizes)) + list(sizes), [0] * (4 - len(strides)) + list(strides)


def _tap(sizes, strides, offset):
    grids = np.meshgrid(*[np.arange(s) for s in sizes], indexing="ij")
    flat = np.full(grids[0].shape, offset, dtype=np.int64)
    for g, st in zip(grids, strides):
        flat = flat + g * st
    return flat.reshape(-1)


def _channels(sizes, strides, offset, ch):
    sizes, strides = _pad4(sizes, strides)
    hi = max(i for i, s in enumerate(sizes) if s >= 1)
    per = sizes[hi] // ch
    split = sizes[:hi] + [per] + sizes[hi + 1 :]
    return [_tap(split, strides, offset + c * per * strides[hi]) for c in range(ch)]


def strided_copy(inp, in_sizes, in_strides, in_offset, out_size, out_sizes, out_strides,
                 out_offset, channels=1, in_addend=0, out_addend=0, out=None):
    """Gather by the input access pattern, scatter by the output one, channel by
    channel; addends are element counts (iron/operators/strided_copy/reference.py:37-75).
    ``out`` (if given) is updated in place, otherwise a zero buffer is used."""
    src = _channels(in_sizes, in_strides, in_offset + in_addend, channels)
    dst = _channels(out_sizes, out_strides, out_offset + out_addend, channels)
    res = torch.zeros(int(out_size), dtype=inp.dtype) if out is None else out.clone()
    for s, d in zip(src, dst):
        if len(s) != len(d):
            raise ValueError("tap element counts differ")
        res[torch.from_numpy(d)] = inp[torch.from_numpy(s)]
    return res


# ---- attention ------------------------------------------------------------
def mha_prefill(Q, K, V, causal=True, chunk=1024):
    """Causal SDPA with GQA via repeat_interleave, scale 1/sqrt(d), fp32
    (iron/operators/mha/reference.py:27-94). Q [H, S, d], K/V [Hkv, S_kv, d].
    Query rows are processed `chunk` at a time (same math, bounded memory)."""
    g = Q.shape[0] // K.shape[0]
    H, S, d = Q.shape
    out = torch.empty(H, S, V.shape[-1], dtype=_OUT[0])
    for h in range(H):
        Kh = _f(K[h // g])
        Vh = _f(V[h // g])
        for r0 in range(0, S, chunk):
            q = _f(Q[h, r0 : r0 + chunk])
            s = q @ Kh.T / math.sqrt(d)
            if causal:
                rows = torch.arange(r0, r0 + q.shape[0]).unsqueeze(1)
                cols = torch.arange(Kh.shape[0]).unsqueeze(0)
                s = s.masked_fill(cols > rows, -math.inf)
            out[h, r0 : r0 + chunk] = (torch.softmax(s, dim=-1) @ Vh).to(_OUT[0])
    return out


def attn_decode(q, k_cache, v_cache, lens):
    """One-query GQA attention per sequence over its first ``lens[b]`` cache
    entries: softmax(q K^T / sqrt(d)) V in fp32 (the decode steps 5-9 of
    iron/applications/llama_3.2_1b/llama_cpu.py:118-140).
    q [B, Hq, d]; caches [B, Hkv, Lmax, d]; returns bf16 [B, Hq, d]."""
    B, Hq, d = q.shape
    Hkv = k_cache.shape[1]
    g = Hq // Hkv
    out = torch.empty(B, Hq, d, dtype=_OUT[0])
    for b in range(B):
        L = int(lens[b])
        K = _f(k_cache[b, :, :L]).repeat_interleave(g, dim=0)
        V = _f(v_cache[b, :, :L]).repeat_interleave(g, dim=0)
        s = torch.einsum("hd,hld->hl", _f(q[b]), K) / math.sqrt(d)
        out[b] = torch.einsum("hl,hld->hd", torch.softmax(s, dim=-1), V).to(_OUT[0])
    return out


def sample_probs(logits: torch.Tensor, temperature: float, top_k: int | None) -> torch.Tensor:
    """Next-token probabilities of IRON's generate_token
    (iron/applications/llama_3.2_1b/llama_inference_harness.py:146-169): logits /
    temperature (when > 0), then every logit below the top_k-th largest set to -inf
    (ties kept), then softmax; fp64 here. logits [B, V] -> probabilities [B, V]."""
    lf = logits.double()
    if temperature > 0:
        lf = lf / temperature
    if top_k is not None and 0 < top_k < lf.shape[-1]:
        kth = torch.topk(lf, top_k, dim=-1).values[..., -1:]
        lf = torch.where(lf < kth, torch.tensor(float("-inf"), dtype=lf.dtype), lf)
    return torch.softmax(lf, dim=-1)


# ---- Llama pieces ------------------------------------------------------------
def rope_angles(head_dim: int, context_length: int, base: float = 500000.0) -> torch.Tensor:
    """Interleaved cos/sin table (iron/applications/llama_3.2_1b/llama_inference_harness.py:109-123)."""
    inv_freq = 1.0 / (base ** (torch.arange(0, head_dim, 2).float() / head_dim))
    freqs = torch.outer(torch.arange(context_length).float(), inv_freq)
    angles = torch.empty(context_length, head_dim)
    angles[:, ::2] = torch.cos(freqs)
    angles[:, 1::2] = torch.sin(freqs)
    return angles


def gemm(A: torch.Tensor, B: torch.Tensor, b_col_maj: bool = False, c_col_maj: bool = False) -> torch.Tensor:
    """C = A @ B from stored layouts (iron/operators/gemm/reference.py:7-18), fp32
    accumulation, bf16 out."""
    Bm = B.T if b_col_maj else B
    C = (_f(A) @ _f(Bm)).to(_OUT[0])
    return C.T if c_col_maj else C


def flm_gemm(A: torch.Tensor, B: torch.Tensor, epilogue: str = "none", clamp=None) -> torch.Tensor:
    """flm GEMM (iron/operators/flm/gemm/reference.py:8-57): fp32 accumulation,
    conversion to bf16, then the activation (gelu = x*sigmoid(1.702x)) and the
    clamp, evaluated in bf16 torch ops as the golden does."""
    C = (_f(A) @ _f(B)).to(A.dtype)
    if epilogue == "gelu":
        C = C * torch.sigmoid(1.702 * C)
    elif epilogue == "silu":
        C = C * torch.sigmoid(C)
    elif epilogue == "sigmoid":
        C = torch.sigmoid(C)
    if clamp is not None:
        C = torch.clamp(C, clamp[0], clamp[1])
    return C
