"""Llama-3.2-1B decode block and model, composed from the oracle ops (test oracle).

Follows iron/applications/llama_3.2_1b/llama_cpu.py:170-218 (transformer block:
RMSNorm -> GQA attention with RoPE and KV-cache append -> residual -> RMSNorm ->
SwiGLU -> residual) and :221-285 (embedding, 16 blocks, final norm, tied
lm-head). Intermediates are rounded to bf16 at the same points as the B200
pipeline stores them, so a kernel-by-kernel comparison is tight; the fp32
golden (llama_cpu run in fp32) is the accuracy reference.
"""

from __future__ import annotations

import math

import torch

from . import ops

BF16 = torch.bfloat16


def _normed_gemv(W, x, w, eps, fold):
    """GEMV of the RMSNorm of x. fold=False: IRON's order, gemv(W, bf16(x * inv * w)).
    fold=True: the RMSNorm folded into the GEMV as the B200 decode chain does it --
    bf16(inv * (W . bf16(x * w))), inv = 1 / sqrt(mean(x^2) + eps) from the bf16 x."""
    if not fold:
        return ops.gemv_multi(W, ops.rms_norm(x, w, eps))
    xf = ops._f(x)
    inv = 1.0 / torch.sqrt((xf * xf).mean(-1, keepdim=True) + eps)
    xw = (xf * ops._f(w)).to(BF16)
    return ((ops._f(xw) @ ops._f(W).T) * inv).to(ops._OUT[0])


def _normed_swiglu(Wg, Wu, x, w, eps, fold):
    """SwiGLU of the gate / up projections of the RMSNorm of x (fold as in _normed_gemv)."""
    if not fold:
        xn = ops.rms_norm(x, w, eps)
        return ops.swiglu_act(ops.gemv_multi(Wg, xn), ops.gemv_multi(Wu, xn))
    return ops.swiglu_act(_normed_gemv(Wg, x, w, eps, True), _normed_gemv(Wu, x, w, eps, True))


def block_decode(x, k_cache, v_cache, pos, W, angles, n_heads, n_kv, head_dim, eps=1e-5, fold=False):
    """One decode step of one block for a batch of sequences.

    x [B, E] bf16; caches [B, n_kv, Lmax, hd] bf16 (updated in place at slot pos[b]);
    pos [B] ints (tokens already cached); W dict of bf16 weights with keys
    n1 q k v o n2 g u d (linear weights [out, in]); angles [ctx, hd] table.
    fold: the RMSNorms folded into the GEMVs' rounding points (_normed_gemv).
    Returns the block output [B, E] bf16.
    """
    B, E = x.shape
    q = _normed_gemv(W["q"], x, W["n1"], eps, fold).view(B, n_heads, head_dim)
    k = _normed_gemv(W["k"], x, W["n1"], eps, fold).view(B, n_kv, head_dim)
    v = _normed_gemv(W["v"], x, W["n1"], eps, fold).view(B, n_kv, head_dim)
    lens = []
    for b in range(B):
        p = int(pos[b])
        ang = angles[p : p + 1]
        q[b] = ops.rope(q[b], ang)
        k[b] = ops.rope(k[b], ang)
        k_cache[b, :, p] = k[b]
        v_cache[b, :, p] = v[b]
        lens.append(p + 1)
    attn = ops.attn_decode(q, k_cache, v_cache, lens).reshape(B, n_heads * head_dim)
    h = ops.add(x, ops.gemv_multi(W["o"], attn))
    act = _normed_swiglu(W["g"], W["u"], h, W["n2"], eps, fold)
    return ops.add(h, ops.gemv_multi(W["d"], act))


def block_decode_runlist(x, k_cache, v_cache, pos, W, angles, n_heads, n_kv, head_dim, eps=1e-5):
    """One decode step of one block for ONE sequence, rounded to bf16 at the operator
    boundaries of IRON's fused decode runlist
    (iron/applications/llama_3.2_1b/llama_npu.py:459-557): the scores GEMV, the scale
    multiply, the masked Softmax and the context GEMV each round their output, and SiLU
    rounds before the ElementwiseMul. x [1, E]; caches [n_kv, Lmax, hd] (row pos written).
    Each step is the operator's own golden (gemv, mul, softmax with its mask, silu, add).
    """
    xn = ops.rms_norm(x, W["n1"], eps)
    q = ops.gemv_multi(W["q"], xn).view(n_heads, head_dim)
    k = ops.gemv_multi(W["k"], xn).view(n_kv, head_dim)
    v = ops.gemv_multi(W["v"], xn).view(n_kv, head_dim)
    ang = angles[pos : pos + 1]
    q, k = ops.rope(q, ang), ops.rope(k, ang)
    k_cache[:, pos] = k
    v_cache[:, pos] = v
    g = n_heads // n_kv
    K = ops.repeat_interleave(k_cache, g)                       # Repeat
    V = ops.repeat_interleave(v_cache, g)
    scores = ops.gemv(K, q)                                     # batched GEMV, [h, Lmax]
    scale = torch.full_like(scores, 1.0 / math.sqrt(head_dim))
    scores = ops.mul(scores, scale)                             # ElementwiseMul by the scale buffer
    w = ops.softmax(scores, pos + 1)                            # Softmax masked past the context
    ctx = ops.gemv(ops.transpose(V), w).reshape(1, n_heads * head_dim)  # Transpose + batched GEMV
    h = ops.add(x, ops.gemv_multi(W["o"], ctx))
    hn = ops.rms_norm(h, W["n2"], eps)
    act = ops.mul(ops.silu(ops.gemv_multi(W["g"], hn)), ops.gemv_multi(W["u"], hn))
    return ops.add(h, ops.gemv_multi(W["d"], act))


def model_decode_runlist(token, pos, layers, nf, embed, lm, k_caches, v_caches, angles, n_heads, n_kv,
                         head_dim, eps=1e-5):
    """IRON's decode runlist for one token (block_decode_runlist per layer, then the
    final RMSNorm and the head GEMV). Caches [n_kv, Lmax, hd] per layer. Returns [1, V]."""
    x = embed[int(token)][None].clone()
    for li, W in enumerate(layers):
        x = block_decode_runlist(x, k_caches[li], v_caches[li], int(pos), W, angles, n_heads, n_kv, head_dim, eps)
    return ops.gemv_multi(lm, ops.rms_norm(x, nf, eps))


def block_mlp_half(x, k_cache, v_cache, pos, W, angles, n_heads, n_kv, head_dim, eps=1e-5):
    """BASELINE config 3's chain: RMSNorm -> QKV -> RoPE -> KV append, then SwiGLU
    on the normed input. Returns (q_roped [B,Hq,hd], mlp_out [B,E])."""
    B, E = x.shape
    xn = ops.rms_norm(x, W["n1"], eps)
    q = ops.gemv_multi(W["q"], xn).view(B, n_heads, head_dim)
    k = ops.gemv_multi(W["k"], xn).view(B, n_kv, head_dim)
    v = ops.gemv_multi(W["v"], xn).view(B, n_kv, head_dim)
    for b in range(B):
        p = int(pos[b])
        ang = angles[p : p + 1]
        q[b] = ops.rope(q[b], ang)
        k_cache[b, :, p] = ops.rope(k[b], ang)
        v_cache[b, :, p] = v[b]
    act = ops.swiglu_act(ops.gemv_multi(W["g"], xn), ops.gemv_multi(W["u"], xn))
    return q, ops.gemv_multi(W["d"], act)


def model_decode(tokens, pos, layers, nf, embed, lm, k_caches, v_caches, angles, n_heads, n_kv,
                 head_dim, eps=1e-5, fold=False, hidden=None):
    """One greedy decode step of the whole model (llama_cpu.py:221-285, decode form):
    embedding, the blocks, final RMSNorm, lm-head. Returns logits [B, V] (bf16).
    fold: the RMSNorms at the B200 decode chain's rounding points (_normed_gemv).
    hidden: a list that receives each block's output (the residual stream)."""
    x = embed[torch.as_tensor(tokens, dtype=torch.long)].clone()
    for li, W in enumerate(layers):
        x = block_decode(x, k_caches[li], v_caches[li], pos, W, angles, n_heads, n_kv, head_dim, eps, fold)
        if hidden is not None:
            hidden.append(x)
    return _normed_gemv(lm, x, nf, eps, fold)


def model_prefill(tokens, layers, nf, embed, lm, k_caches, v_caches, angles, n_heads, n_kv, head_dim,
                  eps=1e-5):
    """A whole prompt through the model (llama_cpu.py:221-285 at prefill: every
    position, causal attention), for one sequence. Caches [n_kv, Lmax, hd] get
    positions 0..S-1. Returns the last position's logits [1, V] (bf16)."""
    tok = torch.as_tensor(tokens, dtype=torch.long)
    S = tok.numel()
    x = embed[tok].clone()
    for li, W in enumerate(layers):
        xn = ops.rms_norm(x, W["n1"], eps)
        q = ops.gemv_multi(W["q"], xn).reshape(S * n_heads, head_dim)
        k = ops.gemv_multi(W["k"], xn).reshape(S * n_kv, head_dim)
        v = ops.gemv_multi(W["v"], xn).reshape(S, n_kv, head_dim)
        # row r of a token-major [S * heads, hd] view is token r // heads: angle row r // heads
        q = ops.rope(q, angles[:S]).reshape(S, n_heads, head_dim)
        k = ops.rope(k, angles[:S]).reshape(S, n_kv, head_dim)
        k_caches[li][:, :S] = k.transpose(0, 1)
        v_caches[li][:, :S] = v.transpose(0, 1)
        att = ops.mha_prefill(q.transpose(0, 1), k.transpose(0, 1), v.transpose(0, 1))
        h = ops.add(x, ops.gemv_multi(W["o"], att.transpose(0, 1).reshape(S, n_heads * head_dim)))
        hn = ops.rms_norm(h, W["n2"], eps)
        act = ops.swiglu_act(ops.gemv_multi(W["g"], hn), ops.gemv_multi(W["u"], hn))
        x = ops.add(h, ops.gemv_multi(W["d"], act))
    return ops.gemv_multi(lm, ops.rms_norm(x[S - 1 : S], nf, eps))
