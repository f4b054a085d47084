"""Real weights for the decode engine: a Llama-3.2-1B checkpoint in safetensors with the
Hugging Face tensor names, quantized to int4 group-32 for the int4 GEMVs.

IRON loads the checkpoint with safetensors.torch.load_file
(iron/applications/llama_3.2_1b/llama_inference_harness.py:62-64) and binds these names
to its decode runlist's weight buffers (iron/applications/llama_3.2_1b/llama_npu.py:
588-639): per layer the two RMSNorm weights and the q / k / v / o / gate / up / down
projections ([out, in], torch Linear layout), the final norm, and the embedding table,
which is also the output head (Llama-3.2-1B ties them; a separate `lm_head.weight` is
used when the checkpoint has one). The embedding lookup keeps the bf16 table, as IRON's
decode pass embeds on the CPU (llama_npu.py:1177-1183).

Quantization (no counterpart in IRON, whose runlist multiplies bf16 weights): symmetric
signed int4 per group of 32 along the input dimension, one bf16 scale per group,
s = bf16(max|w| / 7) and q = clamp(round(w / s), -8, 7); two codes per byte, even k in the
low nibble -- the layout iron_pack_int4g32 takes.
"""

from __future__ import annotations

from pathlib import Path

import torch

LAYER_NAMES = {
    "n1": "input_layernorm.weight",
    "q": "self_attn.q_proj.weight",
    "k": "self_attn.k_proj.weight",
    "v": "self_attn.v_proj.weight",
    "o": "self_attn.o_proj.weight",
    "n2": "post_attention_layernorm.weight",
    "g": "mlp.gate_proj.weight",
    "u": "mlp.up_proj.weight",
    "d": "mlp.down_proj.weight",
}
EMBED = "model.embed_tokens.weight"
FINAL_NORM = "model.norm.weight"
LM_HEAD = "lm_head.weight"


def layer_name(i: int, key: str) -> str:
    return f"model.layers.{i}.{LAYER_NAMES[key]}"


def expected_shapes(shape) -> dict[str, tuple[int, ...]]:
    """Every tensor the engine binds, with its shape, for a LlamaShape."""
    E, H, Hd = shape.emb_dim, shape.hidden_dim, shape.head_dim
    per = {"n1": (E,), "q": (shape.n_heads * Hd, E), "k": (shape.n_kv_groups * Hd, E),
           "v": (shape.n_kv_groups * Hd, E), "o": (E, shape.n_heads * Hd), "n2": (E,), "g": (H, E), "u": (H, E),
           "d": (E, H)}
    out = {layer_name(i, k): v for i in range(shape.n_layers) for k, v in per.items()}
    out[EMBED] = (shape.vocab_size, E)
    out[FINAL_NORM] = (E,)
    return out


def check_checkpoint(state: dict, shape) -> None:
    """KeyError naming the missing tensors, ValueError naming a shape that differs."""
    want = expected_shapes(shape)
    missing = [n for n in want if n not in state]
    if missing:
        raise KeyError(f"checkpoint lacks {len(missing)} tensor(s), e.g. {missing[:4]}")
    for n, s in want.items():
        if tuple(state[n].shape) != s:
            raise ValueError(f"{n}: shape {tuple(state[n].shape)}, expected {s}")
    if LM_HEAD in state and tuple(state[LM_HEAD].shape) != want[EMBED]:
        raise ValueError(f"{LM_HEAD}: shape {tuple(state[LM_HEAD].shape)}, expected {want[EMBED]}")


def load_checkpoint(path) -> dict:
    """The checkpoint's tensors by name (safetensors.torch.load_file, as IRON loads it)."""
    from safetensors.torch import load_file

    return load_file(str(Path(path)))


def quantize_int4g32(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """w [N, K] (K % 32 == 0) -> (codes uint8 [N, K / 2], scales bf16 [N, K / 32]): per
    group of 32, s = bf16(max|w| / 7) (1 for an all-zero group), q = clamp(round(w / s),
    -8, 7) with round half to even; byte j holds q[2j] (low nibble) and q[2j + 1]."""
    if w.dim() != 2 or w.shape[1] % 32:
        raise ValueError(f"need [N, K] with K % 32 == 0, got {tuple(w.shape)}")
    N, K = w.shape
    g = w.float().reshape(N, K // 32, 32)
    amax = g.abs().amax(-1)
    s = torch.where(amax > 0, amax / 7, torch.ones_like(amax)).to(torch.bfloat16)
    q = torch.clamp(torch.round(g / s.float()[..., None]), -8, 7).to(torch.int16).reshape(N, K)
    u = (q & 0xF).to(torch.uint8)
    codes = (u[:, 0::2] | (u[:, 1::2] << 4)).contiguous()
    return codes, s.contiguous()


def dequantize_int4g32(codes: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """Inverse of the packing: bf16(q * s) [N, K] (the values the int4 GEMVs multiply)."""
    lo = (codes & 0xF).to(torch.int16)
    hi = (codes >> 4).to(torch.int16)
    q = torch.stack([lo, hi], -1).reshape(codes.shape[0], -1)
    q = torch.where(q >= 8, q - 16, q).float()
    return (q * scales.float().repeat_interleave(32, dim=1)).to(torch.bfloat16)
