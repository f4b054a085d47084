"""The real-weight path on the CPU: the int4 group-32 quantizer against the oracle's
int4 format (oracle/quant.py: two codes per byte, even k low, bf16(q * s)), its error
bound, and the checkpoint binding of IRON's Hugging Face names
(iron/applications/llama_3.2_1b/llama_npu.py:588-639) through a safetensors file
(llama_inference_harness.py:62-64 loads with safetensors.torch.load_file)."""

import numpy as np
import pytest
import torch

from iron_b200.applications.llama_3_2_1b import weights as W
from iron_b200.applications.llama_3_2_1b.decode import LlamaShape
from oracle import quant


def test_quantizer_format_and_error_bound():
    g = torch.Generator().manual_seed(0)
    w = (torch.randn(64, 256, generator=g) * 0.02).to(torch.bfloat16)
    w[3, 32:64] = 0  # an all-zero group: scale 1, codes 0
    codes, scales = W.quantize_int4g32(w)
    assert codes.dtype == torch.uint8 and codes.shape == (64, 128)
    assert scales.dtype == torch.bfloat16 and scales.shape == (64, 8)
    deq = W.dequantize_int4g32(codes, scales)
    # the same bits as the oracle's dequantization of the same codes / scales
    ref_bits = quant.dequant_s4g32(codes.numpy(), scales.view(torch.int16).numpy().view(np.uint16))
    assert np.array_equal(deq.view(torch.int16).numpy().view(np.uint16), ref_bits)
    # every weight within half a step of its group's grid, plus the rounding of the scale
    # (s = bf16(max / 7) may fall below max / 7: |w / s| <= 7 (1 + 2^-8)) and of bf16(q * s)
    # (half an ulp: <= 7 s 2^-9), i.e. < 0.55 s
    s = scales.float().repeat_interleave(32, dim=1)
    err = (deq.float() - w.float()).abs()
    assert bool((err < 0.55 * s).all()), float((err / s).max())
    assert float(scales[3, 1]) == 1.0 and int(codes[3, 16:32].abs().sum()) == 0
    # codes use the signed range: the group maximum maps to +-7
    q = torch.from_numpy(quant.unpack_s4(codes.numpy()).astype(np.int16))
    assert int(q.abs().max()) == 7 and int(q.min()) >= -8


def _tiny_state(shape, seed=1, tie=True):
    g = torch.Generator().manual_seed(seed)
    st = {}
    for n, s in W.expected_shapes(shape).items():
        t = torch.randn(*s, generator=g) * (0.02 if len(s) == 2 else 0.02)
        if len(s) == 1:
            t = t + 1
        st[n] = t.to(torch.bfloat16)
    if not tie:
        st[W.LM_HEAD] = (torch.randn(shape.vocab_size, shape.emb_dim, generator=g) * 0.02).to(torch.bfloat16)
    return st


def test_checkpoint_names_and_safetensors_round_trip(tmp_path):
    from safetensors.torch import save_file

    shape = LlamaShape(n_layers=2, vocab_size=512, emb_dim=256, n_heads=4, n_kv_groups=2, head_dim=64,
                       hidden_dim=512)
    st = _tiny_state(shape)
    # IRON's names, e.g. the ones llama_npu.py binds for layer 1
    for key in ("model.layers.1.input_layernorm.weight", "model.layers.1.self_attn.q_proj.weight",
                "model.layers.1.mlp.down_proj.weight", "model.norm.weight", "model.embed_tokens.weight"):
        assert key in st
    path = tmp_path / "model.safetensors"
    save_file(st, str(path))
    back = W.load_checkpoint(path)
    W.check_checkpoint(back, shape)
    assert all(torch.equal(back[k], st[k]) for k in st)
    bad = dict(back)
    del bad["model.layers.0.mlp.up_proj.weight"]
    with pytest.raises(KeyError, match="up_proj"):
        W.check_checkpoint(bad, shape)
    bad = dict(back)
    bad["model.norm.weight"] = torch.ones(255, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="model.norm.weight"):
        W.check_checkpoint(bad, shape)
