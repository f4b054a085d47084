"""Split-KV GQA decode attention on the B200 vs the oracle (
32 q heads / 8 kv heads, d 64, bf16 cache ~ N(0,1), ragged lengths U[1, L_max],
batch 1/16/64, L_max 512/4096/32768; rtol 2e-2 / atol 1e-2)."""

import math

import numpy as np
import pytest
import torch

from helpers import assert_close
from oracle import ops

pytestmark = pytest.mark.gpu

from iron_b200 import _lib
from iron_b200.operators import DecodeAttention


def _case(B, L, seed, Hq=32, Hkv=8, D=64, lens=None):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(B, Hq, D, generator=g, device="cuda").to(torch.bfloat16)
    k = torch.randn(B, Hkv, L, D, generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn(B, Hkv, L, D, generator=g, device="cuda").to(torch.bfloat16)
    if lens is None:
        lens = torch.randint(1, L + 1, (B,), generator=g, device="cuda", dtype=torch.int32)
    else:
        lens = torch.tensor(lens, dtype=torch.int32, device="cuda")
    return q, k, v, lens


def _run(q, k, v, lens, Hq=32, Hkv=8):
    B, _, L, D = k.shape
    op = DecodeAttention(batch=B, num_heads=Hq, num_kv_heads=Hkv, head_dim=D, max_seq_len=L)
    out = torch.empty(B, Hq, D, dtype=torch.bfloat16, device="cuda")
    op.get_callable()(q, k, v, lens, out)
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize("B,L", [(1, 512), (16, 512), (64, 512), (1, 4096), (16, 4096), (64, 4096),
                                 (1, 32768), (16, 32768)])
def test_decode_attention_config4(B, L):
    q, k, v, lens = _case(B, L, seed=B * 7 + L)
    out = _run(q, k, v, lens)
    # verify every sequence (subsample for the largest shapes)
    idx = list(range(B)) if B * L <= 16 * 32768 else list(range(0, B, 7))
    exp = ops.attn_decode(q[idx].cpu(), k[idx].cpu(), v[idx].cpu(), lens[idx].cpu())
    assert_close(out[idx].cpu(), exp, 2e-2, 1e-2, what=f"attn B{B} L{L}")


def test_decode_attention_batch64_len32768_sampled():
    q, k, v, lens = _case(64, 32768, seed=3)
    out = _run(q, k, v, lens)
    idx = [0, 13, 31, 63]
    exp = ops.attn_decode(q[idx].cpu(), k[idx].cpu(), v[idx].cpu(), lens[idx].cpu())
    assert_close(out[idx].cpu(), exp, 2e-2, 1e-2, what="attn B64 L32768")


@pytest.mark.parametrize("lens", [[1, 2, 15, 16, 17, 63, 64, 65, 255, 256, 257, 511, 512]])
def test_decode_attention_edge_lengths(lens):
    B, L = len(lens), 512
    q, k, v, lt = _case(B, L, seed=11, lens=lens)
    out = _run(q, k, v, lt)
    exp = ops.attn_decode(q.cpu(), k.cpu(), v.cpu(), lt.cpu())
    assert_close(out.cpu(), exp, 2e-2, 1e-2, what="edge lengths")


@pytest.mark.parametrize("Hq,Hkv", [(32, 32), (8, 2), (16, 1), (12, 4)])
def test_decode_attention_group_sizes(Hq, Hkv):
    q, k, v, lens = _case(4, 1024, seed=Hq + Hkv, Hq=Hq, Hkv=Hkv)
    out = _run(q, k, v, lens, Hq=Hq, Hkv=Hkv)
    exp = ops.attn_decode(q.cpu(), k.cpu(), v.cpu(), lens.cpu())
    assert_close(out.cpu(), exp, 2e-2, 1e-2, what=f"group {Hq}/{Hkv}")


def test_decode_attention_deterministic_and_matches_sdpa():
    q, k, v, lens = _case(8, 4096, seed=5)
    a = _run(q, k, v, lens)
    b = _run(q, k, v, lens)
    assert torch.equal(a, b)
    # torch SDPA (fp32) on one sequence as an independent check
    n = int(lens[2])
    K = k[2, :, :n].float().repeat_interleave(4, 0)
    V = v[2, :, :n].float().repeat_interleave(4, 0)
    ref = torch.nn.functional.scaled_dot_product_attention(q[2].float()[:, None], K, V)[:, 0]
    assert_close(a[2].cpu(), ref.cpu().to(torch.bfloat16), 2e-2, 1e-2, what="sdpa")
