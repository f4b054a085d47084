"""Prefill (causal GQA) attention on the B200 against the oracle.

IRON's MHA shapes and tolerance (iron/operators/mha/test.py:13-80: relative 0.04,
absolute 0.15, 0.5% mismatches allowed, inputs ~ 4 U[0,1)), the goldens it
generates, and the strided token-major layout the Llama prefill uses.
"""

import ctypes
import math

import numpy as np
import pytest
import torch

from helpers import assert_close, bf16, load
from oracle import ops

pytestmark = pytest.mark.gpu

from iron_b200 import _lib
from iron_b200.common.test_utils import run_test
from iron_b200.common.verify import Tolerance
from iron_b200.operators import MHA

TOL = Tolerance.relative(4.0e-2, 1.5e-1, max_mismatch_frac=0.005)


def _golden(S, H, Hkv, pipelines=1, seed=42):
    g = torch.Generator().manual_seed(seed)
    Q = (torch.rand(H, S, 64, generator=g) * 4).to(torch.bfloat16)
    K = (torch.rand(Hkv, S, 64, generator=g) * 4).to(torch.bfloat16)
    V = (torch.rand(Hkv, S, 64, generator=g) * 4).to(torch.bfloat16)
    O = ops.mha_prefill(Q, K, V)
    pad = ((S + 63 * pipelines) // (64 * pipelines)) * (64 * pipelines)

    def p(t):
        return torch.nn.functional.pad(t, (0, 0, 0, pad - S))

    return p(Q), p(K), p(V), p(O)


@pytest.mark.parametrize("S,H,pipes,kv", [(16384, 1, 8, 0), (8192, 8, 8, 2), (16384, 1, 4, 0), (1000, 4, 1, 2),
                                          (130, 6, 1, 3)])
def test_mha(S, H, pipes, kv):
    Q, K, V, O = _golden(S, H, kv if kv else H, pipes)
    op = MHA(num_heads=H, seq_len=S, d=64, num_KV_heads=kv, num_of_pipelines=pipes)
    errors, _, _ = run_test(op, {"Q": Q.flatten(), "K": K.flatten(), "V": V.flatten()}, {"O": O.flatten()},
                            tolerance=TOL)
    assert not errors


@pytest.mark.parametrize("name,S,H,kv", [("mha_h2_kv1_s128", 128, 2, 1), ("mha_h4_kv2_s100", 100, 4, 2)])
def test_mha_golden_fixtures(name, S, H, kv):
    d = {k: bf16(v) for k, v in load(name).items()}
    op = MHA(num_heads=H, seq_len=S, d=64, num_KV_heads=kv)
    errors, _, _ = run_test(op, {"Q": d["Q"].flatten(), "K": d["K"].flatten(), "V": d["V"].flatten()},
                            {"O": d["O"].flatten()}, tolerance=TOL)
    assert not errors


def test_mha_arg_spec_matches_design_shapes():
    for S, H, pipes, kv in [(16384, 8, 8, 2), (16384, 1, 8, 0)]:
        op = MHA(num_heads=H, seq_len=S, d=64, num_KV_heads=kv, num_of_pipelines=pipes)
        q, k, v, o = (s.shape[0] for s in op.get_arg_spec())
        pad = op._calculate_seq_padding(S, pipes)
        assert q == o == H * pad * 64 and k == v == (kv or H) * pad * 64


def _strided_call(q, k, v, out, B, H, Hkv, S, S_pad, qs, kvs, os_, causal=1):
    arr = lambda t: (ctypes.c_int64 * 3)(*t)  # noqa: E731
    _lib.call("iron_attn_prefill", q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), B, H, Hkv, 64, S,
              S_pad, S, arr(qs), arr(kvs), arr(os_), 0.125, causal, 0, _lib.current_stream())
    torch.cuda.synchronize()


def test_llama_prefill_layout():
    """Q read straight from the fused QKV projection ([S, (32 + 2*8) * 64], token-major),
    K / V from a [kv_head, L, 64] cache, O written token-major [S, 32 * 64]."""
    S, H, Hkv, L = 2048, 32, 8, 4096
    g = torch.Generator().manual_seed(3)
    qkv = torch.randn(S, (H + 2 * Hkv) * 64, generator=g).to(torch.bfloat16)
    kc = torch.zeros(Hkv, L, 64, dtype=torch.bfloat16)
    vc = torch.zeros(Hkv, L, 64, dtype=torch.bfloat16)
    kc[:, :S] = torch.randn(Hkv, S, 64, generator=g).to(torch.bfloat16)
    vc[:, :S] = torch.randn(Hkv, S, 64, generator=g).to(torch.bfloat16)
    qd, kd, vd = qkv.cuda(), kc.cuda(), vc.cuda()
    out = torch.full((S, H * 64), float("nan"), dtype=torch.bfloat16, device="cuda")
    _strided_call(qd, kd, vd, out, 1, H, Hkv, S, S, (0, 64, (H + 2 * Hkv) * 64), (0, L * 64, 64), (0, 64, H * 64))
    Q = qkv[:, : H * 64].reshape(S, H, 64).transpose(0, 1).contiguous()
    ref = ops.mha_prefill(Q, kc[:, :S], vc[:, :S]).transpose(0, 1).reshape(S, H * 64)
    assert_close(out.cpu(), ref, 0.04, 0.02, max_mismatch_frac=1e-4)


def test_non_causal_and_batched():
    B, H, Hkv, S = 2, 4, 2, 96
    g = torch.Generator().manual_seed(9)
    q = torch.randn(B, H, 128, 64, generator=g).to(torch.bfloat16)
    k = torch.randn(B, Hkv, S, 64, generator=g).to(torch.bfloat16)
    v = torch.randn(B, Hkv, S, 64, generator=g).to(torch.bfloat16)
    out = torch.full((B, H, 128, 64), float("nan"), dtype=torch.bfloat16, device="cuda")
    _strided_call(q.cuda(), k.cuda(), v.cuda(), out, B, H, Hkv, S, 128, (H * 128 * 64, 128 * 64, 64),
                  (Hkv * S * 64, S * 64, 64), (H * 128 * 64, 128 * 64, 64), causal=0)
    got = out.cpu()
    for b in range(B):
        ref = ops.mha_prefill(q[b, :, :S], k[b], v[b], causal=False)
        assert_close(got[b, :, :S], ref, 0.04, 0.02)
        assert torch.all(got[b, :, S:] == 0)
