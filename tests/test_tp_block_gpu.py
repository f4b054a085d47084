"""Llama-3-8B block decode (head_dim 128) on the B200: tp = 1 against the oracle's
block on the dequantized weights, and tp = 2 / 4 / 8 (NCCL all-reduce) against
tp = 1 on the same weights when the box has that many GPUs."""

import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from helpers import assert_close
from oracle import llama as ollama
from oracle import ops, quant

pytestmark = pytest.mark.gpu

from iron_b200.applications.llama3_8b.sharding import BlockShape
from iron_b200.applications.llama3_8b.tp_block import TPDecoderBlock

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _deq(codes, scales):
    bits = quant.dequant_s4g32(codes.cpu().numpy(), scales.cpu().view(torch.uint16).numpy())
    return torch.from_numpy(bits.astype(np.uint16).view(np.int16)).view(torch.bfloat16)


def test_block_tp1_matches_oracle():
    shape, B, L = BlockShape(), 2, 64
    blk = TPDecoderBlock(shape, 1, 0, B, L, seed=13, keep_full=True)
    g = torch.Generator(device="cuda").manual_seed(5)
    blk.x.copy_(torch.randn(B, shape.hidden, device="cuda", generator=g).to(torch.bfloat16))
    blk.kc.copy_(torch.randn(blk.kc.shape, device="cuda", generator=g).to(torch.bfloat16))
    blk.vc.copy_(torch.randn(blk.vc.shape, device="cuda", generator=g).to(torch.bfloat16))
    pos = [5, 40]
    blk.pos.copy_(torch.tensor(pos, dtype=torch.int32))
    x0, kc0, vc0 = blk.x.cpu(), blk.kc.cpu(), blk.vc.cpu()
    blk.step()
    torch.cuda.synchronize()
    W = {"n1": blk.full["n1"].cpu(), "n2": blk.full["n2"].cpu(),
         **{k: _deq(*blk.full[k]) for k in ("q", "k", "v", "o", "g", "u", "d")}}
    angles = blk.lut.cpu()
    ref = ollama.block_decode(x0, kc0, vc0, pos, W, angles, shape.n_heads, shape.n_kv, shape.head_dim, shape.eps)
    assert_close(blk.x.cpu(), ref, 2e-2, 2e-2, what="block output")
    for b, p in enumerate(pos):
        assert_close(blk.kc[b, :, p].cpu(), kc0[b, :, p], 2e-2, 2e-2, what="k row")
        assert_close(blk.vc[b, :, p].cpu(), vc0[b, :, p], 2e-2, 2e-2, what="v row")


def test_attention_head_dim_128_ragged():
    from iron_b200 import _lib

    B, Hq, Hkv, D, L = 3, 8, 2, 128, 3000
    g = torch.Generator().manual_seed(2)
    q = torch.randn(B, Hq, D, generator=g).to(torch.bfloat16)
    k = torch.randn(B, Hkv, L, D, generator=g).to(torch.bfloat16)
    v = torch.randn(B, Hkv, L, D, generator=g).to(torch.bfloat16)
    lens = torch.tensor([1, 1777, 3000], dtype=torch.int32)
    out = torch.empty(B, Hq, D, dtype=torch.bfloat16, device="cuda")
    wsb = _lib.load().iron_attn_decode_workspace_bytes_d(B, Hq, Hkv, L, D)
    ws = torch.zeros(max(wsb, 16), dtype=torch.uint8, device="cuda")
    qd, kd, vd, ld = q.cuda(), k.cuda(), v.cuda(), lens.cuda()
    _lib.call("iron_attn_decode", qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), ld.data_ptr(), out.data_ptr(), B,
              Hq, Hkv, D, L, Hkv * L * D, L * D, 1 / np.sqrt(D), ws.data_ptr(), ws.numel(), 0,
              _lib.current_stream())
    torch.cuda.synchronize()
    assert_close(out.cpu(), ops.attn_decode(q, k, v, lens.tolist()), 2e-2, 1e-2)


def _block_inputs(blk, x0, kc, vc, pos):
    blk.kc.copy_(kc[:, blk.sh.k0:blk.sh.k1])
    blk.vc.copy_(vc[:, blk.sh.k0:blk.sh.k1])
    blk.x.copy_(x0)
    blk.pos.copy_(pos)


@pytest.mark.parametrize("tp", [2, 4, 8])
def test_block_tp_emulated_on_one_gpu(tp):
    """Every rank's shard run on one GPU, the two all-reduces done by torch between
    the halves (fp32 sum of the bf16 partials, rounded once): the sharded kernels
    (QKV / gate-up rows, o / down columns, local heads and kv heads) against tp = 1."""
    shape, B, L = BlockShape(), 2, 64
    g = torch.Generator(device="cuda").manual_seed(5)
    x0 = torch.randn(B, shape.hidden, device="cuda", generator=g).to(torch.bfloat16)
    kc = torch.randn(B, shape.n_kv, L, shape.head_dim, device="cuda", generator=g).to(torch.bfloat16)
    vc = torch.randn(B, shape.n_kv, L, shape.head_dim, device="cuda", generator=g).to(torch.bfloat16)
    pos = torch.tensor([5, 40], dtype=torch.int32, device="cuda")
    one = TPDecoderBlock(shape, 1, 0, B, L, seed=13)
    _block_inputs(one, x0, kc, vc, pos)
    one.step()
    blks = [TPDecoderBlock(shape, tp, r, B, L, seed=13) for r in range(tp)]
    stream = torch.cuda.current_stream().cuda_stream
    for b in blks:
        _block_inputs(b, x0, kc, vc, pos)
        b._attention_half(stream)
    h = torch.stack([b.h.float() for b in blks]).sum(0).to(torch.bfloat16)
    for b in blks:
        b.h.copy_(h)
        b._mlp_half(stream)
    out = torch.stack([b.x.float() for b in blks]).sum(0).to(torch.bfloat16)
    torch.cuda.synchronize()
    assert_close(out.cpu(), one.x.cpu(), 2e-2, 2e-2, what=f"tp={tp} block output")
    for b in blks:
        for bb, p in enumerate(pos.tolist()):
            assert_close(b.kc[bb, :, p].cpu(), one.kc[bb, b.sh.k0:b.sh.k1, p].cpu(), 2e-2, 2e-2, what="k row")
            assert_close(b.vc[bb, :, p].cpu(), one.vc[bb, b.sh.k0:b.sh.k1, p].cpu(), 2e-2, 2e-2, what="v row")


@pytest.mark.parametrize("tp", [2, 4, 8])
def test_block_tensor_parallel_matches_single_gpu(tp):
    if torch.cuda.device_count() < tp:
        pytest.skip(f"needs {tp} GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={tp}", "--master-addr=127.0.0.1", "--master-port=29617",
           os.path.join(REPO, "tests", "tp_block_worker.py")]
    r = subprocess.run(cmd, cwd=REPO, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
