"""Tensor-parallel partition of the Llama-3-8B block, checked on the CPU with two
gloo ranks: each rank runs the block on its shard (oracle ops on the dequantized
shard weights, rank 0 adding the residuals), the two all-reduces sum the partials,
and the result must match the oracle block on the full weights. The same
partition functions feed the GPU block (iron_b200/applications/llama3_8b)."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import llama as ollama
from oracle import ops, quant

from iron_b200.applications.llama3_8b.sharding import (BlockShape, interleave_gate_up, random_block_weights,
                                                       shard_of, shard_weights)

SHAPE = BlockShape(hidden=256, n_heads=4, n_kv=2, head_dim=64, ffn=512)


def _deq(codes, scales):
    bits = quant.dequant_s4g32(codes.numpy(), scales.view(torch.uint16).numpy())
    return torch.from_numpy(bits.astype(np.uint16).view(np.int16)).view(torch.bfloat16)


def _full_oracle_weights(W):
    return {"n1": W["n1"], "n2": W["n2"], **{k: _deq(*W[k]) for k in ("q", "k", "v", "o", "g", "u", "d")}}


def _inputs(B, L, seed=3):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, SHAPE.hidden, generator=g).to(torch.bfloat16)
    kc = torch.randn(B, SHAPE.n_kv, L, SHAPE.head_dim, generator=g).to(torch.bfloat16)
    vc = torch.randn(B, SHAPE.n_kv, L, SHAPE.head_dim, generator=g).to(torch.bfloat16)
    return x, kc, vc


def _rank_block(rank, tp, x, kc, vc, pos, angles, W):
    """One rank's share of the block, composed like TPDecoderBlock._launch."""
    sh = shard_of(SHAPE, tp, rank)
    S = shard_weights(W, SHAPE, sh)
    hd, E = SHAPE.head_dim, SHAPE.hidden
    hq, hk = sh.h1 - sh.h0, sh.k1 - sh.k0
    B = x.shape[0]
    qkv = _deq(*S["qkv"])
    xn = ops.rms_norm(x, S["n1"], SHAPE.eps)
    y = ops.gemv_multi(qkv, xn)
    q = y[:, : hq * hd].reshape(B, hq, hd)
    k = y[:, hq * hd : (hq + hk) * hd].reshape(B, hk, hd)
    v = y[:, (hq + hk) * hd :].reshape(B, hk, hd)
    kcl, vcl = kc[:, sh.k0 : sh.k1].clone(), vc[:, sh.k0 : sh.k1].clone()
    lens = []
    for b in range(B):
        p = int(pos[b])
        q[b] = ops.rope(q[b], angles[p : p + 1])
        kcl[b, :, p] = ops.rope(k[b], angles[p : p + 1])
        vcl[b, :, p] = v[b]
        lens.append(p + 1)
    att = ops.attn_decode(q, kcl, vcl, lens).reshape(B, hq * hd)
    o = ops.gemv_multi(_deq(*S["o"]), att)
    h = ops.add(x, o) if rank == 0 else o
    h32 = h.float()
    if tp > 1:
        dist.all_reduce(h32)
    h = h32.to(torch.bfloat16)
    hn = ops.rms_norm(h, S["n2"], SHAPE.eps)
    gu = ops.gemv_multi(_deq(*S["gu"]), hn).reshape(B, -1, 16)
    act = ops.swiglu_act(gu[:, :, :8].reshape(B, -1), gu[:, :, 8:].reshape(B, -1))
    d = ops.gemv_multi(_deq(*S["d"]), act)
    out = (ops.add(h, d) if rank == 0 else d).float()
    if tp > 1:
        dist.all_reduce(out)
    return out.to(torch.bfloat16), kcl, vcl


def _worker(rank, tp, port, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=tp)
    try:
        W = random_block_weights(SHAPE, seed=21, device="cpu")
        x, kc, vc = _inputs(2, 32)
        pos = [5, 17]
        angles = ops.rope_angles(SHAPE.head_dim, 32, SHAPE.rope_base)
        out, kcl, vcl = _rank_block(rank, tp, x, kc, vc, pos, angles, W)
        result_q.put((rank, out, kcl, vcl))
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def test_shard_of_partitions_heads_and_ffn():
    shape = BlockShape()
    for tp in (1, 2, 4, 8):
        shards = [shard_of(shape, tp, r) for r in range(tp)]
        assert shards[0].h0 == 0 and shards[-1].h1 == 32 and shards[-1].k1 == 8 and shards[-1].f1 == 14336
        for a, b in zip(shards, shards[1:]):
            assert a.h1 == b.h0 and a.k1 == b.k0 and a.f1 == b.f0
        assert all((s.h1 - s.h0) == 4 * (s.k1 - s.k0) for s in shards)  # GQA groups stay whole
    with pytest.raises(ValueError):
        shard_of(shape, 3, 0)


def test_interleave_gate_up():
    g = torch.arange(16).reshape(16, 1)
    u = 100 + torch.arange(16).reshape(16, 1)
    r = interleave_gate_up(g, u).reshape(-1).tolist()
    assert r[:16] == list(range(8)) + [100 + i for i in range(8)]
    assert r[16:] == list(range(8, 16)) + [108 + i for i in range(8)]


def test_tp2_gloo_matches_full_block():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(2):
        rank, out, kcl, vcl = q.get(timeout=120)
        results[rank] = (out, kcl, vcl)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    W = random_block_weights(SHAPE, seed=21, device="cpu")
    x, kc, vc = _inputs(2, 32)
    pos = [5, 17]
    angles = ops.rope_angles(SHAPE.head_dim, 32, SHAPE.rope_base)
    ref = ollama.block_decode(x, kc, vc, pos, _full_oracle_weights(W), angles, SHAPE.n_heads, SHAPE.n_kv,
                              SHAPE.head_dim, SHAPE.eps)
    from helpers import assert_close

    assert torch.equal(results[0][0], results[1][0])  # both ranks hold the same block output
    assert_close(results[0][0], ref, 2e-2, 2e-2, what="tp2 block")
    # each rank's cache shard got its kv heads' new rows
    assert torch.equal(torch.cat([results[0][1], results[1][1]], dim=1), kc)
    assert torch.equal(torch.cat([results[0][2], results[1][2]], dim=1), vc)
