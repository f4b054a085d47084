"""BASELINE config 3 on the B200: one Llama-3.2-1B decoder block at decode with bf16
weights, batch 1 and 16, positions drawn from 0..4095 -- the operator chain (RMSNorm
-> QKV GEMV -> RoPE -> KV append -> SwiGLU MLP) and the full block -- against the
oracle's restatement of IRON's golden block (llama_cpu.py:170-207). rtol 2e-2 /
atol 1e-2 on every output (the full block's residual sum with a mismatch allowance of
1e-3 and a 1 % error norm); the appended K/V rows are checked in place."""

import pytest
import torch

from helpers import assert_close
from oracle import llama as ollama

pytestmark = pytest.mark.gpu

from iron_b200.applications.llama_3_2_1b.block_bf16 import DecoderBlockBF16


def _oracle_weights(blk):
    s = blk.s
    qr, kvr = s.n_heads * s.head_dim, s.n_kv_groups * s.head_dim
    W = {k: v.cpu() for k, v in blk.W.items() if k != "qkv"}
    qkv = blk.W["qkv"].cpu()
    W.update(q=qkv[:qr], k=qkv[qr:qr + kvr], v=qkv[qr + kvr:])
    return W


def _setup(B, full, seed):
    blk = DecoderBlockBF16(batch=B, max_seq=4096, seed=seed, full=full)
    g = torch.Generator(device="cuda").manual_seed(seed + 1)
    blk.x.copy_(torch.randn(blk.x.shape, device="cuda", generator=g).to(torch.bfloat16))
    blk.kc.copy_(torch.randn(blk.kc.shape, device="cuda", generator=g).to(torch.bfloat16))
    blk.vc.copy_(torch.randn(blk.vc.shape, device="cuda", generator=g).to(torch.bfloat16))
    cg = torch.Generator().manual_seed(seed + 2)
    pos = torch.randint(0, 4096, (B,), generator=cg, dtype=torch.int32)
    pos[0] = 4095  # the last slot
    if B > 1:
        pos[1] = 0  # an empty prefix
    blk.pos.copy_(pos)
    return blk, pos.tolist()


@pytest.mark.parametrize("B", [1, 16])
def test_config3_chain_matches_oracle(B):
    blk, pos = _setup(B, full=False, seed=21)
    x0, kc0, vc0 = blk.x.cpu(), blk.kc.cpu(), blk.vc.cpu()
    blk.step()
    torch.cuda.synchronize()
    s = blk.s
    q, mlp = ollama.block_mlp_half(x0, kc0, vc0, pos, _oracle_weights(blk), blk.lut.cpu(), s.n_heads,
                                   s.n_kv_groups, s.head_dim, s.eps)
    assert_close(blk.q.cpu(), q, 2e-2, 1e-2, what="roped q")
    assert_close(blk.out.cpu(), mlp, 2e-2, 1e-2, what="SwiGLU MLP output")
    assert blk.lens.cpu().tolist() == [p + 1 for p in pos]
    for b, p in enumerate(pos):
        assert_close(blk.kc[b, :, p].cpu(), kc0[b, :, p], 2e-2, 1e-2, what="appended k row")
        assert_close(blk.vc[b, :, p].cpu(), vc0[b, :, p], 2e-2, 1e-2, what="appended v row")
    # every other cache row untouched (bit-exact)
    kc1, vc1 = blk.kc.cpu(), blk.vc.cpu()
    for b, p in enumerate(pos):
        kc1[b, :, p] = kc0[b, :, p]
        vc1[b, :, p] = vc0[b, :, p]
    assert torch.equal(kc1.view(torch.int16), kc0.view(torch.int16))
    assert torch.equal(vc1.view(torch.int16), vc0.view(torch.int16))


@pytest.mark.parametrize("B", [1, 16])
def test_full_block_matches_oracle(B):
    blk, pos = _setup(B, full=True, seed=33)
    x0, kc0, vc0 = blk.x.cpu(), blk.kc.cpu(), blk.vc.cpu()
    blk.step()
    torch.cuda.synchronize()
    s = blk.s
    ref = ollama.block_decode(x0, kc0, vc0, pos, _oracle_weights(blk), blk.lut.cpu(), s.n_heads, s.n_kv_groups,
                              s.head_dim, s.eps)
    # the block output is h + mlp(h) with |h| ~ 1: where the two terms cancel, a 1-ulp
    # difference of a bf16 intermediate (GEMV reduction order) exceeds atol, so a few
    # such points in 1e3 are allowed, and the whole output is held to a 1 % error norm
    assert_close(blk.out.cpu(), ref, 2e-2, 1e-2, max_mismatch_frac=1e-3, what="block output")
    err = (blk.out.cpu().float() - ref.float()).norm() / ref.float().norm()
    assert err < 1e-2, f"relative error norm {err:.3e}"
    for b, p in enumerate(pos):
        assert_close(blk.kc[b, :, p].cpu(), kc0[b, :, p], 2e-2, 1e-2, what="appended k row")
        assert_close(blk.vc[b, :, p].cpu(), vc0[b, :, p], 2e-2, 1e-2, what="appended v row")


def test_graph_replay_is_bitwise_stable():
    """The captured step gives the eager step's outputs bit for bit, replay after replay."""
    blk, _ = _setup(16, full=True, seed=5)
    blk.step()
    torch.cuda.synchronize()
    eager = blk.out.clone()
    blk.capture()
    for _ in range(3):
        blk.step()
    torch.cuda.synchronize()
    assert torch.equal(blk.out.view(torch.int16), eager.view(torch.int16))
