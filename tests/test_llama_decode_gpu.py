"""The fused int4 Llama decode step on the B200 vs the oracle's composition of
IRON's golden block (iron/applications/llama_3.2_1b/llama_cpu.py:170-285) on the
exactly dequantized weights. Reduced depth/vocab keeps the CPU oracle fast; every
kernel runs at the real Llama-3.2-1B layer shapes."""

import pytest
import torch

from helpers import assert_close, conditioned_rows
from oracle import llama as ollama

pytestmark = pytest.mark.gpu

from iron_b200.applications.llama_3_2_1b.decode import LlamaDecodeEngine, LlamaShape


def _oracle_weights(eng):
    s = eng.s
    H, E = s.hidden_dim, s.emb_dim
    out = []
    for lay in eng.layers:
        qkv = lay["qkv"].dequant().cpu()
        gu = lay["gu"].dequant().cpu().reshape(-1, 16, E)
        q_rows, kv_rows = s.n_heads * s.head_dim, s.n_kv_groups * s.head_dim
        out.append({
            "n1": lay["n1"].cpu(), "n2": lay["n2"].cpu(),
            "q": qkv[:q_rows], "k": qkv[q_rows:q_rows + kv_rows], "v": qkv[q_rows + kv_rows:],
            "o": lay["o"].dequant().cpu(),
            "g": gu[:, :8].reshape(H, E), "u": gu[:, 8:].reshape(H, E),
            "d": lay["d"].dequant().cpu(),
        })
    return out


@pytest.mark.parametrize("fuse", [None, ("layers", True), ("none", False)])
@pytest.mark.parametrize("batch,prefix", [(1, [9]), (2, [63, 65]), (3, [0, 5, 40]),
                                          (8, [1, 2, 3, 63, 64, 65, 100, 127]),
                                          (12, [0, 1, 2, 3, 5, 8, 13, 21, 34, 55, 89, 144])])
def test_decode_step_matches_oracle(batch, prefix, fuse):
    if fuse and fuse[0] != "none" and batch > 8:
        pytest.skip("the fused RMSNorm prologue serves batch <= 8")
    shape = LlamaShape(n_layers=2, vocab_size=4096)
    L = 160
    kw = dict(fuse_norm=fuse[0], fuse_rope=fuse[1]) if fuse else {}
    eng = LlamaDecodeEngine(shape, batch, L, seed=7, keep_natural=True, **kw)
    g = torch.Generator(device="cuda").manual_seed(1)
    eng.kc.copy_(torch.randn(eng.kc.shape, generator=g, device="cuda").to(torch.bfloat16))
    eng.vc.copy_(torch.randn(eng.vc.shape, generator=g, device="cuda").to(torch.bfloat16))
    toks = [(31 * i + 3) % shape.vocab_size for i in range(batch)]
    eng.set_state(toks, prefix)
    kc0, vc0 = eng.kc.cpu(), eng.vc.cpu()
    eng.step()
    torch.cuda.synchronize()
    eng.check_status()
    W = _oracle_weights(eng)
    kcs = [kc0[i].clone() for i in range(shape.n_layers)]
    vcs = [vc0[i].clone() for i in range(shape.n_layers)]
    lm_cpu = eng.lm.dequant().cpu()

    # the chained engine folds the RMSNorms into its GEMVs: the oracle at the same rounding
    # points (oracle.llama._normed_gemv); IRON's own order is checked by the KL bound below
    fold = eng.fuse_norm == "chain"

    def oracle_step(kc_out=None, vc_out=None, hidden=None, fold_=fold):
        kk = [k.clone() for k in kcs] if kc_out is None else kc_out
        vv = [v.clone() for v in vcs] if vc_out is None else vc_out
        return ollama.model_decode(toks, prefix, W, eng.nf.cpu(), eng.embed_table.cpu(), lm_cpu, kk, vv,
                                   eng.lut.cpu(), shape.n_heads, shape.n_kv_groups, shape.head_dim, fold=fold_,
                                   hidden=hidden)

    logits, well = conditioned_rows(oracle_step, 2e-2, 1e-2)
    hid = []
    oracle_step(kcs, vcs, hidden=hid)  # the oracle's appended cache rows, for the row checks below
    # a sequence whose residual stream ends as a near-cancellation of far larger terms
    # (final RMS < 5 % of the batch's median final RMS: the blocks' outputs have the same
    # scale for every sequence, so a much smaller sum is a cancellation) turns one-ulp
    # differences of those terms into errors of its own size: not held to the elementwise bar
    rms = torch.stack([h.float().pow(2).mean(-1).sqrt() for h in hid])
    well = well & (rms[-1] > 0.05 * rms[-1].median())
    # 1. The last layer's attention and the lm-head recomputed by the oracle on the
    # engine's OWN inputs (its QKV projection and caches; its final hidden state): every
    # output within the north star's bar, no exceptions -- the kernels' parity, free of
    # the chain's amplification.
    from oracle import ops
    Hq, Hd = shape.n_heads, shape.head_dim
    lut = eng.lut.cpu()
    q_raw = eng.qkv.cpu()[:, :Hq * Hd].reshape(batch, Hq, Hd)
    q_rot = torch.stack([ops.rope(q_raw[b], lut[p:p + 1]) for b, p in enumerate(prefix)])
    att = ops.attn_decode(q_rot, eng.kc[-1].cpu(), eng.vc[-1].cpu(), [p + 1 for p in prefix])
    assert_close(eng.attn.cpu().reshape(batch, Hq, Hd), att, 2e-2, 1e-2, what="attention on the engine's inputs")
    lm = eng.lm.dequant().cpu()
    head = ops.gemv_multi(lm, ops.rms_norm(eng.x.cpu(), eng.nf.cpu(), shape.eps))
    assert_close(eng.logits.cpu(), head, 2e-2, 1e-2, what="lm-head on the engine's hidden state")
    # 2. End to end against the oracle's own chain, for every sequence whose oracle result
    # is stable under fp64 sums (helpers.conditioned_rows) and whose residual stream does
    # not cancel: every logit within the bar. The others (measured on B200 at batch 8:
    # position 63, whose hidden state after layer 1 nearly cancels -- RMS 0.25 against ~40
    # for the others -- and whose logits then move by up to 0.2 between correct
    # implementations) are held to the distribution check only: IRON's own app-level bound
    # is a KL bound (iron/applications/llama_3.2_1b/test.py:77-113).
    d = (eng.logits.cpu().float() - logits.float()).abs()
    bad = d >= torch.maximum(torch.full_like(d, 1e-2), 2e-2 * (eng.logits.cpu().float().abs() + logits.float().abs()))
    print(f"batch {batch} {fuse}: per sequence (pos, well-conditioned, outside 2e-2 / 1e-2, max |diff|): "
          f"{[(p, bool(well[b]), int(bad[b].sum()), round(float(d[b].max()), 4)) for b, p in enumerate(prefix)]}; "
          f"final RMS {[round(float(r), 3) for r in rms[-1]]}")
    assert int(well.sum()) >= (batch + 1) // 2, "most sequences must be well-conditioned"
    assert_close(eng.logits.cpu()[well], logits[well], 2e-2, 1e-2, what="logits (well-conditioned sequences)")
    lp = torch.log_softmax(logits.float(), -1)
    kl = (lp.exp() * (lp - torch.log_softmax(eng.logits.cpu().float(), -1))).sum(-1)
    assert float(kl[well].max()) < 1e-3, kl
    assert float(kl.max()) <= 0.05, kl
    if fold:  # and the distributions against IRON's operator order (rms_norm, then the GEMV)
        iron_order = oracle_step(fold_=False)
        lp = torch.log_softmax(iron_order.float(), -1)
        kl2 = (lp.exp() * (lp - torch.log_softmax(eng.logits.cpu().float(), -1))).sum(-1)
        assert float(kl2[well].max()) < 1e-3, kl2
    # caches got the new rows, positions advanced, greedy token consistent
    # (layer 0's rows for every sequence; deeper rows for the well-conditioned ones)
    for li in range(shape.n_layers):
        for b, p in enumerate(prefix):
            if li > 0 and not bool(well[b]):
                continue
            assert_close(eng.kc[li, b, :, p].cpu(), kcs[li][b, :, p], 2e-2, 2e-2, max_mismatch_frac=1e-2,
                         what="k row")
            assert_close(eng.vc[li, b, :, p].cpu(), vcs[li][b, :, p], 2e-2, 2e-2, max_mismatch_frac=1e-2,
                         what="v row")
    assert eng.pos.cpu().tolist() == [p + 1 for p in prefix]
    top = eng.tokens.cpu().long()
    got = eng.logits.cpu().float()
    assert torch.all(got.gather(1, top[:, None])[:, 0] == got.max(1).values)


def test_graph_replay_matches_eager_steps():
    shape = LlamaShape(n_layers=2, vocab_size=4096)
    runs = []
    for use_graph in (False, True):
        eng = LlamaDecodeEngine(shape, 2, 64, seed=3)
        eng.set_state([11, 12], [4, 9])
        if use_graph:
            eng.capture()
        outs = []
        for _ in range(5):
            eng.step()
            outs.append((eng.tokens.clone(), eng.logits.clone()))
        torch.cuda.synchronize()
        runs.append(outs)
    for (ta, la), (tb, lb) in zip(*runs):
        assert torch.equal(ta, tb) and torch.equal(la, lb)


def test_host_io_graph_matches_device_steps():
    """capture_host_io / step_host: the step's graph with the token ids copied in from and
    out to pinned host memory (the host feeding each read token back) gives bitwise the
    tokens and logits of the device-state graph."""
    shape = LlamaShape(n_layers=2, vocab_size=4096)
    runs = []
    for host in (False, True):
        eng = LlamaDecodeEngine(shape, 2, 64, seed=3)
        eng.set_state([11, 12], [4, 9])
        eng.capture()
        eng.capture_host_io()
        outs = []
        for _ in range(4):
            if host:
                eng.step_host()
                torch.cuda.synchronize()
                toks = eng.host_tokens_out.clone()
                eng.host_tokens_in.copy_(toks)
            else:
                eng.step()
                torch.cuda.synchronize()
                toks = eng.tokens.cpu()
            outs.append((toks, eng.logits.cpu()))
        assert eng.pos.cpu().tolist() == [8, 13]
        runs.append(outs)
    for (ta, la), (tb, lb) in zip(*runs):
        assert torch.equal(ta, tb) and torch.equal(la, lb)


@pytest.mark.parametrize("S", [100, 192])
def test_prefill_matches_oracle_then_decodes(S):
    """Prompt through the tensor-core prefill (int4 weights unpacked to bf16, tcgen05
    GEMMs with fused residual / SwiGLU epilogues, causal prefill attention), then one
    decode step, against the oracle's prefill + decode on the dequantized weights."""
    shape = LlamaShape(n_layers=2, vocab_size=4096)
    L = 256
    eng = LlamaDecodeEngine(shape, 2, L, seed=11, keep_natural=True)
    toks = [(13 * i + 5) % shape.vocab_size for i in range(S)]
    eng.set_state([0, 0], [0, 0])
    eng.prefill(toks, seq=1)
    torch.cuda.synchronize()
    W = _oracle_weights(eng)
    kcs = [torch.zeros(shape.n_kv_groups, L, shape.head_dim, dtype=torch.bfloat16) for _ in range(shape.n_layers)]
    vcs = [torch.zeros_like(k) for k in kcs]
    lm = eng.lm.dequant().cpu()
    logits = ollama.model_prefill(toks, W, eng.nf.cpu(), eng.embed_table.cpu(), lm, kcs, vcs, eng.lut.cpu(),
                                  shape.n_heads, shape.n_kv_groups, shape.head_dim)
    assert_close(eng.logits[1:2].cpu(), logits, 2e-2, 2e-2, what="prefill logits")
    for li in range(shape.n_layers):
        assert_close(eng.kc[li, 1, :, :S].cpu(), kcs[li][:, :S], 2e-2, 2e-2, max_mismatch_frac=1e-3, what="k")
        assert_close(eng.vc[li, 1, :, :S].cpu(), vcs[li][:, :S], 2e-2, 2e-2, max_mismatch_frac=1e-3, what="v")
    assert int(eng.pos[1]) == S
    nxt = int(eng.tokens[1])
    got = eng.logits[1].cpu().float()
    assert got[nxt] == got.max()
    # one decode step continues the sequence from position S
    eng.step()
    torch.cuda.synchronize()
    kcs2 = [torch.stack([torch.zeros_like(k), k]) for k in kcs]
    vcs2 = [torch.stack([torch.zeros_like(v), v]) for v in vcs]
    lg2 = ollama.model_decode([0, nxt], [0, S], W, eng.nf.cpu(), eng.embed_table.cpu(), lm, kcs2, vcs2,
                              eng.lut.cpu(), shape.n_heads, shape.n_kv_groups, shape.head_dim)
    assert_close(eng.logits[1:2].cpu(), lg2[1:2], 3e-2, 3e-2, what="decode after prefill")


@pytest.mark.parametrize("n_vec", [1, 3, 8])
def test_gemv_ex_fused_rmsnorm_and_argmax(n_vec):
    """iron_gemv_int4g32_ex: RMSNorm of x fused into the GEMV's prologue and the greedy
    argmax into its epilogue, against the oracle's rms_norm -> gemv -> argmax."""
    from iron_b200 import _lib
    from iron_b200.applications.llama_3_2_1b.decode import Int4Matrix
    from oracle import ops

    N, K = 4096, 2048
    g = torch.Generator(device="cuda").manual_seed(n_vec)
    W = Int4Matrix(N, K, g, 0.001, 0.004, keep_natural=True)
    x = torch.randn(n_vec, K, device="cuda", generator=g).to(torch.bfloat16)
    w = (1 + 0.02 * torch.randn(K, device="cuda", generator=g)).to(torch.bfloat16)
    y = torch.empty(n_vec, N, dtype=torch.bfloat16, device="cuda")
    keys = torch.zeros(n_vec * 32, dtype=torch.int64, device="cuda")
    tok = torch.zeros(n_vec, dtype=torch.int32, device="cuda")
    s = _lib.current_stream()
    _lib.call("iron_gemv_int4g32_ex", W.packed.data_ptr(), x.data_ptr(), y.data_ptr(), N, K, n_vec, None,
              w.data_ptr(), 1e-5, keys.data_ptr(), 0, s)
    _lib.call("iron_argmax_finalize", keys.data_ptr(), tok.data_ptr(), None, n_vec, 0, s)
    torch.cuda.synchronize()
    ref = ops.gemv_multi(W.dequant().cpu(), ops.rms_norm(x.cpu(), w.cpu(), 1e-5))
    assert_close(y.cpu(), ref, 2e-2, 1e-2, what="normed gemv")
    got = y.cpu().float()
    assert torch.equal(tok.cpu().long(), got.argmax(1))  # first index of the max of what it wrote
    assert int(keys.abs().sum()) == 0  # keys reset for the next step


def test_l2_prefetch_option_leaves_results_unchanged():
    """The side-branch L2 prefetch (an option, off by default) changes no result: the
    same tokens and logits over three graph-replayed steps."""
    shape = LlamaShape(n_layers=2, vocab_size=4096)
    runs = []
    for pf in (False, True):
        eng = LlamaDecodeEngine(shape, 2, 64, seed=3, l2_prefetch=pf)
        eng.set_state([11, 12], [4, 9])
        eng.capture()
        outs = []
        for _ in range(3):
            eng.step()
            outs.append((eng.tokens.clone(), eng.logits.clone()))
        torch.cuda.synchronize()
        runs.append(outs)
    for (ta, la), (tb, lb) in zip(*runs):
        assert torch.equal(ta, tb) and torch.equal(la, lb)
