"""The benched decode configuration itself against the oracle: the full Llama-3.2-1B
shape (16 layers, vocab 128256, int4 group-32 weights), a synthetic KV cache at
context 2048, batch 1 and batch 64, several teacher-forced steps of the captured
decode graph -- the exact path `bench.py` times (16-CTA cluster attention with the
pre-wait L2 prefetch at batch 1, split attention at batch 64, the 128256-row lm-head
GEMV with the fused argmax).

Each step's logits are compared with `oracle.llama.model_decode` (IRON's CPU block,
iron/applications/llama_3.2_1b/llama_cpu.py:170-285, restated) on the exactly
dequantized weights and the same cache:
  - every logit within rtol 2e-2 / atol 1e-2 (the north star's floating-point bar);
  - KL(oracle || B200) of the next-token distribution within IRON's decode bound of
    0.05 (iron/applications/llama_3.2_1b/test.py:77-97);
  - the greedy token equal to the oracle's wherever the oracle's best logit leads the
    runner-up by more than the tolerance (a closer race is a tie at this precision).
Tokens are teacher-forced (the same input token on both sides every step), as IRON's
accuracy check does (llama_inference_harness.py check_accuracy).
"""

import pytest
import torch

from helpers import assert_close
from oracle import llama as ollama

pytestmark = pytest.mark.gpu

from iron_b200.applications.llama_3_2_1b.decode import LlamaDecodeEngine, LlamaShape

CTX = 2048
STEPS = 3


def _oracle_weights_f32(eng):
    """The engine's exactly dequantized weights as fp32 CPU tensors (the oracle's
    matmuls convert to fp32 anyway; converting once keeps the 16-layer steps short)."""
    s = eng.s
    H, E = s.hidden_dim, s.emb_dim
    q_rows, kv_rows = s.n_heads * s.head_dim, s.n_kv_groups * s.head_dim
    out = []
    for lay in eng.layers:
        qkv = lay["qkv"].dequant().float().cpu()
        gu = lay["gu"].dequant().float().cpu().reshape(-1, 16, E)
        out.append({
            "n1": lay["n1"].cpu(), "n2": lay["n2"].cpu(),
            "q": qkv[:q_rows], "k": qkv[q_rows:q_rows + kv_rows], "v": qkv[q_rows + kv_rows:],
            "o": lay["o"].dequant().float().cpu(),
            "g": gu[:, :8].reshape(H, E).contiguous(), "u": gu[:, 8:].reshape(H, E).contiguous(),
            "d": lay["d"].dequant().float().cpu(),
        })
    return out


def _kl(ref_logits, got_logits):
    lp = torch.log_softmax(ref_logits.float(), -1)
    return (lp.exp() * (lp - torch.log_softmax(got_logits.float(), -1))).sum(-1)


@pytest.mark.parametrize("batch", [1, 64])
def test_full_model_decode_matches_oracle(batch):
    torch.set_num_threads(max(1, torch.get_num_threads()))
    shape = LlamaShape()
    eng = LlamaDecodeEngine(shape, batch, CTX + STEPS + 13, seed=1234, keep_natural=True)
    g = torch.Generator(device="cuda").manual_seed(99)
    for li in range(shape.n_layers):  # the prompt's KV cache (synthetic, as bench.py builds it)
        eng.kc[li, :, :, :CTX].normal_(generator=g)
        eng.vc[li, :, :, :CTX].normal_(generator=g)
    if batch == 1:
        pos0 = [CTX]
    else:  # ragged positions up to the context; the first sequences sit at the edges
        pos0 = [CTX, 1, 63, 64, 65, 1000] + torch.randint(1, CTX + 1, (batch - 6,), generator=torch.Generator()
                                                          .manual_seed(3)).tolist()
    teach = torch.randint(0, shape.vocab_size, (STEPS, batch), generator=torch.Generator().manual_seed(7),
                          dtype=torch.int32)
    eng.set_state(teach[0], pos0)
    kc = [eng.kc[li].cpu() for li in range(shape.n_layers)]
    vc = [eng.vc[li].cpu() for li in range(shape.n_layers)]
    eng.capture()  # the benched path: one CUDA graph replay per step

    W = _oracle_weights_f32(eng)
    nf, emb = eng.nf.cpu(), eng.embed_table.cpu()
    lm = eng.lm.dequant().float().cpu()
    lut = eng.lut.cpu()
    worst = {"mismatch": 0.0, "kl": 0.0}
    for t in range(STEPS):
        eng.tokens.copy_(teach[t].cuda())
        eng.step()
        torch.cuda.synchronize()
        got = eng.logits.cpu()
        pos = [p + t for p in pos0]
        ref = ollama.model_decode(teach[t].tolist(), pos, W, nf, emb, lm, kc, vc, lut, shape.n_heads,
                                  shape.n_kv_groups, shape.head_dim)
        d = (got.float() - ref.float()).abs()
        bad = d >= torch.maximum(torch.full_like(d, 1e-2), 2e-2 * (got.float().abs() + ref.float().abs()))
        worst["mismatch"] = max(worst["mismatch"], float(bad.float().mean()))
        kl = _kl(ref, got)
        worst["kl"] = max(worst["kl"], float(kl.max()))
        print(f"batch {batch} step {t}: max |diff| {float(d.max()):.3g}, outside tolerance "
              f"{int(bad.sum())}/{bad.numel()}, max KL {float(kl.max()):.3g}")
        assert_close(got, ref, 2e-2, 1e-2, what=f"logits, step {t}")
        assert float(kl.max()) <= 0.05, kl
        # greedy token: the engine's argmax epilogue vs the oracle where the race is clear
        # (each of the two leading logits may move by the tolerance, in opposite directions)
        top2 = ref.float().topk(2, dim=-1)
        tol = torch.maximum(torch.full_like(top2.values[:, 0], 1e-2), 4e-2 * top2.values[:, 0].abs())
        clear = (top2.values[:, 0] - top2.values[:, 1]) > 2 * tol
        tok = eng.tokens.cpu().long()
        assert torch.equal(tok[clear], top2.indices[clear, 0]), "greedy token differs from the oracle's"
        # the engine's own token is the first maximum of the logits it wrote
        gf = got.float()
        assert torch.all(gf.gather(1, tok[:, None])[:, 0] == gf.max(1).values)
        assert eng.pos.cpu().tolist() == [p + 1 for p in pos]
    # the appended K / V rows of the last step against the oracle's (the cache under test).
    # Layer 0's rows depend on the embedding, one RMSNorm and the QKV GEMV only: every
    # entry within tolerance. The last layer's rows are raw projections of a hidden state
    # that carries 15 layers of bf16 rounding differences (fp32 sums in other orders
    # rounding an ulp apart): measured on B200, 3 of sequence 0's 512 k entries at layer
    # 15 (batch 64) fell outside 2e-2 / 1e-2, the worst 0.113 against 0.102 in a row of
    # RMS ~2.5 -- 0.4 % of the row's scale, while every logit stayed within tolerance.
    # With the tensor-core GEMV at batch 64 (another summation order) 6 of sequence 2's
    # 512 entries, the worst 0.1016 against 0.1118 (0.4 % of the row RMS). So there: at
    # most 2 % of the entries outside, and no error above 2 % of the row RMS.
    for li in (0, shape.n_layers - 1):
        frac = 0.0 if li == 0 else 2e-2
        for b in range(min(batch, 8)):
            p = pos0[b] + STEPS - 1
            for name, got_c, ref_c in (("k", eng.kc, kc), ("v", eng.vc, vc)):
                got_r, ref_r = got_c[li, b, :, p].cpu().float(), ref_c[li][b, :, p].float()
                assert_close(got_r, ref_r, 2e-2, 1e-2, max_mismatch_frac=frac, what=f"{name} row L{li} b{b}")
                rms = float(ref_r.pow(2).mean().sqrt())
                assert float((got_r - ref_r).abs().max()) <= 2e-2 * rms, f"{name} row L{li} b{b}"
    print(f"batch {batch}: worst mismatch fraction {worst['mismatch']:.3g}, worst KL {worst['kl']:.3g}")
