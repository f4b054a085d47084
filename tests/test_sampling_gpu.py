"""On-device next-token sampling (iron_sample_topk) against IRON's generate_token
(iron/applications/llama_3.2_1b/llama_inference_harness.py:146-169), restated as
oracle.ops.sample_probs: the empirical distribution of many draws matches the
oracle's probabilities (chi-square test), tokens outside the top-k are never drawn,
and the draws are bitwise reproducible for a fixed seed."""

import pytest
import torch
from scipy import stats

from oracle import ops

pytestmark = pytest.mark.gpu

from iron_b200 import _lib


def _sample(logits, temperature, top_k, seed, pos=None):
    B, V = logits.shape
    tok = torch.full((B,), -7, dtype=torch.int32, device="cuda")
    _lib.call("iron_sample_topk", logits.data_ptr(), B, V, temperature, top_k, seed, tok.data_ptr(),
              pos.data_ptr() if pos is not None else None, 0, _lib.current_stream())
    torch.cuda.synchronize()
    return tok.cpu().long()


@pytest.mark.parametrize("temperature,top_k", [(0.7, 50), (1.0, 0), (0.0, 20), (2.0, 1000)])
def test_draws_follow_the_harness_distribution(temperature, top_k):
    V, N = 4096, 16384
    g = torch.Generator().manual_seed(int(temperature * 10) + top_k)
    row = (torch.randn(V, generator=g) * 2).to(torch.bfloat16)
    probs = ops.sample_probs(row[None], temperature, top_k if top_k > 0 else None)[0]
    # N rows holding the same logits: row b draws with counter (seed, b, position 0)
    toks = _sample(row.cuda()[None].expand(N, V).contiguous(), temperature, top_k, seed=1234)
    counts = torch.bincount(toks, minlength=V).double()
    assert int(counts[probs == 0].sum()) == 0, "drew a token outside the top-k"
    exp = probs * N
    big = exp >= 5  # chi-square bins; the rest pooled
    obs = torch.cat([counts[big], counts[~big].sum()[None]])
    e = torch.cat([exp[big], exp[~big].sum()[None]])
    keep = e > 0
    chi2 = float(((obs[keep] - e[keep]) ** 2 / e[keep]).sum())
    crit = stats.chi2.ppf(0.999, int(keep.sum()) - 1)
    assert chi2 < crit, f"chi2 {chi2:.1f} >= {crit:.1f} (df {int(keep.sum()) - 1})"


def test_full_vocab_rows_and_determinism():
    B, V, k = 64, 128256, 50
    g = torch.Generator(device="cuda").manual_seed(3)
    logits = (torch.randn(B, V, device="cuda", generator=g) * 3).to(torch.bfloat16)
    pos = torch.arange(B, dtype=torch.int32, device="cuda") * 7
    a = _sample(logits, 0.7, k, seed=99, pos=pos.clone())
    b = _sample(logits, 0.7, k, seed=99, pos=pos.clone())
    c = _sample(logits, 0.7, k, seed=100, pos=pos.clone())
    assert torch.equal(a, b), "not reproducible for a fixed seed"
    assert (a != c).sum() > B // 4, "the seed does not change the draws"
    kth = logits.float().topk(k, dim=-1).values[:, -1].cpu()
    got = logits.float().cpu().gather(1, a[:, None])[:, 0]
    assert torch.all(got >= kth), "a token outside the top-k"
    # positions advance; top_k = 1 is the argmax (all maxima kept: any of them)
    p2 = pos.clone()
    t1 = _sample(logits, 0.7, 1, seed=5, pos=p2)
    assert torch.equal(p2.cpu(), (pos + 1).cpu())
    mx = logits.float().max(1).values.cpu()
    assert torch.all(logits.float().cpu().gather(1, t1[:, None])[:, 0] == mx)


def test_engine_sampling_step():
    from iron_b200.applications.llama_3_2_1b.decode import LlamaDecodeEngine, LlamaShape, SamplingConfig

    shape = LlamaShape(n_layers=2, vocab_size=4096)
    runs = []
    for _ in range(2):
        eng = LlamaDecodeEngine(shape, 4, 64, seed=3, sampling=SamplingConfig(0.7, 50, seed=11))
        eng.set_state([11, 12, 13, 14], [4, 9, 1, 30])
        eng.capture()
        toks = []
        for _ in range(4):
            eng.step()
            toks.append(eng.tokens.clone())
            lg = eng.logits.float()
            kth = lg.topk(50, dim=-1).values[:, -1]
            assert torch.all(lg.gather(1, eng.tokens.long()[:, None])[:, 0] >= kth)
        torch.cuda.synchronize()
        assert eng.pos.cpu().tolist() == [8, 13, 5, 34]
        runs.append(torch.stack(toks).cpu())
    assert torch.equal(runs[0], runs[1])
