"""OperatorSequence on the B200: every dispatch mode, runtime parameters bound to
device words, buffer coherence across calls, and SwiGLUDecode
(iron/tests/infrastructure/sequence.py:184-360, swiglu_decode/test.py:36-101,
strided_copy/test.py:109-153)."""

import numpy as np
import pytest
import torch

from helpers import bf16, load
from iron_b200.common.sequence import CompareDispatch, OperatorSequence
from iron_b200.common.test_utils import verify_buffer
from iron_b200.common.verify import Tolerance
from iron_b200.operators import ElementwiseAdd, GEMV, SiLU, Softmax, StridedCopy, SwiGLUDecode, SwiGLUPrefill

pytestmark = pytest.mark.gpu

SIZE = 4096


def _add_silu(dispatch, input_args=("a", "b")):
    add = ElementwiseAdd(size=SIZE, tile_size=1024, num_aie_columns=4)
    silu = SiLU(size=SIZE, num_aie_columns=4, tile_size=1024)
    return OperatorSequence(name="add_silu", runlist=[(add, "a", "b", "temp"), (silu, "temp", "out")],
                            input_args=list(input_args), output_args=["out"], dispatch=dispatch)


def _run_add_silu(dispatch, a, b):
    seq = _add_silu(dispatch).compile()
    run = seq.get_callable()
    for n, t in (("a", a), ("b", b)):
        run.get_buffer(n).torch_view()[:] = t
        run.get_buffer(n).to("npu")
    run()
    return run.get_buffer("out").torch_view()[:SIZE].clone()


def test_auto_dispatch_is_graph_and_correct():
    torch.manual_seed(0)
    a = torch.rand(SIZE, dtype=torch.bfloat16) * 4 - 2
    b = torch.rand(SIZE, dtype=torch.bfloat16) * 4 - 2
    seq = _add_silu("auto").compile()
    assert seq._dispatch.name == "fused"
    out = _run_add_silu("auto", a, b)
    exp = torch.nn.functional.silu((a + b).float()).to(torch.bfloat16)
    assert not verify_buffer(out, "out", exp, rel_tol=0.04, abs_tol=1e-6)


@pytest.mark.parametrize("dispatch", ["fused", "compare"])
def test_dispatch_modes_bit_identical(dispatch):
    torch.manual_seed(0)
    a = torch.rand(SIZE, dtype=torch.bfloat16) * 4 - 2
    b = torch.rand(SIZE, dtype=torch.bfloat16) * 4 - 2
    assert torch.equal(_run_add_silu(dispatch, a, b), _run_add_silu("separate", a, b))


@pytest.mark.parametrize("exact", [False, True])
def test_compare_mode_judges_each_step_by_its_tolerance(exact):
    # the GEMV's fp32 sums differ from torch's in summation order: within its
    # contract, but a few of 16384 outputs land on the other side of a bf16
    # rounding boundary (about 1 in 1000 at K = 4096)
    torch.manual_seed(0)
    M, K = 16384, 4096
    op = GEMV(M=M, K=K)
    seq = OperatorSequence("cmp_gemv", [(op, "W", "x", "y")], ["x"], ["y"],
                           dispatch=CompareDispatch(tolerance=Tolerance.exact() if exact else None)).compile()
    assert seq._dispatch.name == "compare"
    run = seq.get_callable()
    run.get_buffer("W").torch_view()[:] = torch.randn(M * K).to(torch.bfloat16)
    run.get_buffer("x").torch_view()[:] = torch.randn(K).to(torch.bfloat16)
    if exact:
        with pytest.raises(RuntimeError, match="deviates from reference"):
            run()
    else:
        run()
        assert not any(s["mismatch"] for s in run.last_step_stats)
        assert len(run.last_step_stats) == 1


@pytest.mark.parametrize("dispatch", ["separate", "fused"])
def test_non_input_buffers_sync_without_explicit_flush(dispatch):
    seq = _add_silu(dispatch, input_args=["a"]).compile()
    run = seq.get_callable()
    torch.manual_seed(0)
    for rep in range(4):
        a = torch.rand(SIZE, dtype=torch.bfloat16) * 4 - 2
        b = torch.rand(SIZE, dtype=torch.bfloat16) * 4 - 2
        run.get_buffer("a").torch_view()[:] = a
        run.get_buffer("b").torch_view()[:] = b
        run()
        temp = run.get_buffer("temp").to_torch()[:SIZE]
        out = run.get_buffer("out").to_torch()[:SIZE]
        assert not verify_buffer(temp, "temp", a + b, rel_tol=0.04, abs_tol=1e-6), rep
        exp = torch.nn.functional.silu((a + b).float()).to(torch.bfloat16)
        assert not verify_buffer(out, "out", exp, rel_tol=0.04, abs_tol=1e-6), rep
    assert run.last_elapsed > 0


def test_runtime_parameters_without_recapture():
    """KV append at a runtime cache offset plus a softmax masked to a runtime
    length, in one graph; the parameters change between calls, the graph does
    not. The whole cache is checked each time (strided_copy/test.py:109-153)."""
    H, L, D = 8, 64, 64
    rows, cols = 32, 64
    kv = StridedCopy(input_sizes=(1, H, 1, D), input_strides=(0, D, 0, 1), input_offset=0,
                     output_sizes=(1, H, 1, D), output_strides=(0, L * D, 0, 1), output_offset=0,
                     input_buffer_size=H * D, output_buffer_size=H * L * D,
                     output_offset_parameter="cache_offset")
    sm = Softmax(rows=rows, cols=cols, vector_size_parameter="softmax_vector_size")
    seq = OperatorSequence("kv_sm", [(kv, "k", "cache"), (sm, "scores", "probs")], ["k", "scores"],
                           ["probs"]).compile()
    run = seq.get_callable()
    assert run.params is not None and set(run.params.names) == {"cache_offset", "softmax_vector_size"}
    g = torch.Generator().manual_seed(5)
    expect_cache = torch.zeros(H, L, D, dtype=torch.bfloat16)
    scores = torch.randn(rows, cols, generator=g).to(torch.bfloat16)
    run.get_buffer("scores").torch_view()[:] = scores.reshape(-1)
    graphs = set()
    for pos in (0, 5, 17, L - 1):
        k = torch.randn(H, D, generator=g).to(torch.bfloat16)
        run.get_buffer("k").torch_view()[:] = k.reshape(-1)
        run.params.write("cache_offset", np.int32(pos * D))
        run.params.write("softmax_vector_size", np.int32(pos + 1))
        run.params.sync()
        run()
        graphs.add(id(run.graph))
        expect_cache[:, pos] = k
        cache = run.get_buffer("cache").to_torch()[: H * L * D].reshape(H, L, D)
        assert torch.equal(cache, expect_cache), pos
        probs = run.get_buffer("probs").torch_view()[: rows * cols].reshape(rows, cols).float()
        n = pos + 1
        ref = torch.softmax(scores[:, :n].float(), dim=-1)
        assert torch.all(probs[:, n:] == 0), pos
        assert torch.allclose(probs[:, :n], ref, rtol=0.04, atol=1e-3), pos
    assert len(graphs) == 1


@pytest.mark.parametrize("embedding_dim,hidden_dim", [(2048, 2048), (1024, 3584), (2048, 8192)])
def test_swiglu_decode(embedding_dim, hidden_dim):
    """IRON's swiglu_decode/test.py on the B200: random goldens (IRON's recipe,
    ×4 value range), intermediates chained as IRON checks them."""
    E, H = embedding_dim, hidden_dim
    g = torch.Generator().manual_seed(42)
    x = torch.randn(1, E, generator=g).to(torch.bfloat16) * 4
    w_gate = (torch.randn(H, E, generator=g).to(torch.bfloat16) * 4).T
    w_up = (torch.randn(H, E, generator=g).to(torch.bfloat16) * 4).T
    w_down = torch.randn(H, E, generator=g).to(torch.bfloat16) * 4
    seq = SwiGLUDecode(embedding_dim=E, hidden_dim=H).compile()
    run = seq.get_callable()
    run.get_buffer("w_gate").torch_view()[:] = w_gate.T.reshape(-1)
    run.get_buffer("w_up").torch_view()[:] = w_up.T.reshape(-1)
    run.get_buffer("w_down").torch_view()[:] = w_down.T.reshape(-1)
    for name in ("w_gate", "w_up", "w_down"):
        run.get_buffer(name).to("npu")
    run.get_buffer("in").torch_view()[:] = x.reshape(-1)
    run()
    for name in ("left_swished", "right", "intermediate", "out"):
        run.get_buffer(name).to("cpu")
    left = (x.float() @ w_gate.float()).to(torch.bfloat16)
    assert not verify_buffer(run.get_buffer("left").to_torch().reshape(1, H), "left", left,
                             rel_tol=0.04, abs_tol=0.4)
    ls = run.get_buffer("left_swished").torch_view().reshape(1, H)
    right = run.get_buffer("right").torch_view().reshape(1, H)
    inter = run.get_buffer("intermediate").torch_view().reshape(1, H)
    assert not verify_buffer(inter, "intermediate", ls * right, rel_tol=0.04, abs_tol=0.4)
    out = run.get_buffer("out").torch_view().reshape(1, E)
    assert not verify_buffer(out, "output", inter @ w_down, rel_tol=0.04, abs_tol=0.4)


def test_swiglu_decode_golden_fixture():
    d = {k: bf16(v) for k, v in load("swiglu_decode_e256_h512").items()}
    seq = SwiGLUDecode(embedding_dim=256, hidden_dim=512).compile()
    run = seq.get_callable()
    run.get_buffer("w_gate").torch_view()[:] = d["w_gate"].T.reshape(-1)
    run.get_buffer("w_up").torch_view()[:] = d["w_up"].T.reshape(-1)
    run.get_buffer("w_down").torch_view()[:] = d["w_down"].T.reshape(-1)
    run.get_buffer("in").torch_view()[:] = d["input"].reshape(-1)
    run()
    for name in ("left", "right", "left_swished"):
        got = run.get_buffer(name).to_torch().reshape(1, 512)
        assert not verify_buffer(got, name, d[name], rel_tol=0.04, abs_tol=0.4)
    inter = run.get_buffer("intermediate").to_torch().reshape(1, 512)
    out = run.get_buffer("out").to_torch().reshape(1, 256)
    assert not verify_buffer(out, "output", inter @ d["w_down"], rel_tol=0.04, abs_tol=0.4)


@pytest.mark.parametrize("b_col_maj", [False, True])
def test_swiglu_prefill(b_col_maj):
    """IRON's swiglu_prefill/test.py on the B200 (seq 256, 2048 / 2048, both weight
    layouts): IRON's golden recipe, intermediates chained as IRON checks them
    (gate rel 0.04 / abs 0.4, output rel 0.08 / abs 0.4 with 5 % allowed misses)."""
    S, E, H = 256, 2048, 2048
    g = torch.Generator().manual_seed(42)
    x = torch.randn(S, E, generator=g).to(torch.bfloat16) * 4
    w_gate = (torch.randn(H, E, generator=g).to(torch.bfloat16) * 4).T  # (K, N)
    w_up = (torch.randn(H, E, generator=g).to(torch.bfloat16) * 4).T
    w_down = torch.randn(H, E, generator=g).to(torch.bfloat16) * 4
    seq = SwiGLUPrefill(seq_len=S, embedding_dim=E, hidden_dim=H, b_col_maj=b_col_maj).compile()
    run = seq.get_callable()

    def stored(w):
        return (w.T if b_col_maj else w).contiguous().reshape(-1)

    run.get_buffer("w_gate").torch_view()[:] = stored(w_gate)
    run.get_buffer("w_up").torch_view()[:] = stored(w_up)
    run.get_buffer("w_down").torch_view()[:] = stored(w_down)
    run.get_buffer("in").torch_view()[:] = x.reshape(-1)
    run()
    left = run.get_buffer("left").to_torch().reshape(S, H)
    assert not verify_buffer(left, "left", (x.float() @ w_gate.float()).to(torch.bfloat16), rel_tol=0.04,
                             abs_tol=0.4)
    ls = run.get_buffer("left_swished").to_torch().reshape(S, H)
    right = run.get_buffer("right").to_torch().reshape(S, H)
    inter = run.get_buffer("intermediate").to_torch().reshape(S, H)
    assert not verify_buffer(inter, "intermediate", ls * right, rel_tol=0.04, abs_tol=0.4)
    out = run.get_buffer("out").to_torch().reshape(S, E)
    assert not verify_buffer(out, "output", (inter.float() @ w_down.float()).to(torch.bfloat16), rel_tol=0.08,
                             abs_tol=0.4, max_error_rate=0.05)
