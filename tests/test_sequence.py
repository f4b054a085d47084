"""OperatorSequence host logic on the CPU: buffer layout, slice notation,
the reference dispatch, the coherence map of the buffer shim, and SwiGLUDecode
through the reference dispatch against IRON's golden
(iron/tests/infrastructure/sequence.py:184-271, swiglu_decode/test.py:65-101)."""

import numpy as np
import pytest
import torch

from helpers import bf16, load
from iron_b200.common.sequence import (CompareDispatch, FusedDispatch, OperatorSequence,
                                       ReferenceDispatch)
from iron_b200.common.tensor import CPUOnlyTensor, _Intervals
from iron_b200.common.test_utils import verify_buffer
from iron_b200.operators import ElementwiseAdd, GEMV, SiLU, Softmax, StridedCopy, SwiGLUDecode, SwiGLUPrefill

N = 1024
NB = 2 * N


def _packed_seq(dispatch):
    add0 = ElementwiseAdd(size=N, tile_size=N, num_aie_columns=1)
    add1 = ElementwiseAdd(size=N, tile_size=N, num_aie_columns=1)
    return OperatorSequence(name="packed", runlist=[(add0, "a0", "b0", f"packed[0:{NB}]"),
                                                     (add1, "a1", "b1", f"packed[{NB}:{2 * NB}]")],
                            input_args=["a0", "b0", "a1", "b1"], output_args=["packed"],
                            buffer_sizes={"packed": 2 * NB}, dispatch=dispatch)


def test_layout_and_slices():
    seq = _packed_seq("reference").compile(dry_run=True)
    assert seq.buffer_sizes[0] == 4 * NB and seq.buffer_sizes[1] == 2 * NB
    assert seq.get_layout_for_buffer(f"packed[{NB}:{2 * NB}]") == ("output", NB, 2 * NB)
    kinds = {n: seq.subbuffer_layout[n][0] for n in ("a0", "b1", "packed")}
    assert kinds == {"a0": "input", "b1": "input", "packed": "output"}
    offs = sorted(v[1] for k, v in seq.subbuffer_layout.items() if v[0] == "input")
    assert all(o % 256 == 0 for o in offs)


def test_layout_errors():
    add = ElementwiseAdd(size=N, tile_size=N, num_aie_columns=1)
    with pytest.raises(ValueError, match="requires explicit size"):
        OperatorSequence("s", [(add, "a", "b", "p[0:8]")], ["a", "b"], ["p"]).compile(dry_run=True)
    with pytest.raises(ValueError, match="not found"):
        OperatorSequence("s", [(add, "a", "b", "c")], ["a", "zz"], ["c"]).compile(dry_run=True)
    with pytest.raises(ValueError, match="must match"):
        OperatorSequence("s", [(add, "a", "c")], ["a"], ["c"]).compile(dry_run=True)
    big = ElementwiseAdd(size=2 * N, tile_size=N, num_aie_columns=1)
    with pytest.raises(ValueError, match="conflicting sizes"):
        OperatorSequence("s", [(add, "a", "b", "c"), (big, "c", "c", "d")], ["a", "b"], ["d"]).compile(dry_run=True)
    with pytest.raises(ValueError, match="ends past"):
        OperatorSequence("s", [(add, "a", "b", "p[0:4096]")], ["a", "b"], ["p"],
                         buffer_sizes={"p": 1024}).compile(dry_run=True)
    with pytest.raises(TypeError):
        OperatorSequence("s", [(object(), "a")], ["a"], ["a"])
    with pytest.raises(TypeError):
        OperatorSequence("s", [(add, "a", "b", "c")], ["a", "b"], ["c"], dispatch="bogus")


def test_dispatch_names_and_params():
    assert OperatorSequence("s", [], [], [], dispatch="auto").compile(dry_run=True)._dispatch.name == "fused"
    assert isinstance(OperatorSequence._coerce_dispatch(CompareDispatch()), CompareDispatch)
    sm = Softmax(rows=16, cols=64, vector_size_parameter="softmax_vector_size")
    sc = StridedCopy(input_sizes=(1, 1, 1, 64), input_strides=(0, 0, 0, 1), input_offset=0,
                     output_sizes=(1, 1, 1, 64), output_strides=(0, 0, 0, 1), output_offset=0,
                     input_buffer_size=64, output_buffer_size=640, output_offset_parameter="cache_offset")
    seq = OperatorSequence("p", [(sm, "x", "y"), (sc, "k", "cache")], ["x", "k"], ["y"],
                           dispatch=FusedDispatch())
    assert seq.runtime_parameters() == ["softmax_vector_size", "cache_offset"]
    assert seq.name == "p"
    assert OperatorSequence("p", [], [], [], share_designs=True).name == "p_shared"


def test_reference_dispatch_resolves_sliced_buffer():
    torch.manual_seed(0)
    a0, b0, a1, b1 = (torch.rand(N, dtype=torch.bfloat16) for _ in range(4))
    seq = _packed_seq("reference").compile()
    run = seq.get_callable()
    for name, t in (("a0", a0), ("b0", b0), ("a1", a1), ("b1", b1)):
        buf = run.get_buffer(name)
        assert isinstance(buf, CPUOnlyTensor)
        buf.torch_view()[:] = t
        buf.to("npu")  # a no-op on host-only buffers
    run()
    packed = run.get_buffer("packed").torch_view()[: 2 * N].clone()
    assert not verify_buffer(packed, "packed", torch.cat([a0 + b0, a1 + b1]), rel_tol=0.04, abs_tol=1e-6)
    assert run.params is None


def test_swiglu_decode_reference_dispatch_matches_golden():
    d = {k: bf16(v) for k, v in load("swiglu_decode_e256_h512").items()}
    E, H = 256, 512
    seq = SwiGLUDecode(embedding_dim=E, hidden_dim=H, dispatch=ReferenceDispatch()).compile()
    assert seq.name == "swiglu_decode_e256_h512"
    run = seq.get_callable()
    run.get_buffer("w_gate").torch_view()[:] = d["w_gate"].T.reshape(-1)
    run.get_buffer("w_up").torch_view()[:] = d["w_up"].T.reshape(-1)
    run.get_buffer("w_down").torch_view()[:] = d["w_down"].T.reshape(-1)
    run.get_buffer("in").torch_view()[:] = d["input"].reshape(-1)
    run()
    for name, key in (("left", "left"), ("right", "right"), ("left_swished", "left_swished")):
        got = run.get_buffer(name).torch_view().reshape(1, H)
        assert not verify_buffer(got, name, d[key], rel_tol=0.04, abs_tol=0.4)
    inter = run.get_buffer("intermediate").torch_view().reshape(1, H)
    ls = run.get_buffer("left_swished").torch_view().reshape(1, H)
    right = run.get_buffer("right").torch_view().reshape(1, H)
    assert not verify_buffer(inter, "intermediate", ls * right, rel_tol=0.04, abs_tol=0.4)
    out = run.get_buffer("out").torch_view().reshape(1, E)
    assert not verify_buffer(out, "out", inter @ d["w_down"], rel_tol=0.04, abs_tol=0.4)


def test_swiglu_prefill_reference_dispatch_and_buffers():
    """SwiGLUPrefill's runlist on the CPU reference dispatch: IRON's buffer names and
    layouts, both weight layouts, intermediates chained as IRON checks them."""
    S, E, H = 256, 512, 512
    for b_col_maj in (False, True):
        g = torch.Generator().manual_seed(7)
        x = torch.randn(S, E, generator=g).to(torch.bfloat16)
        w_gate = (torch.randn(E, H, generator=g) * 0.1).to(torch.bfloat16)  # (K, N)
        w_up = (torch.randn(E, H, generator=g) * 0.1).to(torch.bfloat16)
        w_down = (torch.randn(H, E, generator=g) * 0.1).to(torch.bfloat16)
        seq = SwiGLUPrefill(seq_len=S, embedding_dim=E, hidden_dim=H, b_col_maj=b_col_maj,
                            dispatch=ReferenceDispatch()).compile()
        assert seq.name == f"swiglu_prefill_s{S}_e{E}_h{H}" + ("_bc" if b_col_maj else "")
        run = seq.get_callable()

        def stored(w):
            return (w.T if b_col_maj else w).contiguous().reshape(-1)

        run.get_buffer("w_gate").torch_view()[:] = stored(w_gate)
        run.get_buffer("w_up").torch_view()[:] = stored(w_up)
        run.get_buffer("w_down").torch_view()[:] = stored(w_down)
        run.get_buffer("in").torch_view()[:] = x.reshape(-1)
        run()
        left = run.get_buffer("left").torch_view().reshape(S, H)
        assert not verify_buffer(left, "left", (x.float() @ w_gate.float()).to(torch.bfloat16), rel_tol=0.04,
                                 abs_tol=0.4)
        ls = run.get_buffer("left_swished").torch_view().reshape(S, H)
        right = run.get_buffer("right").torch_view().reshape(S, H)
        inter = run.get_buffer("intermediate").torch_view().reshape(S, H)
        assert not verify_buffer(inter, "intermediate", ls * right, rel_tol=0.04, abs_tol=0.4)
        out = run.get_buffer("out").torch_view().reshape(S, E)
        assert not verify_buffer(out, "out", (inter.float() @ w_down.float()).to(torch.bfloat16), rel_tol=0.08,
                                 abs_tol=0.4, max_error_rate=0.05)


def test_intervals():
    iv = _Intervals()
    iv.add(10, 20)
    iv.add(30, 40)
    iv.add(15, 32)
    assert iv.iv == [(10, 40)]
    iv.add(0, 5)
    iv.add(50, 60)
    assert iv.iv == [(0, 5), (10, 40), (50, 60)]
    assert iv.take(12, 55) == [(12, 40), (50, 55)]
    assert iv.iv == [(0, 5), (10, 12), (55, 60)]
    assert iv.take(100, 200) == []
    iv.add(5, 10)
    assert iv.iv == [(0, 12), (55, 60)]


def test_gemv_in_reference_sequence():
    torch.manual_seed(3)
    M, K = 64, 128
    W = torch.randn(M, K).to(torch.bfloat16)
    x = torch.randn(K).to(torch.bfloat16)
    op = GEMV(M=M, K=K)
    seq = OperatorSequence("g", [(op, "W", "x", "y")], ["x"], ["y"], dispatch="reference").compile()
    run = seq.get_callable()
    run.get_buffer("W").torch_view()[:] = W.reshape(-1)
    run.get_buffer("x").torch_view()[:] = x
    run()
    ref = (W.float() @ x.float()).to(torch.bfloat16)
    assert torch.equal(run.get_buffer("y").torch_view(), ref)
