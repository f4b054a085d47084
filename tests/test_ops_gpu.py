"""Row-wise / element-wise / data-movement operators on the B200 vs the oracle.

Shapes and tolerances follow IRON's tests: rms_norm/test.py (relative 0.04, 1e-6),
rope/test.py (relative 0.05), softmax/test.py (relative 0.04, 1e-6), silu / mul /
add (relative 0.04, 1e-6), strided_copy/test.py / repeat / transpose (exact).
"""

import numpy as np
import pytest
import torch

from helpers import assert_close, bf16, bits, load, load_kwargs
from oracle import ops

pytestmark = pytest.mark.gpu

from iron_b200 import _lib
from iron_b200.common.test_utils import run_test
from iron_b200.operators import (RMSNorm, RoPE, Softmax, SiLU, ElementwiseMul, ElementwiseAdd,
                                 StridedCopy, Repeat, Transpose)


# ---- RMSNorm -------------------------------------------------------------------
def test_rms_norm_golden_fixtures():
    d = load("rms_norm_w_4x256")
    op = RMSNorm(size=1024, num_aie_columns=1, num_channels=1, tile_size=256, weighted=True)
    errors, _, _ = run_test(op, {"x": bf16(d["x"]), "w": bf16(d["w"])}, {"out": bf16(d["out"])},
                            rel_tol=0.04, abs_tol=1e-6)
    assert not errors
    d = load("rms_norm_2x2048")
    op = RMSNorm(size=4096, num_aie_columns=1, num_channels=1, tile_size=2048)
    errors, _, _ = run_test(op, {"x": bf16(d["x"])}, {"out": bf16(d["out"])}, rel_tol=0.04, abs_tol=1e-6)
    assert not errors


@pytest.mark.parametrize("rows,cols,weighted", [(1, 2048, True), (64, 2048, True), (16, 4096, False),
                                                (2048, 4096, True), (3, 100, True), (1, 8192, True),
                                                (2, 16384, False)])
def test_rms_norm_shapes(rows, cols, weighted):
    torch.manual_seed(rows + cols)
    x = (torch.rand(rows, cols) * 4).to(torch.bfloat16)
    w = (1 + 0.02 * torch.randn(cols)).to(torch.bfloat16)
    op = RMSNorm(size=rows * cols, num_aie_columns=1, num_channels=1, tile_size=cols, weighted=weighted)
    ins = {"x": x, "w": w} if weighted else {"x": x}
    exp = ops.rms_norm(x, w if weighted else None)
    errors, _, _ = run_test(op, ins, {"out": exp}, rel_tol=0.04, abs_tol=1e-6)
    assert not errors


def test_rms_norm_fused_residual():
    torch.manual_seed(1)
    rows, cols = 16, 2048
    x, r = torch.randn(rows, cols).to(torch.bfloat16), torch.randn(rows, cols).to(torch.bfloat16)
    w = (1 + 0.02 * torch.randn(cols)).to(torch.bfloat16)
    xd, rd, wd = x.cuda(), r.cuda(), w.cuda()
    h = torch.empty_like(xd)
    y = torch.empty_like(xd)
    _lib.call("iron_rmsnorm", xd.data_ptr(), rd.data_ptr(), h.data_ptr(), wd.data_ptr(), y.data_ptr(),
              rows, cols, 1e-5, 0, _lib.current_stream())
    hh = ops.add(x, r)
    assert torch.equal(h.cpu(), hh)
    assert_close(y.cpu(), ops.rms_norm(hh, w), 0.04, 1e-6, what="rmsnorm(x+r)")


# ---- RoPE ------------------------------------------------------------------------
@pytest.mark.parametrize("name", ["rope_32x128_a8", "rope_32x64_a1", "rope_64x128_a32"])
@pytest.mark.parametrize("method", [0, 1])
def test_rope_golden_bit_exact(name, method):
    d = load(name)
    x, ang = bf16(d["x"]), bf16(d["angles"])
    op = RoPE(rows=x.shape[0], cols=x.shape[1], angle_rows=ang.shape[0], method_type=method)
    errors, _, _ = run_test(op, {"x": x, "angles": ang}, {"out": bf16(d[f"out{method}"])},
                            rel_tol=0.0, abs_tol=0.0)
    assert not errors


def test_rope_position_indexed_decode():
    torch.manual_seed(2)
    B, H, D = 5, 32, 64
    lut = ops.rope_angles(D, 4096)
    pos = torch.tensor([0, 7, 1000, 4095, 31], dtype=torch.int32)
    x = torch.randn(B * H, D).to(torch.bfloat16)
    y = torch.empty(B * H, D, dtype=torch.bfloat16, device="cuda")
    xd, lutd, posd = x.cuda(), lut.cuda(), pos.cuda()
    _lib.call("iron_rope", xd.data_ptr(), None, lutd.data_ptr(), y.data_ptr(), B * H, D, B,
              posd.data_ptr(), 0, 0, _lib.current_stream())
    exp = torch.cat([ops.rope(x[b * H:(b + 1) * H], lut[int(pos[b]):int(pos[b]) + 1].to(torch.bfloat16))
                     for b in range(B)])
    # the kernel reads the fp32 table; the oracle row here is bf16-rounded -> compare loosely
    assert_close(y.cpu(), exp, 0.02, 1e-2, what="rope pos")


# ---- Softmax ---------------------------------------------------------------------
def test_softmax_golden_fixture():
    d = load("softmax_16x512")
    op = Softmax(rows=16, cols=512)
    errors, _, _ = run_test(op, {"x": bf16(d["x"]).flatten()}, {"out": bf16(d["out"]).flatten()},
                            rel_tol=0.04, abs_tol=1e-6)
    assert not errors


@pytest.mark.parametrize("rows,cols,valid", [(32, 2048, 1), (32, 2048, 1000), (32, 2048, 2048),
                                             (4096, 512, 512), (16, 32768, 20000)])
def test_softmax_masked(rows, cols, valid):
    torch.manual_seed(valid)
    x = (torch.rand(rows, cols) * 4).to(torch.bfloat16)
    op = Softmax(rows=rows, cols=cols, rtp_vector_size=valid)
    errors, _, _ = run_test(op, {"x": x.flatten()}, {"out": ops.softmax(x, valid).flatten()},
                            rel_tol=0.04, abs_tol=1e-6)
    assert not errors


def test_softmax_runtime_length_from_device():
    rows, cols = 32, 2048
    x = (torch.rand(rows, cols) * 4).to(torch.bfloat16).cuda()
    op = Softmax(rows=rows, cols=cols, rtp_vector_size=cols, vector_size_parameter="n")
    word = torch.zeros(1, dtype=torch.int32, device="cuda")
    op.bind_param("n", word)
    fn = op.get_callable()
    for n in (1, 17, 2048):
        word.fill_(n)
        y = torch.empty(rows * cols, dtype=torch.bfloat16, device="cuda")
        fn(x.flatten(), y)
        assert_close(y.cpu(), ops.softmax(x.cpu(), n).flatten(), 0.04, 1e-6, what=f"n={n}")


# ---- element-wise -----------------------------------------------------------------
@pytest.mark.parametrize("name", ["silu_2048", "mul_2048", "add_2048"])
def test_eltwise_golden(name):
    d = load(name)
    if name.startswith("silu"):
        op = SiLU(size=2048, num_aie_columns=1, tile_size=2048)
        ins = {"x": bf16(d["x"])}
    else:
        cls = ElementwiseMul if name.startswith("mul") else ElementwiseAdd
        op = cls(size=2048, tile_size=256)
        ins = {"a": bf16(d["a"]), "b": bf16(d["b"])}
    errors, _, _ = run_test(op, ins, {"out": bf16(d["out"])}, rel_tol=0.04, abs_tol=1e-6)
    assert not errors


@pytest.mark.parametrize("n", [8192, 1 << 23, 1000])
def test_eltwise_sizes_and_swiglu(n):
    torch.manual_seed(n)
    a, b = (torch.randn(n) * 4).to(torch.bfloat16), (torch.randn(n) * 4).to(torch.bfloat16)
    ad, bd = a.cuda(), b.cuda()
    for op, exp in [(0, ops.silu(a)), (1, ops.mul(a, b)), (2, ops.add(a, b)), (3, ops.swiglu_act(a, b))]:
        y = torch.empty(n, dtype=torch.bfloat16, device="cuda")
        _lib.call("iron_eltwise", ad.data_ptr(), bd.data_ptr(), y.data_ptr(), n, op, 0, _lib.current_stream())
        assert_close(y.cpu(), exp, 0.04, 1e-6, what=f"op{op}")


# ---- StridedCopy / Repeat / Transpose ------------------------------------------------------
@pytest.mark.parametrize("case", ["flat1024", "flat1024_ch4", "kv_slot0", "kv_slot5", "kv_slot_last",
                                  "kv_slot5_ch2", "kv_slot5_ch4", "kv_llama_full", "kv_addend7"])
def test_strided_copy_golden_exact(case):
    d = load(f"strided_copy_{case}")
    kw = load_kwargs(d)
    add = kw.pop("output_offset_addend", 0)
    op = StridedCopy(**kw, output_offset_parameter="cache_offset" if add else None)
    if add:
        word = torch.tensor([add], dtype=torch.int32, device="cuda")
        op.bind_param("cache_offset", word)
    errors, _, _ = run_test(op, {"in": bf16(d["input"])}, {"out": bf16(d["output"])},
                            rel_tol=0.0, abs_tol=0.0)
    assert not errors


def test_strided_copy_cache_offset_runtime_whole_cache():
    """Three appends at slots 0, 5, 127 through one op whose offset is a device word;
    the WHOLE cache is checked (iron/operators/strided_copy/test.py:109-153)."""
    N_KV, HD, SEQ = 8, 64, 128
    kw = dict(input_sizes=[N_KV, HD], input_strides=[HD, 1], input_offset=0,
              input_buffer_size=N_KV * HD, output_sizes=[1, N_KV, HD],
              output_strides=[0, SEQ * HD, 1], output_offset=0, output_buffer_size=N_KV * SEQ * HD)
    op = StridedCopy(**kw, output_offset_parameter="cache_offset")
    word = torch.zeros(1, dtype=torch.int32, device="cuda")
    op.bind_param("cache_offset", word)
    fn = op.get_callable()
    cache = torch.zeros(N_KV * SEQ * HD, dtype=torch.bfloat16, device="cuda")
    expected = torch.zeros(N_KV * SEQ * HD, dtype=torch.bfloat16)
    for i, slot in enumerate((0, 5, SEQ - 1)):
        torch.manual_seed(i + 1)
        src = (torch.rand(N_KV * HD) * 4).to(torch.bfloat16)
        word.fill_(slot * HD)
        fn(src.cuda(), cache)
        expected = ops.strided_copy(src, kw["input_sizes"], kw["input_strides"], 0, kw["output_buffer_size"],
                                    kw["output_sizes"], kw["output_strides"], 0, 1, 0, slot * HD,
                                    out=expected)
        np.testing.assert_array_equal(bits(cache.cpu()), bits(expected))


def test_repeat_and_transpose():
    d = load("repeat_8x256_r4")
    errors, _, _ = run_test(Repeat(rows=8, cols=256, repeat=4), {"x": bf16(d["x"])}, {"out": bf16(d["out"])},
                            rel_tol=0.0, abs_tol=0.0)
    assert not errors
    d = load("transpose_2x64x32")
    op = Transpose(M=64, N=32, num_aie_columns=1, num_channels=1, m=16, n=16, s=8, num_batches=2)
    errors, _, _ = run_test(op, {"x": bf16(d["x"]).reshape(2, -1)}, {"out": bf16(d["out"]).reshape(2, -1)},
                            rel_tol=0.0, abs_tol=0.0)
    assert not errors


def test_repeat_transpose_llama_shapes():
    x = torch.randn(8, 2048 * 64).to(torch.bfloat16)
    errors, _, _ = run_test(Repeat(rows=8, cols=2048 * 64, repeat=4, transfer_size=64), {"x": x},
                            {"out": ops.repeat_interleave(x, 4)}, rel_tol=0.0, abs_tol=0.0)
    assert not errors
    v = torch.randn(32, 2048 * 64).to(torch.bfloat16)
    op = Transpose(M=2048, N=64, num_aie_columns=2, num_channels=1, m=256, n=32, s=8, num_batches=32)
    errors, _, _ = run_test(op, {"x": v}, {"out": ops.transpose(v.reshape(32, 2048, 64)).reshape(32, -1)},
                            rel_tol=0.0, abs_tol=0.0)
    assert not errors
    # odd row width goes through the strided path
    x = torch.randn(3, 5).to(torch.bfloat16)
    errors, _, _ = run_test(Repeat(rows=3, cols=5, repeat=3), {"x": x}, {"out": ops.repeat_interleave(x, 3)},
                            rel_tol=0.0, abs_tol=0.0)
    assert not errors
