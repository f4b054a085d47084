"""The RMSNorm folded into the decode chain (iron_gemv_int4g32_chain, iron_embed_chain)
against the oracle's RMSNorm -> GEMV (iron/operators/rms_norm/reference.py:7-16 then
iron/operators/gemv/reference.py:9-11 on the exactly dequantized int4 weights).

The producer GEMV (residual add) writes y, bf16(y * w) and per-16-row sums of squares of
its stored y; the consumer GEMV takes bf16(y * w) and scales its output by 1 / rms(y).
That differs from IRON's chain only in where the input is rounded (bf16(y * w) against
bf16(y * w / rms)), which the north star's rtol 2e-2 / atol 1e-2 covers."""

import ctypes

import pytest
import torch

from helpers import assert_close
from oracle import ops

pytestmark = pytest.mark.gpu

from iron_b200 import _lib
from iron_b200.applications.llama_3_2_1b.decode import Int4Matrix, interleave_gate_up


def _chain(W, x, y, n_vec, flags=0, **kw):
    c = _lib.GemvChain(**{k: (v.data_ptr() if torch.is_tensor(v) else v) for k, v in kw.items()})
    _lib.call("iron_gemv_int4g32_chain", W.packed.data_ptr(), x.data_ptr(), y.data_ptr(), W.rows, W.cols, n_vec,
              ctypes.byref(c), flags, _lib.current_stream())


@pytest.mark.parametrize("E", [2048, 4096])
@pytest.mark.parametrize("n_vec", [1, 3, 8])
def test_producer_then_consumer(E, n_vec):
    g = torch.Generator(device="cuda").manual_seed(E + n_vec)
    Wp = Int4Matrix(E, 1024, g, 0.001, 0.004, keep_natural=True)     # producer: E outputs
    Wc = Int4Matrix(3072, E, g, 0.001, 0.004, keep_natural=True)     # consumer: K = E
    a = torch.randn(n_vec, 1024, device="cuda", generator=g).to(torch.bfloat16)
    res = (3 * torch.randn(n_vec, E, device="cuda", generator=g)).to(torch.bfloat16)
    w = (1 + 0.02 * torch.randn(E, device="cuda", generator=g)).to(torch.bfloat16)
    y = torch.empty(n_vec, E, dtype=torch.bfloat16, device="cuda")
    yw, ss = torch.empty_like(y), torch.empty(n_vec, E // 16, dtype=torch.float32, device="cuda")
    out = torch.empty(n_vec, 3072, dtype=torch.bfloat16, device="cuda")
    _chain(Wp, a, y, n_vec, residual=res, ss_out=ss, y_weighted=yw, weight=w)
    _chain(Wc, yw, out, n_vec, ss_in=ss, eps=1e-5)
    torch.cuda.synchronize()
    # producer: the GEMV + residual, the weighted copy (exact from its own y) and the sums
    ref_y = ops.add(ops.gemv_multi(Wp.dequant().cpu(), a.cpu()), res.cpu())
    assert_close(y.cpu(), ref_y, 2e-2, 1e-2, what="producer y")
    assert torch.equal(yw.cpu(), (y.cpu().float() * w.cpu().float()).to(torch.bfloat16))
    exp_ss = y.cpu().float().view(n_vec, E // 16, 16).pow(2).sum(-1)
    assert torch.allclose(ss.cpu(), exp_ss, rtol=1e-5, atol=1e-6)
    # consumer: GEMV of the RMSNorm of the producer's y
    ref = ops.gemv_multi(Wc.dequant().cpu(), ops.rms_norm(y.cpu(), w.cpu(), 1e-5))
    assert_close(out.cpu(), ref, 2e-2, 1e-2, what="consumer (folded RMSNorm)")


def test_consumer_swiglu_and_argmax():
    E, H, n_vec = 2048, 1024, 2
    g = torch.Generator(device="cuda").manual_seed(9)
    h = (4 * torch.randn(n_vec, E, device="cuda", generator=g)).to(torch.bfloat16)
    w = (1 + 0.02 * torch.randn(E, device="cuda", generator=g)).to(torch.bfloat16)
    hw = (h.float() * w.float()).to(torch.bfloat16)
    ss = h.float().view(n_vec, E // 16, 16).pow(2).sum(-1).contiguous()
    gate_up = Int4Matrix(2 * H, E, g, 0.001, 0.004, keep_natural=True)  # interleaved per 8 rows
    act = torch.empty(n_vec, H, dtype=torch.bfloat16, device="cuda")
    _chain(gate_up, hw, act, n_vec, flags=_lib.IRON_FLAG_SWIGLU, ss_in=ss, eps=1e-5)
    lm = Int4Matrix(4096, E, g, 0.001, 0.004, keep_natural=True)
    logits = torch.empty(n_vec, 4096, dtype=torch.bfloat16, device="cuda")
    keys = torch.zeros(n_vec * 32, dtype=torch.int64, device="cuda")
    tok = torch.zeros(n_vec, dtype=torch.int32, device="cuda")
    _chain(lm, hw, logits, n_vec, ss_in=ss, eps=1e-5, argmax_keys=keys)
    _lib.call("iron_argmax_finalize", keys.data_ptr(), tok.data_ptr(), None, n_vec, 0, _lib.current_stream())
    torch.cuda.synchronize()
    hn = ops.rms_norm(h.cpu(), w.cpu(), 1e-5)
    Wgu = gate_up.dequant().cpu().view(-1, 16, E)
    ref_act = ops.swiglu_act(ops.gemv_multi(Wgu[:, :8].reshape(H, E), hn), ops.gemv_multi(Wgu[:, 8:].reshape(H, E), hn))
    assert_close(act.cpu(), ref_act, 2e-2, 1e-2, what="SwiGLU after the folded RMSNorm")
    assert_close(logits.cpu(), ops.gemv_multi(lm.dequant().cpu(), hn), 2e-2, 1e-2, what="lm-head")
    got = logits.cpu().float()
    assert torch.equal(tok.cpu().long(), got.argmax(1))


def test_embed_chain():
    B, E, V = 3, 2048, 1000
    g = torch.Generator(device="cuda").manual_seed(4)
    table = torch.randn(V, E, device="cuda", generator=g).to(torch.bfloat16)
    w = (1 + 0.02 * torch.randn(E, device="cuda", generator=g)).to(torch.bfloat16)
    tokens = torch.tensor([5, V + 3, 999], dtype=torch.int32, device="cuda")  # one out of range
    x, xw = torch.empty(B, E, dtype=torch.bfloat16, device="cuda"), torch.empty(B, E, dtype=torch.bfloat16, device="cuda")
    ss = torch.empty(B, E // 16, dtype=torch.float32, device="cuda")
    _lib.call("iron_embed_chain", tokens.data_ptr(), table.data_ptr(), x.data_ptr(), xw.data_ptr(), w.data_ptr(),
              ss.data_ptr(), B, E, V, 0, _lib.current_stream())
    torch.cuda.synchronize()
    exp = torch.stack([table[5], torch.zeros(E, dtype=torch.bfloat16, device="cuda"), table[999]]).cpu()
    assert torch.equal(x.cpu(), exp)
    assert torch.equal(xw.cpu(), (exp.float() * w.cpu().float()).to(torch.bfloat16))
    assert torch.allclose(ss.cpu(), exp.float().view(B, E // 16, 16).pow(2).sum(-1), rtol=1e-5, atol=1e-6)
