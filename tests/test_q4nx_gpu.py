"""The q4 GEMV on IRON's asymmetric int4 weights (q4nx: min + scale * code) against the
oracle: the blob restated in oracle/quant.py (pinned to IRON's flm/dequant golden by
tests/test_oracle_golden.py), dequantized in fp32 as iron/operators/flm/dequant/
reference.py:40-77 does, rounded once to bf16, then IRON's GEMV golden
(iron/operators/gemv/reference.py:9-11, fp32 accumulate). The weights the kernel
multiplies are checked bit for bit (iron_unpack_q4g32); the GEMV at rtol 2e-2 / atol 1e-2."""

import numpy as np
import pytest
import torch

from helpers import assert_close, load
from oracle import ops, quant

pytestmark = pytest.mark.gpu

from iron_b200 import _lib
from iron_b200.operators import GEMV


def _random_blob(K, N, seed):
    rng = np.random.default_rng(seed)
    codes = rng.integers(0, 16, (N, K), dtype=np.uint8)
    sb = quant.f32_to_bf16_bits(rng.uniform(0.002, 0.05, (N, K // 32)).astype(np.float32))
    mb = quant.f32_to_bf16_bits(rng.uniform(-0.4, 0.4, (N, K // 32)).astype(np.float32))
    return quant.q4nx_from_natural(codes, sb, mb)


def _blob(case):
    if isinstance(case, str):
        d = load(case)
        K, N = (int(v) for v in d["dims"])
        return d["blob"], K, N
    K, N, seed = case
    return _random_blob(K, N, seed), K, N


@pytest.mark.parametrize("case,n_vec", [("q4nx_K1024_N128", 1), ("q4nx_K512_N192", 3), ((2048, 8192, 5), 1),
                                        ((2048, 8192, 6), 8), ((8192, 2048, 7), 2)])
def test_q4nx_gemv_matches_oracle(case, n_vec):
    blob, K, N = _blob(case)
    w32 = quant.q4nx_dequant(*quant.q4nx_to_natural(blob, K, N))
    wb = torch.from_numpy(w32).to(torch.bfloat16)  # the one rounding to bf16 (nearest even)
    packed = GEMV.pack_q4nx(torch.from_numpy(blob).cuda(), K, N)
    # the weights the kernel multiplies, bit for bit
    got_w = torch.empty(N, K, dtype=torch.bfloat16, device="cuda")
    _lib.call("iron_unpack_q4g32", packed.data_ptr(), got_w.data_ptr(), N, K, _lib.current_stream())
    g = torch.Generator().manual_seed(N + K + n_vec)
    x = torch.randn(n_vec, K, generator=g).to(torch.bfloat16)
    res = torch.randn(n_vec, N, generator=g).to(torch.bfloat16)
    y = torch.empty(n_vec, N, dtype=torch.bfloat16, device="cuda")
    yr = torch.empty_like(y)
    xd, rd = x.cuda(), res.cuda()  # held: the kernels read them after the calls return
    op = GEMV(M=N, K=K, weight_dtype="q4nx", n_vec=n_vec)
    op.get_callable()(packed, xd, y)
    _lib.call("iron_gemv_q4g32", packed.data_ptr(), xd.data_ptr(), yr.data_ptr(), N, K, n_vec, rd.data_ptr(), 0,
              _lib.current_stream())
    torch.cuda.synchronize()
    assert torch.equal(got_w.cpu().view(torch.int16), wb.view(torch.int16)), "dequantized q4nx weights differ"
    ref = ops.gemv_multi(wb, x)
    assert_close(y.cpu(), ref, 2e-2, 1e-2, what=f"q4nx GEMV {case}")
    assert_close(yr.cpu(), ops.add(ref, res), 2e-2, 1e-2, what=f"q4nx GEMV + residual {case}")


def test_q4nx_rejects_bad_shapes():
    with pytest.raises(ValueError):
        GEMV(M=100, K=1024, weight_dtype="q4nx")
    with pytest.raises(ValueError):
        GEMV(M=128, K=1000, weight_dtype="q4nx")
    assert _lib.load().iron_gemv_q4g32(16, 16, 16, 128, 1024, 9, None, 0, None) == -2  # > 8 vectors
