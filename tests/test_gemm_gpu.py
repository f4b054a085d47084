"""Tensor-core GEMM (tcgen05 + TMEM + TMA) on the B200 against the oracle.

IRON's GEMM shapes and tolerance (iron/operators/gemm/test.py:18-210: relative
0.005 / 0.005, A ~ 4 N(0,1), B ~ 4 U[0,1)) and the flm GEMM's
(iron/operators/flm/gemm/test.py:137-200: an absolute bound that is a fraction of
the accumulated mass K mean|A| mean|B|, the fraction of a native bf16 / fp32-sum
device; relative 0.04).
"""

import numpy as np
import pytest
import torch

from helpers import assert_close, bf16, load
from oracle import ops

pytestmark = pytest.mark.gpu

from iron_b200 import _lib
from iron_b200.common.test_utils import run_test
from iron_b200.operators import GEMM
from iron_b200.operators.flm import GEMM as FlmGEMM
from iron_b200.operators.flm.gemm.design import Epilogue, Rounding


@pytest.fixture(autouse=True)
def _no_timeouts():
    _lib.load().iron_gemm_status(1)
    yield
    assert _lib.load().iron_gemm_status(1) == 0, "a GEMM hit its bounded-wait deadline"


def _inputs(M, K, N, seed=42, b_col_maj=False, scale=4.0):
    g = torch.Generator().manual_seed(seed)
    A = (torch.randn(M, K, generator=g) * scale).to(torch.bfloat16)
    B = (torch.rand(K, N, generator=g) * scale).to(torch.bfloat16)
    return A, (B.T.contiguous() if b_col_maj else B)


def _run(op, A, B):
    dev = [A.cuda(), B.cuda()]
    spec = op.get_arg_spec()[2]
    C = torch.empty(spec.shape, dtype=torch.bfloat16, device="cuda")
    op.get_callable()(dev[0], dev[1], C)
    torch.cuda.synchronize()
    return C.cpu()


# ---- iron GEMM -------------------------------------------------------------------
# M, K, N, num_aie_columns, b_col_maj, c_col_maj, m, k, n (gemm/test.py:24-56)
PARAMS = [
    (2048, 2048, 2048, 1, False, False, 64, 64, 64),
    (2048, 2048, 2048, 2, True, False, 64, 64, 64),
    (2048, 2048, 2048, 8, True, True, 64, 64, 64),
    (384, 1536, 1792, 4, True, False, 32, 48, 64),
    (1792, 896, 1152, 8, False, True, 64, 32, 48),
    (896, 1792, 640, 8, False, True, 32, 64, 80),
    (192, 384, 64, 4, False, False, 48, 96, 16),
    (192, 384, 64, 4, True, True, 48, 96, 16),
    (2048, 2048, 8192, 2, True, False, 64, 64, 64),
    (2048, 8192, 2048, 2, True, False, 64, 64, 64),
    (2048, 64, 2048, 2, False, False, 64, 64, 64),
    (2048, 2560, 10240, 8, False, False, 64, 64, 64),
]


@pytest.mark.parametrize("M,K,N,cols,bc,cc,m,k,n", PARAMS)
def test_gemm(M, K, N, cols, bc, cc, m, k, n):
    A, B = _inputs(M, K, N, b_col_maj=bc)
    op = GEMM(M=M, K=K, N=N, tile_m=m, tile_k=k, tile_n=n, num_aie_columns=cols, prio_accuracy=True,
              emulate_bf16_mmul_with_bfp16=False, b_col_maj=bc, c_col_maj=cc)
    C = _run(op, A, B)
    # IRON's 0.005 / 0.005, widened for long K where both sides' fp32 sums (in
    # different orders) carry rounding of order eps_fp32 * K mean|A| mean|B|
    mass = K * A.abs().float().mean() * B.abs().float().mean()
    assert_close(C, ops.gemm(A, B, bc, cc), 0.005, max(0.005, float(1e-6 * mass)), what=op.name)


def test_gemm_partitioned_b():
    """B split into column blocks through partition_B (gemm/test.py:155-210)."""
    M, K, N, parts = 64, 512, 256, 4
    A, B = _inputs(M, K, N * parts, b_col_maj=True)
    op = GEMM(M=M, K=K, N=N, tile_m=16, tile_k=64, tile_n=64, num_aie_columns=4, b_col_maj=True,
              emulate_bf16_mmul_with_bfp16=False)
    Bn = B.view(torch.uint16).numpy()
    parts_np = op.partition_B(Bn, parts)
    Cs = [_run(op, A, torch.from_numpy(p.copy()).view(torch.bfloat16)) for p in parts_np]
    assert_close(torch.cat(Cs, dim=1), ops.gemm(A, B, True, False), 0.005, 0.005)


@pytest.mark.parametrize("name,bc,cc,M,K,N", [("gemm_M128_K256_N64_bc0_cc0", False, False, 128, 256, 64),
                                              ("gemm_M128_K256_N64_bc1_cc0", True, False, 128, 256, 64),
                                              ("gemm_M128_K256_N64_bc1_cc1", True, True, 128, 256, 64),
                                              ("gemm_M64_K512_N256_bc0_cc1", False, True, 64, 512, 256)])
def test_gemm_golden_fixtures(name, bc, cc, M, K, N):
    d = {k: bf16(v) for k, v in load(name).items()}
    op = GEMM(M=M, K=K, N=N, tile_m=16, tile_k=64, tile_n=16, num_aie_columns=4, b_col_maj=bc, c_col_maj=cc,
              emulate_bf16_mmul_with_bfp16=False)
    errors, _, _ = run_test(op, {"A": d["A"].flatten(), "B": d["B"].flatten()}, {"C": d["C"].flatten()},
                            rel_tol=0.005, abs_tol=0.005)
    assert not errors


@pytest.mark.parametrize("block_n", [64, 128, 192, 256])
def test_gemm_tile_widths_and_ragged_m(block_n):
    """Every tile width on shapes with partial tiles in M and N."""
    M, K, N = 200, 328, 376
    A, Bt = _inputs(M, K, N, b_col_maj=True, seed=block_n)
    Ad, Bd = A.cuda(), Bt.cuda()
    C = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
    _lib.call("iron_gemm_bf16", Ad.data_ptr(), Bd.data_ptr(), C.data_ptr(), M, N, K, K, K, N, None, 0, 0, 0, 0.0, 0.0,
              block_n, 0, _lib.current_stream())
    torch.cuda.synchronize()
    assert_close(C.cpu(), ops.gemm(A, Bt, True, False), 0.005, 0.005)


def test_gemm_pdl_chain_in_graph():
    """Dependent GEMMs (C1 = A B1^T, C2 = C1 B2^T) launched with PDL inside a CUDA graph."""
    M, K, N = 1024, 1024, 1024
    g = torch.Generator().manual_seed(1)
    A = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()
    B1 = (torch.randn(N, K, generator=g) * 0.03).to(torch.bfloat16).cuda()
    B2 = (torch.randn(N, N, generator=g) * 0.03).to(torch.bfloat16).cuda()
    C1 = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    C2 = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    s = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        for X, W, Y, k in ((A, B1, C1, K), (C1, B2, C2, N)):
            _lib.call("iron_gemm_bf16", X.data_ptr(), W.data_ptr(), Y.data_ptr(), M, N, k, k, k, N, None, 0, 0, 0, 0.0,
                      0.0, 0, _lib.IRON_FLAG_PDL, s.cuda_stream)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    r1 = ops.gemm(A.cpu(), B1.cpu(), True, False)
    assert_close(C1.cpu(), r1, 0.005, 0.005, what="C1")
    assert_close(C2.cpu(), ops.gemm(C1.cpu(), B2.cpu(), True, False), 0.005, 0.005, what="C2")


def test_gemm_rejects_bad_arguments():
    lib = _lib.load()
    A = torch.zeros(128, 64, dtype=torch.bfloat16, device="cuda")
    s = _lib.current_stream()
    assert lib.iron_gemm_bf16(A.data_ptr(), A.data_ptr(), A.data_ptr(), 128, 64, 60, 64, 64, 64, None, 0, 0, 0, 0.0,
                              0.0, 0, 0, s) == _lib.IRON_ERR_SHAPE
    assert lib.iron_gemm_bf16(A.data_ptr(), A.data_ptr(), A.data_ptr(), 128, 64, 64, 64, 64, 64, None, 0, 9, 0, 0.0,
                              0.0, 0, 0, s) == _lib.IRON_ERR_ARG
    assert lib.iron_gemm_bf16(A.data_ptr(), A.data_ptr(), A.data_ptr(), 128, 64, 64, 64, 64, 64, None, 0, 0, 0, 0.0,
                              0.0, 96, 0, s) == _lib.IRON_ERR_ARG
    assert lib.iron_gemm_bf16(A.data_ptr() + 2, A.data_ptr(), A.data_ptr(), 64, 64, 64, 64, 64, 64, None, 0, 0, 0, 0.0,
                              0.0, 0, 0, s) == _lib.IRON_ERR_ALIGN


# ---- flm GEMM ------------------------------------------------------------------------
NONE, GELU, SILU, SIGMOID = Epilogue
CONV_EVEN, FLOOR = Rounding
FLM_PARAMS = [  # flm/gemm/test.py:55-86 (NPU2 regular + extensive)
    (256, 512, 1024, NONE, None, CONV_EVEN),
    (512, 1024, 2048, NONE, None, CONV_EVEN),
    (256, 512, 1536, NONE, None, CONV_EVEN),
    (256, 512, 128, NONE, None, CONV_EVEN),
    (256, 512, 1024, SILU, None, CONV_EVEN),
    (256, 512, 1024, GELU, None, CONV_EVEN),
    (256, 512, 1024, NONE, (-2.0, 2.0), CONV_EVEN),
    (256, 512, 1024, NONE, None, FLOOR),
    (2048, 2048, 2048, NONE, None, CONV_EVEN),
    (512, 1536, 1536, SILU, None, CONV_EVEN),
    (256, 512, 1024, SIGMOID, None, CONV_EVEN),
    (512, 1024, 2048, SILU, (-4.0, 4.0), CONV_EVEN),
    (2048, 10240, 2560, NONE, None, CONV_EVEN),
    (2048, 2560, 10240, NONE, None, CONV_EVEN),
]


@pytest.mark.parametrize("M,K,N,epilogue,clamp,rounding", FLM_PARAMS)
def test_flm_gemm(M, K, N, epilogue, clamp, rounding):
    scale = 4.0 if epilogue is NONE else 0.5
    A, B = _inputs(M, K, N, scale=scale)
    op = FlmGEMM(M=M, K=K, N=N, epilogue=epilogue, clamp=clamp, rounding=rounding)
    ref = ops.flm_gemm(A, B, str(epilogue), clamp)
    mass = K * A.abs().float().mean() * B.abs().float().mean()
    budget = 0.002 if rounding is FLOOR else 0.0002
    errors, _, _ = run_test(op, {"A": A.flatten(), "B": op.pack_B(B)}, {"C": ref.flatten()}, rel_tol=0.04,
                            abs_tol=float(budget * mass))
    assert not errors


@pytest.mark.parametrize("epi,clamp", [("none", None), ("silu", None), ("gelu", None), ("sigmoid", None),
                                       ("none", (-2.0, 2.0)), ("silu", (-4.0, 4.0))])
def test_flm_gemm_golden_fixtures(epi, clamp):
    tag = f"_cl{int(clamp[1])}" if clamp else ""
    d = {k: bf16(v) for k, v in load(f"flm_gemm_{epi}{tag}_M128_K512_N128").items()}
    op = FlmGEMM(M=256, K=512, N=128, epilogue=Epilogue(epi), clamp=clamp)
    pad = torch.zeros_like(d["A"])  # IRON's M unit on NPU2 is 256: pad the golden's 128 rows
    A = torch.cat([d["A"], pad])
    errors, _, _ = run_test(op, {"A": A.flatten(), "B": op.pack_B(d["B"])},
                            {"C": torch.cat([d["C"], ops.flm_gemm(pad, d["B"], epi, clamp)]).flatten()},
                            rel_tol=0.04, abs_tol=float(0.0002 * 512 * d["A"].abs().float().mean()
                                                        * d["B"].abs().float().mean()))
    assert not errors


@pytest.mark.parametrize("block_n", [0, 192])
def test_gemm_residual_epilogue(block_n):
    """C = bf16(bf16(A B^T) + R): the o_proj / down_proj residual of a decoder block
    (the chosen tile width, and 192-wide tiles with a partial last tile)."""
    M, K, N = 384, 1024, 768
    g = torch.Generator().manual_seed(11)
    A = torch.randn(M, K, generator=g).to(torch.bfloat16)
    W = (torch.randn(N, K, generator=g) * 0.03).to(torch.bfloat16)
    R = torch.randn(M, N, generator=g).to(torch.bfloat16)
    Ad, Wd, Rd = A.cuda(), W.cuda(), R.cuda()
    C = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    _lib.call("iron_gemm_bf16", Ad.data_ptr(), Wd.data_ptr(), C.data_ptr(), M, N, K, K, K, N, Rd.data_ptr(), N,
              0, 0, 0.0, 0.0, block_n, 0, _lib.current_stream())
    torch.cuda.synchronize()
    assert_close(C.cpu(), ops.add(R, ops.gemm(A, W, True, False)), 0.02, 0.01)


@pytest.mark.parametrize("block_n", [0, 192])
def test_gemm_swiglu_epilogue(block_n):
    """Interleaved gate/up rows (8 + 8 per 16) -> silu(gate) * up, N/2 outputs."""
    M, K, H = 256, 512, 1024
    g = torch.Generator().manual_seed(12)
    A = torch.randn(M, K, generator=g).to(torch.bfloat16)
    Wg = (torch.randn(H, K, generator=g) * 0.05).to(torch.bfloat16)
    Wu = (torch.randn(H, K, generator=g) * 0.05).to(torch.bfloat16)
    t = torch.arange(H // 8)
    idx = torch.stack([t * 8 + i for i in range(8)] + [H + t * 8 + i for i in range(8)], 1).reshape(-1)
    Wgu = torch.cat([Wg, Wu])[idx].contiguous()
    Ad, Wd = A.cuda(), Wgu.cuda()
    C = torch.empty(M, H, dtype=torch.bfloat16, device="cuda")
    _lib.call("iron_gemm_bf16", Ad.data_ptr(), Wd.data_ptr(), C.data_ptr(), M, 2 * H, K, K, K, H, None, 0,
              _lib.IRON_GEMM_EPI_SWIGLU, 0, 0.0, 0.0, block_n, 0, _lib.current_stream())
    torch.cuda.synchronize()
    ref = ops.swiglu_act(ops.gemm(A, Wg, True, False), ops.gemm(A, Wu, True, False))
    assert_close(C.cpu(), ref, 0.04, 1e-3)
