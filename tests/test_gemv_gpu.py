"""GEMV (bf16 and int4-g32) and Dequant on the B200 against the CPU oracle.

Shapes follow IRON's own tests (iron/operators/gemv/test.py:20-41, :83-98,
iron/operators/dequant/test.py:13-55) and BASELINE configs 1-2. Tolerances:
IRON's GEMV bar rel 0.04 / abs 1e-3 (gemv/test.py:69-71) for bf16; the north
star's rtol 2e-2 / atol 1e-2 for the int4 GEMV; exact for dequantized weights.
"""

import numpy as np
import pytest
import torch

from helpers import assert_close, bf16, bits, load
from oracle import ops, quant

pytestmark = pytest.mark.gpu

from iron_b200 import _lib
from iron_b200.common.test_utils import run_test
from iron_b200.operators import GEMV, Dequant


def _golden_like(M, K, seed=42, b=None):
    """The input distribution of gemv/reference.py:28-36 (randn * 4, bf16)."""
    torch.manual_seed(seed)
    if b is None:
        return torch.randn(M, K, dtype=torch.bfloat16) * 4, torch.randn(K, dtype=torch.bfloat16) * 4
    return (torch.randn(b, M, K, dtype=torch.bfloat16) * 4,
            torch.randn(b, K, dtype=torch.bfloat16) * 4)


@pytest.mark.parametrize("name", ["gemv_M128_K128", "gemv_M64_K256"])
def test_gemv_golden_fixture(name):
    d = load(name)
    A, B, C = bf16(d["A"]), bf16(d["B"]), bf16(d["C"])
    op = GEMV(M=A.shape[0], K=A.shape[1])
    errors, _, _ = run_test(op, {"matrix": A, "vector": B}, {"output": C}, rel_tol=0.04, abs_tol=1e-3)
    assert not errors


@pytest.mark.parametrize("M,K", [(128, 128), (2048, 8192), (8192, 2048), (512, 2048), (2048, 2048),
                                 (128256 // 8, 2048), (40, 96), (1026, 64)])
def test_gemv_bf16_shapes(M, K):
    A, B = _golden_like(M, K)
    C = ops.gemv(A, B)
    errors, lat, bw = run_test(GEMV(M=M, K=K), {"matrix": A, "vector": B}, {"output": C},
                               rel_tol=0.04, abs_tol=1e-3)
    assert not errors


@pytest.mark.parametrize("M,K,nb", [(256, 128, 4), (256, 128, 100), (448, 64, 192), (64, 1536, 8),
                                    (1026, 64, 2), (1024, 1024, 2), (512, 64, 32), (2048, 64, 32),
                                    (64, 2048, 32)])
def test_gemv_batched(M, K, nb):
    A, B = _golden_like(M, K, b=nb)
    C = ops.gemv(A, B)
    errors, _, _ = run_test(GEMV(M=M, K=K, num_batches=nb),
                            {"matrix": A.flatten(), "vector": B.flatten()},
                            {"output": C.flatten()}, rel_tol=0.04, abs_tol=1e-3)
    assert not errors


def test_gemv_gelu_fixture():
    d = load("gemv_gelu_M64_K128")
    op = GEMV(M=64, K=128, epilogue="gelu", tile_size_input=16, tile_size_output=16)
    errors, _, _ = run_test(op, {"matrix": bf16(d["A"]), "vector": bf16(d["B"])},
                            {"output": bf16(d["C"])}, rel_tol=0.06, abs_tol=2e-2)
    assert not errors


@pytest.mark.parametrize("n_vec", [1, 2, 7, 8, 9, 16, 33, 64])
def test_gemv_decode_batch(n_vec):
    torch.manual_seed(n_vec)
    M, K = 2048, 2048
    A = (torch.randn(M, K) * 0.02).to(torch.bfloat16)
    X = torch.randn(n_vec, K).to(torch.bfloat16)
    op = GEMV(M=M, K=K, n_vec=n_vec)
    errors, _, _ = run_test(op, {"matrix": A, "vector": X}, {"output": ops.gemv_multi(A, X)},
                            rel_tol=2e-2, abs_tol=1e-2)
    assert not errors


def test_gemv_residual_epilogue():
    torch.manual_seed(3)
    M, K, nv = 2048, 8192, 4
    A = (torch.randn(M, K) * 0.02).to(torch.bfloat16).cuda()
    X = torch.randn(nv, K).to(torch.bfloat16).cuda()
    R = torch.randn(nv, M).to(torch.bfloat16).cuda()
    Y = torch.empty(nv, M, dtype=torch.bfloat16, device="cuda")
    op = GEMV(M=M, K=K, n_vec=nv)
    op._launch(A, X, Y, stream=_lib.current_stream(), residual=R)
    exp = ops.add(ops.gemv_multi(A.cpu(), X.cpu()), R.cpu())
    assert_close(Y.cpu(), exp, 2e-2, 1e-2, what="gemv+residual")


# ---- int4 group-32 --------------------------------------------------------------
def _s4_case(N, K, nv, seed=42):
    codes, sbits, _ = quant.make_s4g32(N, K, seed=seed)
    torch.manual_seed(seed)
    X = torch.randn(nv, K).to(torch.bfloat16)
    W = bf16(quant.dequant_s4g32(codes, sbits))
    return torch.from_numpy(codes), bf16(sbits), X, W


@pytest.mark.parametrize("N,K", [(8192, 2048), (2048, 8192), (16, 128), (512, 2048), (128256 // 4, 2048)])
def test_dequant_s4g32_rows_bit_exact(N, K):
    codes, scales, _, W = _s4_case(N, K, 1)
    out = torch.empty(N, K, dtype=torch.bfloat16, device="cuda")
    c, s = codes.cuda(), scales.cuda()  # keep the device copies alive until the kernel ran
    _lib.call("iron_dequant_s4g32_rows", c.data_ptr(), s.data_ptr(), out.data_ptr(), N, K,
              _lib.current_stream())
    torch.cuda.synchronize()
    np.testing.assert_array_equal(bits(out), bits(W))


@pytest.mark.parametrize("N,K", [(8192, 2048), (16, 128), (2048, 8192), (14336, 4096)])
def test_pack_int4g32_matches_oracle_packer(N, K):
    codes, scales, _, _ = _s4_case(N, K, 1)
    c, s = codes.cuda(), scales.cuda()
    packed = GEMV.pack_int4g32(c, s)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(packed.cpu().numpy(),
                                  quant.pack_s4g32_units(codes.numpy(), bits(scales)))


@pytest.mark.parametrize("N,K,nv", [(8192, 2048, 1), (8192, 2048, 4), (8192, 2048, 8), (16, 128, 1),
                                    (2048, 8192, 1), (512, 2048, 3), (8192, 2048, 16), (2048, 2048, 64),
                                    (14336, 4096, 1), (128256, 2048, 1), (3072, 2048, 5), (32, 1024, 9)])
def test_gemv_int4g32(N, K, nv):
    codes, scales, X, W = _s4_case(N, K, nv)
    op = GEMV(M=N, K=K, weight_dtype="int4g32", n_vec=nv)
    packed = GEMV.pack_int4g32(codes.cuda(), scales.cuda()).cpu()
    vec = X if nv > 1 else X[0]
    exp = ops.gemv_multi(W, X) if nv > 1 else ops.gemv(W, X[0])
    errors, _, _ = run_test(op, {"packed": packed, "vector": vec}, {"output": exp},
                            rel_tol=2e-2, abs_tol=1e-2)
    assert not errors


def test_gemv_int4g32_residual_and_determinism():
    N, K, nv = 8192, 2048, 2
    codes, scales, X, W = _s4_case(N, K, nv, seed=5)
    R = torch.randn(nv, N).to(torch.bfloat16)
    x, r = X.cuda(), R.cuda()
    packed = GEMV.pack_int4g32(codes.cuda(), scales.cuda())
    outs = []
    for _ in range(3):
        y = torch.empty(nv, N, dtype=torch.bfloat16, device="cuda")
        _lib.call("iron_gemv_int4g32", packed.data_ptr(), x.data_ptr(), y.data_ptr(), N, K, nv,
                  r.data_ptr(), 0, _lib.current_stream())
        outs.append(y.cpu())
    assert all(torch.equal(outs[0], o) for o in outs[1:]), "int4 GEMV not bitwise deterministic"
    assert_close(outs[0], ops.add(ops.gemv_multi(W, X), R), 2e-2, 1e-2, what="int4+residual")


def test_gemv_int4g32_pdl_chain_in_graph():
    """A CUDA graph of PDL-launched GEMVs over different weights gives the same
    results as plain launches (weights streamed before the dependency wait)."""
    N, K = 2048, 2048
    outs_ref, mats = [], []
    for i in range(4):
        codes, scales, X, W = _s4_case(N, K, 1, seed=20 + i)
        mats.append(GEMV.pack_int4g32(codes.cuda(), scales.cuda()))
    x = torch.randn(K).to(torch.bfloat16).cuda()
    ys = [torch.empty(N, dtype=torch.bfloat16, device="cuda") for _ in mats]
    for m, y in zip(mats, ys):
        _lib.call("iron_gemv_int4g32", m.data_ptr(), x.data_ptr(), y.data_ptr(), N, K, 1, None,
                  0, _lib.current_stream())
    ref = [y.clone() for y in ys]
    s = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for m, y in zip(mats, ys):
            _lib.call("iron_gemv_int4g32", m.data_ptr(), x.data_ptr(), y.data_ptr(), N, K, 1, None,
                      _lib.IRON_FLAG_PDL, s.cuda_stream)
    for y in ys:
        y.zero_()
    g.replay()
    torch.cuda.synchronize()
    for a, b in zip(ys, ref):
        assert torch.equal(a, b)


# ---- Dequant (IRON uint4 tiles) -----------------------------------------------
@pytest.mark.parametrize("name,tile", [("dequant_2048_t1024_g32", 1024), ("dequant_4096_t4096_g32", 4096),
                                       ("dequant_1024_t256_g32", 256)])
def test_dequant_golden_bit_exact(name, tile):
    d = load(name)
    size = len(d["out"])
    op = Dequant(size=size, num_aie_columns=1, num_channels=1, tile_size=tile)
    errors, _, _ = run_test(op, {"payload": torch.from_numpy(d["payload"])},
                            {"output": bf16(d["out"])}, rel_tol=0.0, abs_tol=0.0)
    assert not errors


def test_dequant_bench_size_bit_exact():
    size, tile = 1 << 23, 4096
    rng = np.random.default_rng(0)
    codes = rng.integers(0, 16, size=size, dtype=np.uint8)
    sb = quant.f32_to_bf16_bits(rng.uniform(0.25, 1.0, size=size // 32).astype(np.float32))
    payload = quant.pack_u4_tiles(codes, sb, tile, 32)
    exp = quant.dequant_u4_tiles(payload, tile, 32)
    op = Dequant(size=size, num_aie_columns=8, num_channels=2, tile_size=tile)
    errors, _, _ = run_test(op, {"payload": torch.from_numpy(payload)}, {"output": bf16(exp)},
                            rel_tol=0.0, abs_tol=0.0)
    assert not errors


# ---- int4 GEMV: the Llama-3-8B tensor-parallel shards and ragged / tiny cases ----------
def _s4_ex(packed, x, N, K, nv, flags, residual=None, norm_w=None, swiglu=False):
    y = torch.empty(nv, N // 2 if swiglu else N, dtype=torch.bfloat16, device="cuda")
    f = flags | (_lib.IRON_FLAG_SWIGLU if swiglu else 0)
    _lib.call("iron_gemv_int4g32_ex", packed.data_ptr(), x.data_ptr(), y.data_ptr(), N, K, nv,
              residual.data_ptr() if residual is not None else None,
              norm_w.data_ptr() if norm_w is not None else None, 1e-5, None, f, _lib.current_stream())
    return y


# the Llama-3.2-1B projections, the Llama-3-8B tensor-parallel shards (o / down / qkv at
# tp 2 and 8), tiny and ragged cases
@pytest.mark.parametrize("N,K,nv", [(2048, 8192, 2), (16384, 2048, 1), (16, 128, 8), (48, 256, 3),
                                    (1024, 128, 5), (4096, 512, 2), (4096, 1792, 2), (768, 4096, 2),
                                    (4096, 7168, 1)])
def test_gemv_int4g32_shards(N, K, nv):
    codes, scales, X, W = _s4_case(N, K, nv, seed=N + K + nv)
    packed = GEMV.pack_int4g32(codes.cuda(), scales.cuda())
    x = X.cuda()
    y = _s4_ex(packed, x, N, K, nv, 0)
    y2 = _s4_ex(packed, x, N, K, nv, 0)
    torch.cuda.synchronize()
    assert torch.equal(y, y2), "not bitwise deterministic"
    assert_close(y.cpu(), ops.gemv_multi(W, X), 2e-2, 1e-2, what=f"{N}x{K} n_vec={nv}")


def test_gemv_int4g32_epilogues():
    """Residual add, the SwiGLU of interleaved gate/up rows and the RMSNorm prologue,
    against the oracle."""
    N, K, nv = 4096, 2048, 3
    codes, scales, X, W = _s4_case(N, K, nv, seed=11)
    packed = GEMV.pack_int4g32(codes.cuda(), scales.cuda())
    R = torch.randn(nv, N).to(torch.bfloat16)
    y = _s4_ex(packed, X.cuda(), N, K, nv, 0, residual=R.cuda())
    gu = _s4_ex(packed, X.cuda(), N, K, nv, 0, swiglu=True)
    w = (1 + 0.02 * torch.randn(K)).to(torch.bfloat16)
    yn = _s4_ex(packed, X.cuda(), N, K, nv, 0, norm_w=w.cuda())
    torch.cuda.synchronize()
    assert_close(y.cpu(), ops.add(ops.gemv_multi(W, X), R), 2e-2, 1e-2, what="residual")
    full = ops.gemv_multi(W, X).reshape(nv, N // 16, 16)
    gate, up = full[:, :, :8].reshape(nv, N // 2), full[:, :, 8:].reshape(nv, N // 2)
    assert_close(gu.cpu(), ops.swiglu_act(gate, up), 2e-2, 1e-2, what="swiglu")
    assert_close(yn.cpu(), ops.gemv_multi(W, ops.rms_norm(X, w, 1e-5)), 2e-2, 1e-2, what="rmsnorm prologue")


def test_gemv_int4g32_dependent_chain_in_graph():
    """PDL-launched GEMVs captured in a graph, each reading the previous
    one's output (the dependency the early weight copies must not break)."""
    N = K = 2048
    mats, Ws = [], []
    for i in range(6):
        codes, scales, _, W = _s4_case(N, K, 1, seed=40 + i)
        mats.append(GEMV.pack_int4g32(codes.cuda(), scales.cuda()))
        Ws.append(W)
    x0 = (torch.randn(1, K) * 0.5).to(torch.bfloat16)
    bufs = [x0.cuda()] + [torch.empty(1, N, dtype=torch.bfloat16, device="cuda") for _ in mats]
    s = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for i, m in enumerate(mats):
            _lib.call("iron_gemv_int4g32", m.data_ptr(), bufs[i].data_ptr(), bufs[i + 1].data_ptr(), N, K, 1,
                      None, _lib.IRON_FLAG_PDL, s.cuda_stream)
    g.replay()
    torch.cuda.synchronize()
    ref = x0
    for i, W in enumerate(Ws):
        # the oracle fed with the kernel's own previous output, so errors do not compound
        ref = ops.gemv_multi(W, bufs[i].cpu())
        assert_close(bufs[i + 1].cpu(), ref, 2e-2, 1e-2, what=f"link {i}")
