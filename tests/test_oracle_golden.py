"""Pin the CPU oracle to IRON's own goldens (fixtures made by golden/make_golden.py).

CPU only. Every oracle function is checked against the output IRON's reference
code produced for the same inputs: exactly for byte/index work and the fp32-
computed ops, within a bf16-rounding bound where IRON's golden computes in bf16.
"""

import numpy as np
import pytest
import torch

from helpers import assert_close, bf16, bits, load, load_kwargs
from oracle import ops, quant
from oracle import llama as ollama


@pytest.mark.parametrize("name", ["gemv_M128_K128", "gemv_M64_K256", "gemv_batched_M64_K128_b4"])
def test_gemv_matches_golden(name):
    d = load(name)
    got = ops.gemv(bf16(d["A"]), bf16(d["B"]))
    # IRON's golden is torch's bf16 matmul; ours accumulates in fp32 and rounds
    # once: the two agree to within one bf16 rounding of the output.
    assert_close(got, bf16(d["C"]), 2**-7, 1e-3, what=name)


def test_gemv_gelu_matches_golden():
    d = load("gemv_gelu_M64_K128")
    c = ops.gemv(bf16(d["A"]), bf16(d["B"]))
    got = ops.gelu_tanh(c).to(torch.bfloat16)
    assert_close(got, bf16(d["C"]), 2**-7, 1e-3, what="gelu")


@pytest.mark.parametrize("name", ["dequant_2048_t1024_g32", "dequant_4096_t4096_g32", "dequant_1024_t256_g32"])
def test_dequant_u4_bit_exact(name):
    d = load(name)
    tile = int(name.split("_t")[1].split("_")[0])
    out = quant.dequant_u4_tiles(d["payload"], tile, 32)
    np.testing.assert_array_equal(out, d["out"])
    # The oracle's packer reproduces IRON's payload byte for byte.
    repacked = quant.pack_u4_tiles(d["codes"].reshape(-1), d["scales"], tile, 32)
    np.testing.assert_array_equal(repacked, d["payload"])


def test_s4g32_roundtrip_exact():
    codes, sbits, q = quant.make_s4g32(64, 256, seed=1)
    np.testing.assert_array_equal(quant.unpack_s4(codes), q.astype(np.int8))
    deq = quant.dequant_s4g32(codes, sbits)
    expect = quant.f32_to_bf16_bits(
        q.astype(np.float32) * np.repeat(quant.bf16_bits_to_f32(sbits), 32, axis=1))
    np.testing.assert_array_equal(deq, expect)


def test_s4g32_unit_packing_roundtrip_and_nibble_order():
    """The GEMV's packed unit layout: unpacking restores codes and scales exactly, and
    a word's even / odd k sit in its low / high halves (consecutive k share a pair)."""
    codes, sbits, _ = quant.make_s4g32(64, 512, seed=3)
    units = quant.pack_s4g32_units(codes, sbits)
    assert units.size == (64 // 16) * (512 // 128) * 1152
    c2, s2 = quant.unpack_s4g32_units(units, 64, 512)
    np.testing.assert_array_equal(c2, codes)
    np.testing.assert_array_equal(s2, sbits)
    # unit (0, 0), lane 0 (row 0), word j = 0: natural k 0..7 of row 0
    w = int(units[:4].view(np.uint32)[0])
    nat = [(int(codes[0, i // 2]) >> (4 * (i % 2))) & 15 for i in range(8)]
    got = [(w >> ((16 if i % 2 else 0) + 4 * (i // 2))) & 15 for i in range(8)]
    assert got == nat


def test_f32_to_bf16_rounding_matches_torch():
    x = torch.randn(100000) * 10
    x[:5] = torch.tensor([0.0, -0.0, float("inf"), float("-inf"), 1e-40])
    np.testing.assert_array_equal(quant.f32_to_bf16_bits(x.numpy()), bits(x.to(torch.bfloat16)))


def test_rms_norm_matches_golden():
    d = load("rms_norm_w_4x256")
    got = ops.rms_norm(bf16(d["x"]), bf16(d["w"]))
    # IRON's golden squares and averages in bf16; ours in fp32.
    assert_close(got, bf16(d["out"]), 2e-2, 1e-6, what="rms_norm weighted")
    d = load("rms_norm_2x2048")
    assert_close(ops.rms_norm(bf16(d["x"])), bf16(d["out"]), 2e-2, 1e-6, what="rms_norm")


@pytest.mark.parametrize("name", ["rope_32x128_a8", "rope_32x64_a1", "rope_64x128_a32"])
def test_rope_matches_golden_exactly(name):
    d = load(name)
    x, ang = bf16(d["x"]), bf16(d["angles"])
    assert torch.equal(ops.rope(x, ang, 0), bf16(d["out0"]))
    assert torch.equal(ops.rope(x, ang, 1), bf16(d["out1"]))


def test_rope_angle_row_convention():
    """Row r uses angle row r // (rows / angle_rows)
    (iron/tests/operators/rope_reference_convention.py:21-64)."""
    for rows, arows in [(6, 3), (8, 2), (1024, 1), (4, 4), (13, 13), (12, 4)]:
        torch.manual_seed(0)
        x = torch.randn(rows, 4).to(torch.bfloat16)
        ang = torch.zeros(arows, 4, dtype=torch.bfloat16)
        ang[:, 0::2] = torch.rand(arows, 2).to(torch.bfloat16)
        ang[:, 1::2] = torch.rand(arows, 2).to(torch.bfloat16)
        exp = torch.empty(rows, 4)
        for r in range(rows):
            a = r // (rows // arows)
            c, s = ang[a, 0::2].float(), ang[a, 1::2].float()
            x1, x2 = x[r, :2].float(), x[r, 2:].float()
            exp[r, :2] = x1 * c - x2 * s
            exp[r, 2:] = x2 * c + x1 * s
        assert torch.equal(ops.rope(x, ang), exp.to(torch.bfloat16))


def test_softmax_matches_golden():
    d = load("softmax_16x512")
    assert_close(ops.softmax(bf16(d["x"])), bf16(d["out"]), 2**-7, 1e-6, what="softmax")


def test_masked_softmax_definition():
    x = torch.randn(4, 64).to(torch.bfloat16)
    got = ops.softmax(x, valid=10)
    assert torch.all(got[:, 10:] == 0)
    assert_close(got[:, :10], torch.softmax(x[:, :10].float(), -1).to(torch.bfloat16), 2**-8, 0)


@pytest.mark.parametrize("name,fn", [("silu_2048", "silu"), ("mul_2048", "mul"), ("add_2048", "add")])
def test_eltwise_matches_golden(name, fn):
    d = load(name)
    if fn == "silu":
        got = ops.silu(bf16(d["x"]))
    else:
        got = getattr(ops, fn)(bf16(d["a"]), bf16(d["b"]))
    assert_close(got, bf16(d["out"]), 2**-8, 0, what=name)


def test_swiglu_decode_chain_matches_golden():
    d = {k: bf16(v) for k, v in load("swiglu_decode_e256_h512").items()}
    x = d["input"]
    left = ops.gemv_multi(d["w_gate"].T.contiguous(), x)
    right = ops.gemv_multi(d["w_up"].T.contiguous(), x)
    assert_close(left, d["left"], 2**-7, 1e-3, what="left")
    assert_close(right, d["right"], 2**-7, 1e-3, what="right")
    # chained on the golden's own intermediates, as swiglu_decode/test.py:65-101 does
    inter = ops.swiglu_act(d["left"], d["right"])
    assert_close(inter, d["intermediate"], 0.04, 0.4, what="intermediate")
    out = ops.gemv_multi(d["w_down"].T.contiguous(), d["intermediate"])
    assert_close(out, d["output"], 0.04, 0.4, what="output")


@pytest.mark.parametrize("case", ["flat1024", "flat1024_ch4", "kv_slot0", "kv_slot5", "kv_slot_last",
                                  "kv_slot5_ch2", "kv_slot5_ch4", "kv_llama_full", "kv_addend7"])
def test_strided_copy_exact(case):
    d = load(f"strided_copy_{case}")
    kw = load_kwargs(d)
    got = ops.strided_copy(
        bf16(d["input"]), kw["input_sizes"], kw["input_strides"], kw["input_offset"],
        kw["output_buffer_size"], kw["output_sizes"], kw["output_strides"], kw["output_offset"],
        kw.get("num_aie_channels", 1), 0, kw.get("output_offset_addend", 0))
    np.testing.assert_array_equal(bits(got), d["output"])


def test_repeat_and_transpose_exact():
    d = load("repeat_8x256_r4")
    np.testing.assert_array_equal(bits(ops.repeat_interleave(bf16(d["x"]), 4)), d["out"])
    d = load("transpose_2x64x32")
    np.testing.assert_array_equal(bits(ops.transpose(bf16(d["x"]))), d["out"])


@pytest.mark.parametrize("name,S", [("mha_h2_kv1_s128", 128), ("mha_h4_kv2_s100", 100)])
def test_mha_prefill_matches_golden(name, S):
    d = load(name)
    Q, K, V = bf16(d["Q"])[:, :S], bf16(d["K"])[:, :S], bf16(d["V"])[:, :S]
    got = ops.mha_prefill(Q, K, V)
    assert_close(got, bf16(d["O"])[:, :S], 2e-2, 2e-2, what=name)


def test_rope_angles_match_harness():
    d = load("rope_angles_hd64_ctx64")
    torch.testing.assert_close(ops.rope_angles(64, 64), torch.from_numpy(d["angles"]), rtol=0, atol=0)


def test_llama_block_decode_matches_llama_cpu():
    d = load("llama_block_decode_small")
    emb, nh, nkv, hd, hid, past = (int(v) for v in d["dims"])
    W = {k[2:]: bf16(v) for k, v in d.items() if k.startswith("W_")}
    Lmax = past + 4
    kc = torch.zeros(1, nkv, Lmax, hd, dtype=torch.bfloat16)
    vc = torch.zeros(1, nkv, Lmax, hd, dtype=torch.bfloat16)
    kc[:, :, :past] = bf16(d["kc"])
    vc[:, :, :past] = bf16(d["vc"])
    x = bf16(d["x"]).reshape(1, emb)
    angles = torch.from_numpy(d["angles"])
    y = ollama.block_decode(x, kc, vc, [past], W, angles, nh, nkv, hd)
    # fp32 golden vs a bf16-rounded pipeline
    assert_close(y, bf16(d["y"]).reshape(1, emb), 2e-2, 2e-2, what="block output")
    assert_close(kc[:, :, : past + 1], bf16(d["k_new"]), 2e-2, 2e-2, what="k cache")
    assert_close(vc[:, :, : past + 1], bf16(d["v_new"]), 2e-2, 2e-2, what="v cache")


# ---- GEMM (iron/operators/gemm/reference.py, flm/gemm/reference.py) ------------------
@pytest.mark.parametrize("name,bc,cc", [("gemm_M128_K256_N64_bc0_cc0", False, False),
                                        ("gemm_M128_K256_N64_bc1_cc0", True, False),
                                        ("gemm_M128_K256_N64_bc1_cc1", True, True),
                                        ("gemm_M64_K512_N256_bc0_cc1", False, True)])
def test_gemm_matches_golden(name, bc, cc):
    d = {k: bf16(v) for k, v in load(name).items()}
    got = ops.gemm(d["A"], d["B"], bc, cc)
    # IRON's golden runs torch's bf16 matmul; both accumulate in fp32 and round once
    assert_close(got, d["C"], 0.005, 0.005, what=name)
    assert (got.view(torch.int16) == d["C"].view(torch.int16)).float().mean() > 0.99


@pytest.mark.parametrize("epi,clamp", [("none", None), ("silu", None), ("gelu", None), ("sigmoid", None),
                                       ("none", (-2.0, 2.0)), ("silu", (-4.0, 4.0))])
def test_flm_gemm_matches_golden(epi, clamp):
    tag = f"_cl{int(clamp[1])}" if clamp else ""
    d = {k: bf16(v) for k, v in load(f"flm_gemm_{epi}{tag}_M128_K512_N128").items()}
    got = ops.flm_gemm(d["A"], d["B"], epi, clamp)
    assert_close(got, d["C"], 0.005, 0.005, what=epi)


@pytest.mark.parametrize("name", ["q4nx_K1024_N128", "q4nx_K512_N192"])
def test_q4nx_restatement_matches_iron(name):
    """The q4nx block walk restated in oracle/quant.py gives IRON's own dequantized values
    bit for bit (fixture from iron/operators/flm/dequant/reference.py: random_q4nx and
    dequantize), and its inverse rebuilds the blob byte for byte."""
    from oracle import quant

    d = load(name)
    K, N = (int(v) for v in d["dims"])
    codes, sbits, mbits = quant.q4nx_to_natural(d["blob"], K, N)
    assert np.array_equal(quant.q4nx_dequant(codes, sbits, mbits), d["w"])
    assert np.array_equal(quant.q4nx_from_natural(codes, sbits, mbits), d["blob"])


@pytest.mark.parametrize("name", ["q4nx_K1024_N128", "q4nx_K512_N192"])
def test_q4nx_importer_matches_restatement(name):
    """The product's q4nx importer (torch index arithmetic, run here on the CPU) yields the
    restatement's natural arrays: codes two per byte, bf16 scales and mins."""
    from iron_b200.operators.gemv.q4nx import q4nx_natural
    from oracle import quant

    d = load(name)
    K, N = (int(v) for v in d["dims"])
    codes, scales, mins = q4nx_natural(torch.from_numpy(d["blob"]), K, N)
    oc, osb, omb = quant.q4nx_to_natural(d["blob"], K, N)
    assert np.array_equal(codes.numpy(), (oc[:, 0::2] | (oc[:, 1::2] << 4)).astype(np.uint8))
    assert np.array_equal(scales.view(torch.int16).numpy().view(np.uint16), osb)
    assert np.array_equal(mins.view(torch.int16).numpy().view(np.uint16), omb)
