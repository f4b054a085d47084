"""Generate the golden fixtures in tests/golden/ by running IRON's own goldens.

Run from the repository root in a checkout that has the reference next to it:

    python tests/golden/make_golden.py /path/to/IRON

Each IRON golden module (``iron/operators/<op>/reference.py``,
``iron/applications/llama_3.2_1b/llama_cpu.py``) is loaded by file path and run
at small, seeded sizes; inputs and outputs are saved as ``<case>.npz`` (bf16 as
uint16 bit patterns). The fixtures are committed, so tests never need the
reference at run time.

``iron/operators/dequant/reference.py`` imports ``expand_ref`` from the absent
third-party package ``mlir_aie`` (pinned ``1.4.4.dev53+gd53582d`` in IRON's
requirements.txt). Only its packer ``generate_inputs`` is used here, with that
import satisfied by a stub that refuses to run; the expected output is rebuilt
from the same seeded quantization steps the packer performs
(dequant/reference.py:32-64), so the fixture pins both the byte layout and the
arithmetic.
"""

from __future__ import annotations

import importlib.util
import sys
import types
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent


def _load(ref: Path, rel: str, name: str):
    spec = importlib.util.spec_from_file_location(name, ref / rel)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _np(t):
    if isinstance(t, torch.Tensor):
        t = t.detach().contiguous()
        if t.dtype == torch.bfloat16:
            return t.view(torch.uint16).numpy().copy()
        return t.numpy().copy()
    return np.asarray(t)


def _save(name, **arrays):
    np.savez_compressed(OUT / f"{name}.npz", **{k: _np(v) for k, v in arrays.items()})
    print("wrote", name)


def main(ref: Path):
    ops = ref / "iron" / "operators"

    g = _load(ref, "iron/operators/gemv/reference.py", "ref_gemv")
    for M, K in [(128, 128), (64, 256)]:
        d = g.generate_golden_reference(M=M, K=K)
        _save(f"gemv_M{M}_K{K}", A=d["A"], B=d["B"], C=d["C"])
    d = g.generate_golden_reference_batched(M=64, K=128, num_batches=4)
    _save("gemv_batched_M64_K128_b4", A=d["A"], B=d["B"], C=d["C"])
    d = g.generate_golden_reference(M=64, K=128)
    c_gelu = torch.from_numpy(g.gelu_tanh_approx(d["C"].float().numpy()).astype(np.float32))
    _save("gemv_gelu_M64_K128", A=d["A"], B=d["B"], C=c_gelu.to(torch.bfloat16))

    # Dequant: the packer needs `aie.iron.kernels.datamovement.expand_ref` importable.
    stub = types.ModuleType("aie.iron.kernels.datamovement")

    def _refuse(*a, **k):
        raise RuntimeError("expand_ref (mlir_aie) is not available here")

    stub.expand_ref = _refuse
    for mname in ("aie", "aie.iron", "aie.iron.kernels"):
        sys.modules.setdefault(mname, types.ModuleType(mname))
    sys.modules["aie.iron.kernels.datamovement"] = stub
    dq = _load(ref, "iron/operators/dequant/reference.py", "ref_dequant")
    for length, tile, group in [(2048, 1024, 32), (4096, 4096, 32), (1024, 256, 32)]:
        payload = dq.generate_inputs(input_length=length, tile_size=tile, group_size=group)
        # Same seeded steps as the packer (dequant/reference.py:32-64).
        torch.manual_seed(42)
        nt, ns = length // tile, tile // group
        A = torch.rand(nt * ns, group, dtype=torch.bfloat16) * 3.75
        r1 = 1 / 3.75
        scales = r1 + (1 - r1) * torch.rand(nt * ns, dtype=torch.bfloat16)
        q = torch.quantize_per_channel(
            A.to(torch.float32), scales=scales.to(torch.float32),
            zero_points=torch.zeros(nt * ns), axis=0, dtype=torch.quint8,
        ).int_repr()
        expected = (q.to(torch.float32) * scales.to(torch.float32)[:, None]).to(torch.bfloat16)
        _save(f"dequant_{length}_t{tile}_g{group}", payload=payload, codes=q.to(torch.uint8),
              scales=scales, out=expected.reshape(-1))

    rn = _load(ref, "iron/operators/rms_norm/reference.py", "ref_rms")
    x, w = rn.generate_inputs(rows=4, cols=256, weighted=True)
    _save("rms_norm_w_4x256", x=x, w=w, out=rn.reference(x, w=w, weighted=True))
    (x,) = rn.generate_inputs(rows=2, cols=2048)
    _save("rms_norm_2x2048", x=x, out=rn.reference(x))

    rp = _load(ref, "iron/operators/rope/reference.py", "ref_rope")
    for rows, cols, arows in [(32, 128, 8), (32, 64, 1), (64, 128, 32)]:
        x, ang = rp.generate_inputs(rows=rows, cols=cols, context_len=arows)
        _save(f"rope_{rows}x{cols}_a{arows}", x=x, angles=ang,
              out0=rp.reference(x, ang, 0), out1=rp.reference(x, ang, 1))

    sm = _load(ref, "iron/operators/softmax/reference.py", "ref_softmax")
    x = sm.generate_inputs(rows=16, cols=512)
    _save("softmax_16x512", x=x, out=sm.reference(x))

    si = _load(ref, "iron/operators/silu/reference.py", "ref_silu")
    x = si.generate_inputs(2048)
    _save("silu_2048", x=x, out=si.reference(x))
    mu = _load(ref, "iron/operators/elementwise_mul/reference.py", "ref_mul")
    a, b = mu.generate_inputs(2048)
    _save("mul_2048", a=a, b=b, out=mu.reference(a, b))
    ad = _load(ref, "iron/operators/elementwise_add/reference.py", "ref_add")
    a, b = ad.generate_inputs(2048)
    _save("add_2048", a=a, b=b, out=ad.reference(a, b))

    sw = _load(ref, "iron/operators/swiglu_decode/reference.py", "ref_swiglu")
    d = sw.generate_golden_reference(M=1, K=256, N=512)
    _save("swiglu_decode_e256_h512", **{k: v for k, v in d.items()})

    sc = _load(ref, "iron/operators/strided_copy/reference.py", "ref_sc")
    N_KV, HD = 8, 64

    def kv(seq, slot, ch=1):
        return dict(input_sizes=[N_KV, HD], input_strides=[HD, 1], input_offset=0,
                    input_buffer_size=N_KV * HD, output_sizes=[1, N_KV, HD],
                    output_strides=[0, seq * HD, 1], output_offset=slot * HD,
                    output_buffer_size=N_KV * seq * HD, num_aie_channels=ch)

    def flat(n, ch=1):
        return dict(input_sizes=[n], input_strides=[1], input_offset=0, input_buffer_size=n,
                    output_sizes=[n], output_strides=[1], output_offset=0,
                    output_buffer_size=n, num_aie_channels=ch)

    cases = {"flat1024": flat(1024), "flat1024_ch4": flat(1024, 4),
             "kv_slot0": kv(128, 0), "kv_slot5": kv(128, 5), "kv_slot_last": kv(128, 127),
             "kv_slot5_ch2": kv(128, 5, 2), "kv_slot5_ch4": kv(128, 5, 4),
             "kv_llama_full": kv(2048, 1000)}
    import json
    for cname, kw in cases.items():
        dd = sc.generate_golden_reference(**kw)
        _save(f"strided_copy_{cname}", input=dd["input"], output=dd["output"],
              kwargs=np.frombuffer(json.dumps(kw).encode(), dtype=np.uint8))
    kw = kv(128, 0)
    dd = sc.generate_golden_reference(**kw, output_offset_addend=7 * HD, seed=3)
    _save("strided_copy_kv_addend7", input=dd["input"], output=dd["output"],
          kwargs=np.frombuffer(json.dumps(dict(kw, output_offset_addend=7 * HD)).encode(), dtype=np.uint8))

    rep = _load(ref, "iron/operators/repeat/reference.py", "ref_repeat")
    x = rep.generate_inputs(8, 256)
    _save("repeat_8x256_r4", x=x, out=rep.reference(x, 4))
    tr = _load(ref, "iron/operators/transpose/reference.py", "ref_tr")
    x = tr.generate_inputs(64, 32, num_batches=2)
    _save("transpose_2x64x32", x=x, out=tr.reference(x).contiguous())

    mh = _load(ref, "iron/operators/mha/reference.py", "ref_mha")
    d = mh.generate_golden_reference(heads=2, S_q=128, S_kv=128, d=64, num_kv_heads=1)
    _save("mha_h2_kv1_s128", Q=d["Q"], K=d["K"], V=d["V"], O=d["O"])
    d = mh.generate_golden_reference(heads=4, S_q=100, S_kv=100, d=64, num_kv_heads=2)
    _save("mha_h4_kv2_s100", Q=d["Q"], K=d["K"], V=d["V"], O=d["O"])

    # Llama decode block at reduced width through llama_cpu's own functions.
    app = ref / "iron" / "applications" / "llama_3.2_1b"
    sys.path.insert(0, str(app))
    harness = _load(ref, "iron/applications/llama_3.2_1b/llama_inference_harness.py", "llama_inference_harness")
    sys.modules["llama_inference_harness"] = harness
    lc = _load(ref, "iron/applications/llama_3.2_1b/llama_cpu.py", "ref_llama_cpu")
    angles = harness.compute_rope_angles(64, 64, 500000.0)
    _save("rope_angles_hd64_ctx64", angles=angles)
    torch.manual_seed(7)
    emb, nh, nkv, hd, hid, past = 256, 4, 2, 64, 512, 9
    W = {
        "n1": 1 + 0.02 * torch.randn(emb), "q": 0.02 * torch.randn(nh * hd, emb),
        "k": 0.02 * torch.randn(nkv * hd, emb), "v": 0.02 * torch.randn(nkv * hd, emb),
        "o": 0.02 * torch.randn(emb, nh * hd), "n2": 1 + 0.02 * torch.randn(emb),
        "g": 0.02 * torch.randn(hid, emb), "u": 0.02 * torch.randn(hid, emb),
        "d": 0.02 * torch.randn(emb, hid),
    }
    W = {k: v.to(torch.bfloat16) for k, v in W.items()}
    x = torch.randn(1, 1, emb).to(torch.bfloat16)
    kc = torch.randn(1, nkv, past, hd).to(torch.bfloat16)
    vc = torch.randn(1, nkv, past, hd).to(torch.bfloat16)
    Wf = {k: v.float() for k, v in W.items()}
    y, k2, v2 = lc.transformer_block_forward(
        x.float(), kc.float(), vc.float(), nh, nkv, Wf["n1"], Wf["q"], Wf["k"], Wf["v"],
        Wf["o"], Wf["n2"], Wf["g"], Wf["u"], Wf["d"], angles.float(), None)
    _save("llama_block_decode_small", x=x, kc=kc, vc=vc, angles=angles,
          **{f"W_{k}": v for k, v in W.items()}, y=y.to(torch.bfloat16),
          k_new=k2.to(torch.bfloat16), v_new=v2.to(torch.bfloat16),
          dims=np.array([emb, nh, nkv, hd, hid, past]))


def gemm_fixtures(ref: Path):
    """GEMM goldens: iron/operators/gemm/reference.py as is, and the flm GEMM
    golden (flm/gemm/reference.py), whose import of its design module (which
    needs mlir_aie) is satisfied by a module holding only the Epilogue enum with
    IRON's member names and order."""
    gm = _load(ref, "iron/operators/gemm/reference.py", "ref_gemm")
    for M, K, N, bc, cc in [(128, 256, 64, False, False), (128, 256, 64, True, False),
                            (128, 256, 64, True, True), (64, 512, 256, False, True)]:
        d = gm.generate_golden_reference(M=M, K=K, N=N, b_col_maj=bc, c_col_maj=cc)
        _save(f"gemm_M{M}_K{K}_N{N}_bc{int(bc)}_cc{int(cc)}", A=d["input"], B=d["input_b"][0],
              C=d["output"][0])

    import enum

    class Epilogue(enum.StrEnum):
        NONE = "none"
        GELU = "gelu"
        SILU = "silu"
        SIGMOID = "sigmoid"

    for mname in ("iron", "iron.operators", "iron.operators.flm", "iron.operators.flm.gemm"):
        sys.modules.setdefault(mname, types.ModuleType(mname))
    design = types.ModuleType("iron.operators.flm.gemm.design")
    design.Epilogue = Epilogue
    sys.modules["iron.operators.flm.gemm.design"] = design
    fm = _load(ref, "iron/operators/flm/gemm/reference.py", "ref_flm_gemm")
    for epi, clamp, scale in [("none", None, 4.0), ("silu", None, 0.5), ("gelu", None, 0.5),
                              ("sigmoid", None, 0.5), ("none", (-2.0, 2.0), 4.0), ("silu", (-4.0, 4.0), 0.5)]:
        d = fm.generate_golden_reference(M=128, K=512, N=128, epilogue=Epilogue(epi), clamp=clamp, scale=scale)
        tag = f"_cl{int(clamp[1])}" if clamp else ""
        _save(f"flm_gemm_{epi}{tag}_M128_K512_N128", A=d["input"], B=d["input_b"], C=d["output"])


def q4nx_fixtures(ref: Path):
    """q4nx goldens (the asymmetric int4 input format: min + scale * code): IRON's own
    iron/operators/flm/dequant/reference.py generates a blob (random_q4nx) and
    dequantizes it (dequantize, fp32). Its design module needs mlir_aie; a module holding
    only the geometry constants it imports stands in (values from
    iron/operators/flm/dequant/design.py and iron/operators/flm/gemm/design.py:51-67),
    and pack_b (unused by these two functions) is stubbed."""
    for mname in ("iron", "iron.operators", "iron.operators.flm", "iron.operators.flm.dequant"):
        sys.modules.setdefault(mname, types.ModuleType(mname))
    design = types.ModuleType("iron.operators.flm.dequant.design")
    design.M_TILE, design.K_TILE, design.GROUP = 32, 256, 32
    design.K_TILE_B, design.N_TILE, design.S, design.T, design.CT_K = 512, 64, 8, 8, 128

    def qw_bytes_for(K, N, run_out_features=None, run_period_out_features=None):
        raise RuntimeError("not used by the fixtures")

    design.qw_bytes_for = qw_bytes_for
    sys.modules["iron.operators.flm.dequant.design"] = design
    packing = types.ModuleType("iron.operators.flm.packing")
    packing.pack_b = qw_bytes_for
    sys.modules["iron.operators.flm.packing"] = packing
    qm = _load(ref, "iron/operators/flm/dequant/reference.py", "ref_q4nx")
    for K, N, seed in [(1024, 128, 0), (512, 192, 1)]:
        blob = qm.random_q4nx(K, N, seed=seed)
        w = qm.dequantize(blob, K, N)
        _save(f"q4nx_K{K}_N{N}", blob=blob, w=np.asarray(w, dtype=np.float32), dims=np.array([K, N]))


if __name__ == "__main__":
    import os

    args = [a for a in sys.argv[1:] if not a.startswith("--")]
    src = args[0] if args else os.environ.get("IRON_REFERENCE_DIR")
    if not src:
        sys.exit("usage: make_golden.py <path to the IRON checkout> [--only-gemm | --only-q4nx]")
    if "--only-q4nx" in sys.argv:
        q4nx_fixtures(Path(src))
        sys.exit(0)
    if "--only-gemm" not in sys.argv:
        main(Path(src))
    gemm_fixtures(Path(src))
    q4nx_fixtures(Path(src))
