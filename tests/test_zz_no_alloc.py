"""The allocation-free decode attention entry point (iron_attn_decode_noalloc).

Some callers cannot allocate device memory: their GPU memory is owned by another
allocator (a serving engine that reserves it all up front), or they sit on a
latency-critical path where cudaMalloc's implicit synchronisation is not
acceptable. For them the split partials live in a fixed array inside the library.
This file is collected last on purpose; it must also pass when run alone in a
fresh process, where the first call performs the per-device address lookup.
Both calls below go through the C ABI and are compared with iron_attn_decode
(which takes a caller-provided workspace) at the attention tolerance of the
other tests (rtol 2e-2, atol 1e-2).
"""

import math

import pytest
import torch

from helpers import assert_close

pytestmark = pytest.mark.gpu

from iron_b200 import _lib


def _inputs(B, L, seed, Hq=32, Hkv=8, D=64):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(B, Hq, D, generator=g, device="cuda").to(torch.bfloat16)
    k = torch.randn(B, Hkv, L, D, generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn(B, Hkv, L, D, generator=g, device="cuda").to(torch.bfloat16)
    lens = torch.randint(1, L + 1, (B,), generator=g, device="cuda", dtype=torch.int32)
    return q, k, v, lens


def _call(fn, q, k, v, lens, ws=None):
    B, Hkv, L, D = k.shape
    Hq = q.shape[1]
    out = torch.empty_like(q)
    args = [q.data_ptr(), k.data_ptr(), v.data_ptr(), lens.data_ptr(), out.data_ptr(), B, Hq, Hkv,
            D, L, Hkv * L * D, L * D, 1.0 / math.sqrt(D)]
    if fn == "iron_attn_decode":
        args += [ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0]
    _lib.call(fn, *args, 0, _lib.current_stream())
    return out


def test_noalloc_matches_workspace_entry_point_twice():
    lib = _lib.load()
    # two calls in a row with different shapes and inputs: the second reuses
    # (and fully rewrites) the partials the first left in the fixed array
    for B, L, seed in [(1, 32768, 1), (4, 4096, 2)]:
        q, k, v, lens = _inputs(B, L, seed)
        need = lib.iron_attn_decode_workspace_bytes(B, 32, 8, L)
        assert 0 < need <= 1 << 20, "case must use split partials within the fixed array"
        ws = torch.zeros(need, dtype=torch.uint8, device="cuda")
        ref = _call("iron_attn_decode", q, k, v, lens, ws)
        got = _call("iron_attn_decode_noalloc", q, k, v, lens)
        torch.cuda.synchronize()
        assert_close(got.cpu(), ref.cpu(), 2e-2, 1e-2, what=f"noalloc B{B} L{L}")


def test_noalloc_rejects_requests_beyond_the_fixed_array():
    lib = _lib.load()
    B, Hq, Hkv, L = 8, 128, 8, 32768  # 16-head groups: partials beyond the 1 MiB array
    assert lib.iron_attn_decode_workspace_bytes(B, Hq, Hkv, L) > 1 << 20
    st = lib.iron_attn_decode_noalloc(16, 16, 16, 16, 16, B, Hq, Hkv, 64, L, Hkv * L * 64, L * 64,
                                      0.125, 0, None)
    assert st == -6  # IRON_ERR_WORKSPACE, raised before any launch
