"""The allocation-free decode attention entry point (iron_attn_decode_noalloc).

Some callers cannot allocate device memory: their GPU memory is owned by another
allocator (a serving engine that reserves it all up front), or they sit on a
latency-critical path where cudaMalloc's implicit synchronisation is not
acceptable. For them the split partials live in a fixed array inside the library.
This file is collected last on purpose; it must also pass when run alone in a
fresh process, where the first call performs the per-device address lookup.
Both calls below go through the C ABI and are compared with iron_attn_decode
(which takes a caller-provided workspace) at the attention tolerance of the
other tests (rtol 2e-2, atol 1e-2). The cases whose usual split partials exceed
the fixed array (fewer splits, longer chunks) are also compared with the CPU
oracle (oracle.ops.attn_decode, IRON's decode attention restated).
"""

import math

import pytest
import torch

from helpers import assert_close
from oracle import ops

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


@pytest.mark.parametrize("B,L,D", [(16, 32768, 64), (5, 32768, 128)])
def test_noalloc_fewer_splits_matches_oracle(B, L, D):
    """B 16 x 32768 tokens at head_dim 64: the usual 8 splits' partials (1.08 MB) exceed
    the 1 MiB array, so the call drops to 4 splits of 8192 tokens (past the usual
    4096-token cap). B 5 x 32768 at head_dim 128 fits as is. Ragged lengths; two calls
    in a row on different inputs; both against the oracle and iron_attn_decode."""
    lib = _lib.load()
    need = lib.iron_attn_decode_workspace_bytes_d(B, 32, 8, L, D)
    if D == 64:
        assert need > 1 << 20, "case must take the split-reduction branch"
    else:
        assert 0 < need <= 1 << 20
    for seed in (5, 6):
        q, k, v, lens = _inputs(B, L, seed, D=D)
        lens[0] = L  # one full-length sequence, one of a single token
        lens[1] = 1
        ws = torch.zeros(need, dtype=torch.uint8, device="cuda")
        ref = _call("iron_attn_decode", q, k, v, lens, ws)
        got = _call("iron_attn_decode_noalloc", q, k, v, lens)
        torch.cuda.synchronize()
        exp = ops.attn_decode(q.cpu(), k.cpu(), v.cpu(), lens.cpu().tolist())
        assert_close(got.cpu(), exp, 2e-2, 1e-2, what=f"noalloc vs oracle B{B} L{L} D{D}")
        assert_close(got.cpu(), ref.cpu(), 2e-2, 1e-2, what=f"noalloc vs workspace form B{B} L{L} D{D}")


def test_noalloc_rejects_requests_beyond_the_fixed_array():
    lib = _lib.load()
    B, Hq, Hkv, L = 8, 128, 8, 32768  # 16-head groups: partials beyond the 1 MiB array
    assert lib.iron_attn_decode_workspace_bytes(B, Hq, Hkv, L) > 1 << 20
    st = lib.iron_attn_decode_noalloc(16, 16, 16, 16, 16, B, Hq, Hkv, 64, L, Hkv * L * 64, L * 64,
                                      0.125, 0, None)
    assert st == -6  # IRON_ERR_WORKSPACE, raised before any launch
    # head_dim 128, batch 18 x 32768 tokens: even the two-wave count's partials
    # (18 * 32 * 4 splits * 130 * 4 B = 1,198,080 B) exceed the array
    assert lib.iron_attn_decode_noalloc(16, 16, 16, 16, 16, 18, 32, 8, 128, 32768, 8 * 32768 * 128, 32768 * 128,
                                        0.088, 0, None) == -6
    # the argument checks come first: a null pointer is reported as such
    assert lib.iron_attn_decode_noalloc(None, 16, 16, 16, 16, 18, 32, 8, 128, 32768, 8 * 32768 * 128,
                                        32768 * 128, 0.088, 0, None) == -1
