"""Host-side split rules of the decode attention, read through the C ABI without a GPU
(the SM count falls back to the B200's 148): enough split CTAs for two waves, at most
4096 tokens per split CTA, clusters only while a CTA's share is at most 512 tokens.
The split count s shows in the workspace size of the split-and-combine form,
B * Hq * s * (2 + D) * 4 bytes (0 when s = 1; reported also where the splits merge in a
cluster instead), and in the launches per call (1: one split or one cluster per
(sequence, kv head); 2: split kernel + combine)."""

import pytest

from iron_b200 import _lib

HQ, HKV, D = 32, 8, 64


def _splits(B, L):
    ws = _lib.load().iron_attn_decode_workspace_bytes_d(B, HQ, HKV, L, D)
    return ws // (B * HQ * (2 + D) * 4) if ws else 1


@pytest.mark.parametrize("B,L,splits,launches", [
    (1, 2320, 37, 1),     # decode batch 1: 37 chunks of 64 tokens, merged in clusters of 16
    (2, 2320, 32, 1),     # batch 2: clusters of 8
    (8, 2320, 8, 2),      # batch 8: two waves of split CTAs, combine kernel
    (64, 2320, 1, 1),     # batch 64: one CTA per (sequence, kv head) already fills two waves
    (64, 4096, 1, 1),     # 4096 tokens still fit one CTA
    (1, 32768, 64, 2),    # a cluster CTA would get 2048 tokens: independent splits instead
    (16, 32768, 8, 2),    # the 4096-token cap, not the waves, sets the count
    (64, 32768, 8, 2),
])
def test_split_rules(B, L, splits, launches):
    assert _splits(B, L) == splits
    assert _lib.load().iron_attn_decode_kernels(B, HQ, HKV, L) == launches


def test_fused_form_uses_the_same_splits():
    lib = _lib.load()
    for B, L in [(1, 2320), (8, 2320), (64, 32768)]:
        assert lib.iron_attn_decode_qkv_workspace_bytes(B, HQ, HKV, L, D) == \
            lib.iron_attn_decode_workspace_bytes_d(B, HQ, HKV, L, D)


def test_noalloc_argument_checks_and_capacity_on_the_host():
    """iron_attn_decode_noalloc runs iron_attn_decode's argument checks first, then sizes
    its fixed 1 MiB array; every status below is returned before any CUDA call."""
    lib = _lib.load()
    ok = 16  # any non-null, 16-byte aligned stand-in: nothing is launched
    L = 32768

    def call(q=ok, B=18, Hq=32, Hkv=8, D=128, kv_b=8 * L * 128, kv_h=L * 128):
        return lib.iron_attn_decode_noalloc(q, ok, ok, ok, ok, B, Hq, Hkv, D, L, kv_b, kv_h, 0.088, 0, None)

    assert call() == -6                   # head_dim 128, batch 18: 1,198,080 B of partials even at 4 splits
    assert call(q=None) == -1             # null pointer
    assert call(Hq=30) == -2              # query heads not a multiple of kv heads
    assert call(D=96) == -4               # head size not served
    assert call(q=24) == -3               # misaligned q
    assert call(kv_h=L * 128 + 4) == -3   # misaligned head stride
