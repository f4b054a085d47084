"""Test helpers: golden fixture loading and bf16 conversions."""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"


def bf16(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).astype(np.uint16)).view(torch.bfloat16)


def bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.uint16).numpy()


def load(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}


def load_kwargs(d: dict) -> dict:
    return json.loads(bytes(d["kwargs"]).decode())


def assert_close(got, exp, rtol, atol, max_mismatch_frac=0.0, what=""):
    """IRON's relative tolerance: |a-b| < max(atol, rtol(|a|+|b|)) (or equal)."""
    from iron_b200.common.verify import Tolerance, compare

    v = compare(torch.as_tensor(got).float().numpy(), torch.as_tensor(exp).float().numpy(),
                Tolerance.relative(rtol, atol, max_mismatch_frac))
    assert v, f"{what}: {v.detail}"


def conditioned_rows(run, rtol, atol):
    """Run the oracle twice -- fp32 sums (the reference) and fp64 sums, same bf16 rounding
    points -- and mark the rows whose result agrees with itself within half the tolerance.
    Only those rows can be held to the elementwise bar: in a random-init network some
    inputs amplify a one-ulp difference in an intermediate (a near-cancelling hidden
    state, an attention dominated by the new token) far past it, whichever correct
    summation order computed them. `run` must not depend on state it mutates.
    Returns (reference rows, bool mask of well-conditioned rows)."""
    import torch

    from oracle import ops

    ref = run()
    with ops.accumulate(torch.float64):
        ref64 = run()
    a, b = ref.float(), ref64.float()
    d = (a - b).abs()
    tol = torch.maximum(torch.full_like(d, atol), rtol * (a.abs() + b.abs()))
    return ref, (d < 0.5 * tol).all(dim=-1)
