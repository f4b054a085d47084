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
