"""Tolerance and element-wise comparison with IRON's semantics.

IRON judges a buffer with mlir-aie's ``aie.utils.verify`` (used from
iron/common/test_utils.py:18-55): under a relative tolerance an element passes at
``|a - b| < max(atol, rtol * (|a| + |b|))``; equal values always pass, so
``rtol = atol = 0`` demands exact equality; a NaN or infinity must meet the same
value in the reference, whatever mismatch fraction is allowed; and
``max_mismatch_frac`` lets that fraction of finite elements fail.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class Tolerance:
    kind: str = "relative"  # "relative" | "exact"
    rtol: float | None = None
    atol: float = 0.0
    max_mismatch_frac: float = 0.0
    range_frac: float | None = None

    @classmethod
    def relative(cls, rtol: float, atol: float = 0.0, max_mismatch_frac: float = 0.0):
        return cls("relative", float(rtol), float(atol), float(max_mismatch_frac))

    @classmethod
    def exact(cls, max_mismatch_frac: float = 0.0):
        return cls("exact", 0.0, 0.0, float(max_mismatch_frac))


@dataclass
class Verdict:
    n_mismatch: int
    n_checked: int
    n_nonfinite_mismatch: int
    allowed: int
    detail: str

    def __bool__(self) -> bool:
        return self.n_nonfinite_mismatch == 0 and self.n_mismatch <= self.allowed


def _f64(x) -> np.ndarray:
    return np.asarray(x).astype(np.float64).reshape(-1)


def nearly_equal(a, b, rtol: float, atol: float) -> np.ndarray:
    """Element-wise pass mask (NaN never passes here; `compare` pairs NaNs)."""
    a, b = _f64(a), _f64(b)
    with np.errstate(invalid="ignore", over="ignore"):
        bound = np.maximum(atol, rtol * (np.abs(a) + np.abs(b)))
        return (a == b) | (np.abs(a - b) < bound)


def compare(output, expected, tol: Tolerance) -> Verdict:
    out, exp = _f64(output), _f64(expected)
    if out.shape != exp.shape:
        return Verdict(len(exp), len(exp), 0, 0, f"shape {out.shape} vs {exp.shape}")
    both_nan = np.isnan(out) & np.isnan(exp)
    nonfinite = ~np.isfinite(out) | ~np.isfinite(exp)
    if tol.kind == "exact":
        ok = (out == exp) | both_nan
    else:
        ok = nearly_equal(out, exp, tol.rtol or 0.0, tol.atol) | both_nan
    bad = ~ok
    n_bad = int(bad.sum())
    n_nf = int((bad & nonfinite).sum())
    allowed = int(math.floor(tol.max_mismatch_frac * len(exp)))
    detail = "ok"
    if n_bad:
        i = int(np.flatnonzero(bad)[0])
        detail = (
            f"{n_bad}/{len(exp)} mismatches (allowed {allowed}); first at {i}: "
            f"got {out[i]!r}, expected {exp[i]!r}"
        )
    return Verdict(n_bad, len(exp), n_nf, allowed, detail)
