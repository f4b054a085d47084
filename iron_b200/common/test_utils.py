"""Operator test harness with IRON's interface (iron/common/test_utils.py:18-296).

``verify_buffer``, ``run_test`` and ``assert_matches_reference`` behave as IRON's:
buffers are allocated from ``get_arg_spec()`` ("in" from the given data, "out"
fresh), the operator's callable runs ``warmup_iters`` + ``timed_iters`` times,
each output is judged under IRON's tolerance rule, and latency / effective
bandwidth (summed payload bytes / time) are returned. Timing uses CUDA events on
the launching stream.
"""

from __future__ import annotations

import numpy as np
import torch

from .base import AIEOperatorBase
from .tensor import Tensor
from .verify import Tolerance, compare, nearly_equal


def verify_buffer(output, buf_name, reference, rel_tol=0.04, abs_tol=1e-6, max_error_rate=0.0,
                  tolerance: Tolerance | None = None) -> list[int]:
    if tolerance is None:
        tolerance = Tolerance.relative(rel_tol, abs_tol, max_mismatch_frac=max_error_rate)

    def _np(x):
        if isinstance(x, torch.Tensor):
            return x.detach().cpu().float().numpy()
        return np.asarray(x, dtype=np.float32)

    exp = _np(reference).reshape(-1)
    out = _np(output).reshape(-1)
    if len(out) < len(exp):
        print(f"Buffer size mismatch for {buf_name}: expected {len(exp)}, got {len(out)}")
        return list(range(len(out), len(exp)))
    out = out[: len(exp)]
    verdict = compare(out, exp, tolerance)
    if verdict:
        return []
    print(f"{buf_name}: {verdict.detail}")
    both_nan = np.isnan(out) & np.isnan(exp)
    if tolerance.kind == "exact":
        bad = out != exp
    else:
        bad = ~nearly_equal(out, exp, tolerance.rtol or 0.0, tolerance.atol)
    idx = np.flatnonzero(bad & ~both_nan).tolist()
    for i in idx[:10]:
        print(f"Mismatch in {buf_name}[{i}]: expected {exp[i]:.6f}, got {out[i]:.6f}")
    return idx


def time_callable(fn, *args, warmup=1, iters=1) -> float:
    """Mean device time per call in microseconds (CUDA events, current stream)."""
    for _ in range(warmup):
        fn(*args)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record()
    for _ in range(iters):
        fn(*args)
    end.record()
    end.synchronize()
    return start.elapsed_time(end) * 1e3 / max(iters, 1)


def run_test(operator: AIEOperatorBase, input_buffers: dict, output_buffers: dict,
             rel_tol=0.04, abs_tol=1e-6, max_error_rate=0.0, warmup_iters=1, timed_iters=1,
             tolerance: Tolerance | None = None):
    if not isinstance(operator, AIEOperatorBase):
        raise ValueError("run_test only supports AIEOperatorBase subclasses")
    operator.compile()
    op_func = operator.get_callable()
    args, output_map, total = [], {}, 0
    in_iter, out_iter = iter(input_buffers.items()), iter(output_buffers.items())
    for spec in operator.get_arg_spec():
        if spec.direction in ("in", "inout"):
            name, data = next(in_iter)
            buf = Tensor.from_torch(data)
            if spec.direction == "inout":
                output_map[name] = buf
        else:
            name, _ = next(out_iter)
            buf = Tensor(spec.shape, spec.dtype)
            buf.to("npu")
            output_map[name] = buf
        args.append(buf)
        total += buf.data.nbytes
    latency_us = time_callable(op_func, *args, warmup=warmup_iters, iters=timed_iters)
    errors = {}
    for name, expected in output_buffers.items():
        if expected is None or name not in output_map:
            continue
        errs = verify_buffer(output_map[name].to_torch(), name, expected, rel_tol, abs_tol,
                             max_error_rate, tolerance=tolerance)
        if errs:
            errors[name] = errs
    bandwidth_gbps = total / (latency_us * 1e-6) / 1e9
    return errors, latency_us, bandwidth_gbps


def assert_matches_reference(operator, *inputs, tolerance: Tolerance | None = None) -> None:
    in_specs = [s for s in operator.get_arg_spec() if s.direction == "in"]
    if len(inputs) != len(in_specs):
        raise ValueError(f"{type(operator).__name__} takes {len(in_specs)} inputs, got {len(inputs)}")
    expected = operator.reference(*(x.reshape(s.shape) for x, s in zip(inputs, in_specs)))
    if tolerance is None:
        tolerance = operator.reference_tolerance()
    if tolerance is None:
        raise ValueError(f"{type(operator).__name__} declares no tolerance; pass tolerance=")
    errors, latency_us, bandwidth_gbps = run_test(
        operator, {f"input{i}": x for i, x in enumerate(inputs)}, {"output": expected},
        tolerance=tolerance)
    print(f"\nLatency (us): {latency_us:.1f}")
    print(f"Effective Bandwidth: {bandwidth_gbps:.6e} GB/s\n")
    assert not errors, f"Test failed with errors: {errors}"
