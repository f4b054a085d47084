"""OperatorSequence: a runlist of operators run as one dispatch per call.

Mirrors iron/common/sequence.py:307-538 (construction, buffer layout, slice
notation, dispatch modes) and its callables :558-736 (``get_buffer``,
``params.write`` / ``params.sync``, input/output/scratch arenas,
``last_elapsed``). On a B200 the modes mean:

* ``"fused"`` (what ``"auto"`` picks): every buffer is a sub-range of three HBM
  arenas (input, output, scratch) and the whole runlist is captured once as a
  CUDA graph whose kernels are chained with programmatic dependent launch; each
  call is one graph launch. Runtime parameters live in a small device array the
  kernels read when they run, so ``params.write`` + ``params.sync`` change them
  without re-capture.
* ``"separate"``: one buffer per name; the steps are launched one by one.
* ``"compare"``: ``"separate"`` plus, after each step, the operator's CPU
  ``reference()`` on the same inputs, held to its tolerance.
* ``"reference"``: CPU only, every step through ``reference()``.

The reference modes are explicit debugging aids; no mode falls back to them.
"""

from __future__ import annotations

import inspect
import logging
import time

import numpy as np
import torch

from .base import AIEOperatorBase, MLIROperator
from .tensor import CPUOnlyTensor, Tensor, np_dtype
from .verify import Tolerance, compare

try:
    import ml_dtypes

    BF16 = np.dtype(ml_dtypes.bfloat16)
except ImportError:  # pragma: no cover
    BF16 = np.dtype(np.uint16)

logger = logging.getLogger(__name__)


def _n_elements(nbytes: int) -> int:
    return max(int(nbytes), BF16.itemsize) // BF16.itemsize


def _accepts_flags(op) -> bool:
    try:
        return "flags" in inspect.signature(op._launch).parameters
    except (TypeError, ValueError):
        return False


# ---------------------------------------------------------------------------
# Dispatch policies (iron/common/sequence.py:62-297)
# ---------------------------------------------------------------------------


class SequenceDispatch:
    name = "base"

    def resolve(self, device=None) -> "SequenceDispatch":
        return self

    def set_up_artifacts(self, seq) -> None:
        """Nothing to build: every kernel ships in libiron_b200.so."""

    def make_callable(self, seq):  # pragma: no cover - abstract
        raise NotImplementedError


class FusedDispatch(SequenceDispatch):
    """Arena buffers, one CUDA graph per call."""

    name = "fused"

    def __init__(self, pdl: bool = True):
        self.pdl = pdl

    def make_callable(self, seq):
        return SequenceGraphCallable(seq, pdl=self.pdl)


class AutoDispatch(SequenceDispatch):
    """Resolves to ``fused`` (IRON picks by NPU generation; every B200 takes the graph path)."""

    name = "auto"

    def resolve(self, device=None):
        return FusedDispatch()


class SeparateDispatch(SequenceDispatch):
    name = "separate"

    def make_callable(self, seq):
        return SequenceStepCallable(seq)


class CompareDispatch(SeparateDispatch):
    """``separate`` plus a per-step check against each operator's ``reference()``.

    Args:
        tolerance: held to every step; by default each step uses its operator's
            ``reference_tolerance()``, else ``FALLBACK_TOLERANCE``.
        raise_on_mismatch: raise ``RuntimeError`` on the first failing step.
    """

    name = "compare"
    FALLBACK_TOLERANCE = Tolerance.relative(0.025, 1e-2)

    def __init__(self, tolerance=None, raise_on_mismatch=True):
        self.tolerance = tolerance
        self.raise_on_mismatch = raise_on_mismatch

    def step_tolerance(self, op):
        if self.tolerance is not None:
            return self.tolerance
        tol = op.reference_tolerance() if isinstance(op, MLIROperator) else None
        if tol is None or tol.range_frac is not None:
            return self.FALLBACK_TOLERANCE
        return tol

    def make_callable(self, seq):
        return SequenceCompareCallable(seq, self)


class ReferenceDispatch(SequenceDispatch):
    name = "reference"

    def make_callable(self, seq):
        return SequenceReferenceCallable(seq)


_DISPATCH_ALIASES = {
    "auto": AutoDispatch,
    "fused": FusedDispatch,
    "separate": SeparateDispatch,
    "compare": CompareDispatch,
    "reference": ReferenceDispatch,
}


# ---------------------------------------------------------------------------
# The sequence
# ---------------------------------------------------------------------------


class OperatorSequence(AIEOperatorBase):
    """A runlist of ``(operator, *buffer_names)`` run as one dispatch.

    Buffer names are shared between steps (zero-copy hand-off); a name of the
    form ``"base[start:end]"`` is a byte slice of ``base``, whose size must be
    given in ``buffer_sizes``. Arguments ``extra_flags``, ``trace_size`` and
    ``share_designs`` are accepted for IRON compatibility; there is no compiler
    to pass flags to and no design to share.
    """

    def __init__(self, name, runlist, input_args, output_args, buffer_sizes=None, dispatch="auto",
                 extra_flags=None, trace_size=0, share_designs=False, *args, **kwargs):
        dispatch = self._coerce_dispatch(dispatch)
        if not all(isinstance(op, MLIROperator) and all(isinstance(b, str) for b in bufs)
                   for op, *bufs in runlist):
            raise TypeError("runlist entries must be (MLIROperator, *str) tuples; "
                            "each operator must be an MLIROperator and each buffer name must be a str")
        super().__init__(*args, **kwargs)
        self.runlist = runlist
        self.name = name + "_shared" if share_designs else name
        self.input_args = list(input_args)
        self.output_args = list(output_args)
        self.explicit_buffer_sizes = dict(buffer_sizes or {})
        self.extra_flags = list(extra_flags or [])
        self.trace_size = trace_size
        self.share_designs = share_designs
        self._dispatch = dispatch

    @staticmethod
    def _coerce_dispatch(dispatch):
        if isinstance(dispatch, SequenceDispatch):
            return dispatch
        if isinstance(dispatch, str) and dispatch in _DISPATCH_ALIASES:
            return _DISPATCH_ALIASES[dispatch]()
        raise TypeError("selected dispatch mode not supported")

    def unique_operators(self):
        seen = {}
        for op, *_ in self.runlist:
            seen.setdefault(id(op), op)
        return list(seen.values())

    def runtime_parameters(self) -> list[str]:
        """Names of the runtime parameters the runlist's operators read."""
        names = []
        for op in self.unique_operators():
            for n in op.runtime_parameters():
                if n not in names:
                    names.append(n)
        return names

    # -- layout (iron/common/sequence.py:408-500) -----------------------------
    def calculate_buffer_layout(self):
        args = {}
        sliced = {}
        for op, *bufs in self.runlist:
            specs = op.get_arg_spec()
            if len(specs) != len(bufs):
                raise ValueError(f"Number of buffers ({len(bufs)}) must match operator argument "
                                 f"specification ({len(specs)}) for operator {op!r}")
            for buf, spec in zip(bufs, specs):
                if "[" in buf and buf.endswith("]"):
                    base = buf[: buf.index("[")]
                    start, end = map(int, buf[buf.index("[") + 1 : -1].split(":"))
                    if base not in args and base not in self.explicit_buffer_sizes:
                        raise ValueError(f"Sliced buffer '{buf}' requires explicit size for base buffer "
                                         f"'{base}' in buffer_sizes parameter")
                    if not 0 <= start <= end:
                        raise ValueError(f"Sliced buffer '{buf}' has an invalid byte range")
                    sliced[buf] = (base, start, end, spec)
                elif buf not in args:
                    args[buf] = spec
                elif np.prod(args[buf].shape) != np.prod(spec.shape):
                    raise ValueError(f"Buffer '{buf}' has conflicting sizes between operators: "
                                     f"{args[buf].shape} vs {spec.shape}")
        names = set(args) | set(sliced)
        for a in self.input_args:
            if a not in names and a not in self.explicit_buffer_sizes:
                raise ValueError(f"Input argument {a} not found in runlist buffers")
        for a in self.output_args:
            if a not in names and a not in self.explicit_buffer_sizes:
                raise ValueError(f"Output argument {a} not found in runlist buffers")

        layout = {}

        def place(kind, names_):
            off = 0
            for a in names_:
                if a in self.explicit_buffer_sizes:
                    length = int(self.explicit_buffer_sizes[a])
                elif a in args:
                    length = int(np.prod(args[a].shape)) * np_dtype(args[a].dtype).itemsize
                else:
                    continue
                layout[a] = (kind, off, length)
                off += -(-length // 256) * 256  # 256-byte aligned sub-buffers (vector loads, TMA)
            return off

        slice_info = {b: (base, s, e) for b, (base, s, e, _) in sliced.items()}
        for b, (base, s, e, spec) in sliced.items():
            cap = self.explicit_buffer_sizes.get(base)
            if cap is not None and e > cap:
                raise ValueError(f"Sliced buffer '{b}' ends past its base buffer ({e} > {cap} bytes)")
        in_sz = place("input", self.input_args)
        out_sz = place("output", self.output_args)
        scratch = [a for a in args if a not in self.input_args and a not in self.output_args]
        scratch += [a for a in self.explicit_buffer_sizes
                    if a not in self.input_args and a not in self.output_args and a not in scratch]
        sc_sz = place("scratch", scratch)
        return layout, (in_sz, out_sz, sc_sz), slice_info

    def set_up_artifacts(self):
        self.subbuffer_layout, self.buffer_sizes, self.slice_info = self.calculate_buffer_layout()
        self._dispatch = self._dispatch.resolve()
        self._dispatch.set_up_artifacts(self)

    def compile(self, dry_run: bool = False):
        self.set_up_artifacts()
        if not dry_run and self._dispatch.name != "reference":
            from .. import _lib

            _lib.load()
        return self

    def get_arg_spec(self):
        raise NotImplementedError("OperatorSequence does not expose a unified arg spec; "
                                  "use get_layout_for_buffer() to inspect individual buffer layouts")

    def get_callable(self):
        if not hasattr(self, "subbuffer_layout"):
            self.compile()
        return self._dispatch.make_callable(self)

    def get_layout_for_buffer(self, buffer_name):
        """(buffer_type, start_byte, end_byte) of a named buffer; slices resolve to
        their parent's absolute offset (iron/common/sequence.py:515-536)."""
        if buffer_name in self.slice_info:
            base, s, e = self.slice_info[buffer_name]
            kind, ps, _ = self.get_layout_for_buffer(base)
            return kind, ps + s, ps + e
        kind, off, length = self.subbuffer_layout[buffer_name]
        return kind, off, length


# ---------------------------------------------------------------------------
# Runtime parameters (the ParameterScratchpad of iron/common/sequence.py:641-666)
# ---------------------------------------------------------------------------


class SequenceParams:
    """int32 runtime parameters in one device array; operators read their word
    when they run. ``write`` sets the host copy, ``sync`` uploads it on the
    current stream (so it orders before the next dispatch)."""

    def __init__(self, names):
        self.names = list(names)
        self._index = {n: i for i, n in enumerate(self.names)}
        self.host = torch.zeros(len(self.names), dtype=torch.int32, pin_memory=True)
        self.device = torch.zeros(len(self.names), dtype=torch.int32, device="cuda")

    def word(self, name) -> torch.Tensor:
        i = self._index[name]
        return self.device[i : i + 1]

    def write(self, name, value) -> None:
        if name not in self._index:
            raise KeyError(f"unknown runtime parameter {name!r}; declared: {self.names}")
        self.host[self._index[name]] = int(np.int32(value))

    def read(self, name) -> int:
        return int(self.host[self._index[name]])

    def sync(self) -> None:
        self.device.copy_(self.host, non_blocking=True)


# ---------------------------------------------------------------------------
# Callables
# ---------------------------------------------------------------------------


class SequenceCallable:
    """Shared runtime: step iteration, syncs, timing (iron/common/sequence.py:558-603)."""

    def __init__(self, op):
        self.op = op
        self.last_elapsed = 0.0
        self._buffer_cache = {}
        self._allocate_buffers()
        self._params = None

    def _allocate_buffers(self):  # pragma: no cover - abstract
        raise NotImplementedError

    def get_buffer(self, buffer_name):  # pragma: no cover - abstract
        raise NotImplementedError

    def _iter_steps(self):
        for step_op, *names in self.op.runlist:
            specs = step_op.get_arg_spec()
            if len(specs) != len(names):
                raise ValueError(f"Operator {step_op!r} arg-spec count {len(specs)} does not "
                                 f"match runlist buffer count {len(names)}")
            *in_names, out_name = names
            *in_specs, out_spec = specs
            yield step_op, in_names, in_specs, out_name, out_spec

    @property
    def params(self):
        """Runtime parameters, or None when no operator of the runlist declares one."""
        if self._params is None:
            names = self.op.runtime_parameters()
            if not names:
                return None
            self._params = SequenceParams(names)
            for step_op in self.op.unique_operators():
                for n in step_op.runtime_parameters():
                    step_op.bind_param(n, self._params.word(n))
        return self._params

    def _sync_inputs(self):
        pass

    def _sync_outputs(self):
        pass

    def _run(self):  # pragma: no cover - abstract
        raise NotImplementedError

    def __call__(self):
        self._sync_inputs()
        t0 = time.perf_counter()
        self._run()
        self.last_elapsed = time.perf_counter() - t0
        self._sync_outputs()


class _DeviceCallable(SequenceCallable):
    def _prepare_ops(self):
        _ = self.params  # bind parameter words before any launch
        for step_op in self.op.unique_operators():
            step_op.prepare()

    def _launch_step(self, step_op, bufs, stream, pdl=False):
        if pdl and _accepts_flags(step_op):
            from .. import _lib

            step_op._launch(*bufs, stream=stream, flags=_lib.IRON_FLAG_PDL)
        else:
            step_op._launch(*bufs, stream=stream)


class SequenceGraphCallable(_DeviceCallable):
    """Fused dispatch: three HBM arenas addressed by offset, the runlist captured
    once as a CUDA graph and replayed per call."""

    def __init__(self, op, pdl=True):
        self.pdl = pdl
        self.graph = None
        super().__init__(op)
        self._plan = [(step_op, [self.get_buffer(n) for n in names]) for step_op, *names in op.runlist]
        self._stream = torch.cuda.Stream()

    def _allocate_buffers(self):
        in_sz, out_sz, sc_sz = self.op.buffer_sizes
        self.input_buffer = Tensor((_n_elements(in_sz),), BF16)
        self.output_buffer = Tensor((_n_elements(out_sz),), BF16)
        self.scratch_buffer = Tensor((_n_elements(sc_sz),), BF16)
        for arena in (self.input_buffer, self.output_buffer, self.scratch_buffer):
            arena.to("npu")  # allocate in HBM before any capture

    def get_buffer(self, buffer_name):
        if buffer_name not in self._buffer_cache:
            kind, start, end = self.op.get_layout_for_buffer(buffer_name)
            parent = {"input": self.input_buffer, "output": self.output_buffer,
                      "scratch": self.scratch_buffer}[kind]
            length = (end - start) if buffer_name in self.op.slice_info else end
            self._buffer_cache[buffer_name] = parent.subview(start, (length // BF16.itemsize,), BF16)
        return self._buffer_cache[buffer_name]

    def _capture(self):
        from .. import _lib

        self._prepare_ops()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=self._stream):
            s = _lib.current_stream()
            for step_op, bufs in self._plan:
                self._launch_step(step_op, bufs, s, self.pdl)
        self.graph = g

    def invalidate(self):
        """Drop the captured graph (e.g. after rebinding buffers); the next call re-captures."""
        self.graph = None

    def _sync_inputs(self):
        self.input_buffer.to("npu")
        self.scratch_buffer.to("npu")

    def _sync_outputs(self):
        self.output_buffer.mark_device_written()
        self.scratch_buffer.mark_device_written()
        self.output_buffer.to("cpu")

    def _run(self):
        if self.graph is None:
            self._capture()
        self.graph.replay()
        torch.cuda.current_stream().synchronize()


class _PerBufferCallable(SequenceCallable):
    tensor_cls = Tensor

    def _allocate_buffers(self):
        self._buffers = {}
        for name, (_, _, length) in self.op.subbuffer_layout.items():
            self._buffers[name] = self.tensor_cls((_n_elements(length),), BF16)

    def _resolve_buffer(self, name):
        if name in self._buffers:
            return self._buffers[name]
        if name in self.op.slice_info:
            base, s, e = self.op.slice_info[name]
            sub = self._buffers[base].subview(s, ((e - s) // BF16.itemsize,), BF16)
            self._buffers[name] = sub
            return sub
        raise ValueError(f"Unknown buffer '{name}' in runlist")

    def get_buffer(self, buffer_name):
        if buffer_name not in self._buffer_cache:
            self._buffer_cache[buffer_name] = self._resolve_buffer(buffer_name)
        return self._buffer_cache[buffer_name]


class SequenceStepCallable(_PerBufferCallable, _DeviceCallable):
    """Separate dispatch: one HBM buffer per name, steps launched in order."""

    def _sync_inputs(self):
        for name in self.op.subbuffer_layout:
            self._buffers[name].to("npu")  # uploads only host-written ranges

    def _sync_outputs(self):
        for name in self.op.subbuffer_layout:
            if name not in self.op.input_args:
                self._buffers[name].mark_device_written()
                self._buffers[name].to("cpu")

    def _run(self):
        from .. import _lib

        self._prepare_ops()
        s = _lib.current_stream()
        for step_idx, step in enumerate(self._iter_steps()):
            self._run_step(step_idx, step, s)
        torch.cuda.current_stream().synchronize()

    def _run_step(self, step_idx, step, stream):
        step_op, in_names, _, out_name, _ = step
        self._launch_step(step_op, [self._resolve_buffer(n) for n in in_names + [out_name]], stream)


def _reshape_for_spec(flat, spec):
    n = int(np.prod(spec.shape)) if spec.shape else 1
    return flat[:n].reshape(spec.shape)


class SequenceReferenceCallable(_PerBufferCallable):
    """CPU evaluation through each operator's ``reference()``; no kernel runs."""

    tensor_cls = CPUOnlyTensor

    def _run(self):
        for step_op, in_names, in_specs, out_name, out_spec in self._iter_steps():
            inputs = [_reshape_for_spec(self._resolve_buffer(n)._host_view(), s).clone()
                      for n, s in zip(in_names, in_specs)]
            out = step_op.reference(*inputs)
            flat = self._resolve_buffer(out_name)._host_view()
            n = int(np.prod(out_spec.shape)) if out_spec.shape else 1
            flat[:n].copy_(out.reshape(-1).to(torch.bfloat16))


class SequenceCompareCallable(SequenceStepCallable):
    """Separate dispatch plus a per-step check of each output against the
    operator's ``reference()`` on the same (GPU-produced) inputs, so every
    comparison isolates one operator (iron/common/sequence.py:884-985)."""

    def __init__(self, op, dispatch):
        self.dispatch = dispatch
        self.raise_on_mismatch = dispatch.raise_on_mismatch
        self.last_step_stats = []
        super().__init__(op)

    def _run(self):
        self.last_step_stats = []
        super()._run()

    def _read(self, name, spec):
        buf = self._resolve_buffer(name)
        n = int(np.prod(spec.shape)) if spec.shape else 1
        return buf.device_tensor.reshape(-1)[:n].cpu().clone().reshape(spec.shape)

    def _run_step(self, step_idx, step, stream):
        step_op, in_names, in_specs, out_name, out_spec = step
        torch.cuda.current_stream().synchronize()
        cpu_inputs = [self._read(n, s) for n, s in zip(in_names, in_specs)]
        super()._run_step(step_idx, step, stream)
        torch.cuda.current_stream().synchronize()
        got = self._read(out_name, out_spec)
        ref = step_op.reference(*cpu_inputs).reshape(out_spec.shape)
        gf, rf = got.to(torch.float32), ref.to(torch.float32)
        diff = (gf - rf).abs()
        stats = {"step": step_idx, "op": type(step_op).__name__,
                 "op_name": getattr(step_op, "name", type(step_op).__name__),
                 "inputs": list(in_names), "output": out_name, "skipped": False,
                 "max_abs": float(diff.max()) if diff.numel() else 0.0,
                 "mean_abs": float(diff.mean()) if diff.numel() else 0.0,
                 "max_rel": float((diff / (rf.abs() + 1e-6)).max()) if diff.numel() else 0.0,
                 "ref_max": float(rf.abs().max()) if diff.numel() else 0.0}
        tol = self.dispatch.step_tolerance(step_op)
        verdict = compare(gf.numpy(), rf.numpy(), tol)
        stats["mismatch"] = not verdict
        logger.log(logging.ERROR if not verdict else logging.INFO,
                   "[compare step %d] %s -> %s: max_abs=%.4g mean_abs=%.4g max_rel=%.4g ref_max=%.4g%s",
                   step_idx, stats["op"], out_name, stats["max_abs"], stats["mean_abs"], stats["max_rel"],
                   stats["ref_max"], f"  MISMATCH: {verdict.detail}" if not verdict else "")
        self.last_step_stats.append(stats)
        if not verdict and self.raise_on_mismatch:
            raise RuntimeError(
                f"[compare step {step_idx}] {stats['op']} (name={stats['op_name']}) -> {out_name}: "
                f"GPU output deviates from reference ({verdict.detail}; max_abs={stats['max_abs']:.4g}, "
                f"max_rel={stats['max_rel']:.4g}, ref_max={stats['ref_max']:.4g}; inputs={list(in_names)}; "
                f"tolerance {tol})")
