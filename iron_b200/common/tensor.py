"""Device buffer with the XRTTensor surface IRON's callers use.

IRON's application and sequence code move data with an explicit-sync host/device
buffer (``XRTTensor``; used at iron/applications/llama_3.2_1b/llama_npu.py:651-716
and iron/common/sequence.py:670-730): ``Tensor(shape, dtype)``, ``from_torch``,
``subview(byte_offset, shape, dtype)``, ``torch_view()``, ``to("npu"|"cpu")``,
``to_torch()``, ``fill_()``, ``numpy()``, ``shape``, ``device``,
``buffer_object()``. Here "npu" is the current CUDA device: each buffer owns a
byte array in HBM and a pinned host mirror, and data moves only when the caller
asks, exactly as with XRT. Kernels read ``device_tensor``, a typed CUDA view.
"""

from __future__ import annotations

import numpy as np
import torch

try:
    from ml_dtypes import bfloat16 as _np_bf16
except ImportError:  # pragma: no cover - ml_dtypes ships with this image
    _np_bf16 = None

_NP_TO_TORCH = {
    np.dtype(np.float32): torch.float32,
    np.dtype(np.float16): torch.float16,
    np.dtype(np.float64): torch.float64,
    np.dtype(np.int8): torch.int8,
    np.dtype(np.uint8): torch.uint8,
    np.dtype(np.int16): torch.int16,
    np.dtype(np.uint16): torch.uint16,
    np.dtype(np.int32): torch.int32,
    np.dtype(np.uint32): torch.uint32,
    np.dtype(np.int64): torch.int64,
}
if _np_bf16 is not None:
    _NP_TO_TORCH[np.dtype(_np_bf16)] = torch.bfloat16


def np_dtype(dtype) -> np.dtype:
    if isinstance(dtype, torch.dtype):
        for k, v in _NP_TO_TORCH.items():
            if v == dtype:
                return k
        raise TypeError(f"unsupported dtype {dtype}")
    return np.dtype(dtype)


def torch_dtype(dtype) -> torch.dtype:
    if isinstance(dtype, torch.dtype):
        return dtype
    try:
        return _NP_TO_TORCH[np.dtype(dtype)]
    except KeyError as e:
        raise TypeError(f"unsupported dtype {dtype}") from e


def _cuda_ok() -> bool:
    return torch.cuda.is_available()


class _Intervals:
    """Sorted, disjoint half-open byte ranges."""

    def __init__(self):
        self.iv: list[tuple[int, int]] = []

    def add(self, s: int, e: int) -> None:
        if e <= s:
            return
        out, placed = [], False
        for a, b in self.iv:
            if b < s or a > e:
                if a > e and not placed:
                    out.append((s, e))
                    placed = True
                out.append((a, b))
            else:
                s, e = min(a, s), max(b, e)
        if not placed:
            out.append((s, e))
        self.iv = sorted(out)

    def take(self, s: int, e: int) -> list[tuple[int, int]]:
        """Remove and return the parts of the set inside [s, e)."""
        got, keep = [], []
        for a, b in self.iv:
            lo, hi = max(a, s), min(b, e)
            if lo < hi:
                got.append((lo, hi))
                if a < lo:
                    keep.append((a, lo))
                if hi < b:
                    keep.append((hi, b))
            else:
                keep.append((a, b))
        self.iv = sorted(keep)
        return got


class _Storage:
    """Byte arrays shared by a tensor and its subviews, with a coherence map:
    ``host_dirty`` ranges were written on the host since the last upload,
    ``dev_dirty`` ranges were written by kernels since the last download."""

    def __init__(self, nbytes: int, host_only: bool = False):
        self.nbytes = max(int(nbytes), 1)
        self.host_only = host_only
        pin = _cuda_ok() and not host_only
        self.host = torch.zeros(self.nbytes, dtype=torch.uint8, pin_memory=pin)
        self._dev = None
        self.host_dirty = _Intervals()
        self.dev_dirty = _Intervals()

    @property
    def allocated(self) -> bool:
        return self._dev is not None

    @property
    def dev(self) -> torch.Tensor:
        if self._dev is None:
            if self.host_only:
                raise RuntimeError("this buffer is host-only (reference dispatch)")
            if not _cuda_ok():
                raise RuntimeError("no CUDA device: iron_b200 buffers live in B200 HBM")
            self._dev = torch.zeros(self.nbytes, dtype=torch.uint8, device="cuda")
        return self._dev


class Tensor:
    """Explicit-sync host/HBM buffer (the XRTTensor surface on a B200).

    A host view handed out by ``torch_view()`` / ``numpy()`` is assumed written:
    its range is uploaded by the next ``to("npu")``. Ranges that kernels wrote
    (``mark_device_written``, done by the sequence callables after a run) are
    downloaded before the host view is handed out, so host reads never see
    stale data and a host write never clobbers newer device data; ``to("cpu")``
    likewise keeps host-written ranges that have not been uploaded yet.
    """

    _host_only = False

    def __init__(self, shape, dtype=None, *, _storage=None, _offset=0):
        if dtype is None:
            dtype = _np_bf16
        self.dtype = np_dtype(dtype)
        self.shape = tuple(int(s) for s in (shape if isinstance(shape, (tuple, list)) else (shape,)))
        self._offset = int(_offset)
        self._nbytes = int(np.prod(self.shape, dtype=np.int64)) * self.dtype.itemsize
        self._storage = _storage if _storage is not None else _Storage(self._nbytes, self._host_only)
        if self._offset + self._nbytes > self._storage.nbytes:
            raise ValueError("subview exceeds its parent buffer")
        self.device = "cpu"

    # -- construction --------------------------------------------------------
    @classmethod
    def from_torch(cls, t: torch.Tensor) -> "Tensor":
        t = t.detach()
        out = cls(tuple(t.shape), np_dtype(t.dtype))
        out.torch_view().copy_(t.reshape(out.shape).cpu())
        if _cuda_ok() and not cls._host_only:
            out.to("npu")
        return out

    def subview(self, byte_offset: int, shape, dtype) -> "Tensor":
        sub = type(self)(shape, dtype, _storage=self._storage, _offset=self._offset + int(byte_offset))
        sub.device = self.device
        return sub

    # -- views ---------------------------------------------------------------
    @property
    def _range(self) -> tuple[int, int]:
        return self._offset, self._offset + self._nbytes

    def _bytes(self, t: torch.Tensor) -> torch.Tensor:
        return t[self._offset : self._offset + self._nbytes]

    def _pull_stale(self) -> None:
        st = self._storage
        for s, e in st.dev_dirty.take(*self._range):
            st.host[s:e].copy_(st.dev[s:e])

    def _host_view(self) -> torch.Tensor:
        return self._bytes(self._storage.host).view(torch_dtype(self.dtype)).view(self.shape)

    def torch_view(self) -> torch.Tensor:
        """Host view (what the next ``to("npu")`` uploads)."""
        self._pull_stale()
        self._storage.host_dirty.add(*self._range)
        return self._host_view()

    @property
    def device_tensor(self) -> torch.Tensor:
        """Typed CUDA view of this buffer's HBM bytes."""
        return self._bytes(self._storage.dev).view(torch_dtype(self.dtype)).view(self.shape)

    def buffer_object(self) -> torch.Tensor:
        return self.device_tensor

    @property
    def data(self) -> np.ndarray:
        return self.numpy()

    def numpy(self) -> np.ndarray:
        self._pull_stale()
        self._storage.host_dirty.add(*self._range)
        raw = self._bytes(self._storage.host).numpy()
        return raw.view(self.dtype).reshape(self.shape)

    # -- synchronisation -----------------------------------------------------
    def to(self, where: str) -> "Tensor":
        st = self._storage
        if where in ("npu", "cuda", "gpu"):
            if st.host_only:
                return self
            dev = st.dev
            for s, e in st.host_dirty.take(*self._range):
                dev[s:e].copy_(st.host[s:e], non_blocking=False)
            self.device = "npu"
        elif where == "cpu":
            # refresh the host copy from HBM, except the ranges written on the host since
            # the last upload: those are newer and stay for the next to("npu") (IRON's
            # decode pass writes x and the angles, then calls input_buffer.to("cpu"),
            # then runs: llama_npu.py:1177-1188)
            if st.allocated:
                s0, e0 = self._range
                cur = s0
                for a, b in [iv for iv in st.host_dirty.iv if iv[1] > s0 and iv[0] < e0] + [(e0, e0)]:
                    a, b = max(a, s0), min(b, e0)
                    if a > cur:
                        st.host[cur:a].copy_(st.dev[cur:a], non_blocking=False)
                    cur = max(cur, b)
            st.dev_dirty.take(*self._range)
            self.device = "cpu"
        else:
            raise ValueError(f"unknown location {where!r}")
        return self

    def mark_device_written(self) -> None:
        """Kernels rewrote this range: the device copy is authoritative."""
        st = self._storage
        if st.host_only:
            return
        st.host_dirty.take(*self._range)
        st.dev_dirty.add(*self._range)
        self.device = "npu"

    def to_torch(self) -> torch.Tensor:
        if self._storage.allocated:
            self.to("cpu")
        return self._host_view().clone()

    def fill_(self, value) -> "Tensor":
        self.torch_view().fill_(value)
        if _cuda_ok():
            self.to("npu")
        return self

    def __repr__(self) -> str:
        return f"{type(self).__name__}(shape={self.shape}, dtype={self.dtype}, device={self.device})"


class CPUOnlyTensor(Tensor):
    """Host-only buffer for CPU evaluation (the reference dispatch); device syncs are no-ops."""

    _host_only = True


XRTTensor = Tensor
DEFAULT_TENSOR_CLASS = Tensor
