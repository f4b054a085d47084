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


class _Storage:
    """Byte arrays shared by a tensor and its subviews."""

    def __init__(self, nbytes: int):
        self.nbytes = max(int(nbytes), 1)
        pin = _cuda_ok()
        self.host = torch.zeros(self.nbytes, dtype=torch.uint8, pin_memory=pin)
        self._dev = None

    @property
    def dev(self) -> torch.Tensor:
        if self._dev is None:
            if not _cuda_ok():
                raise RuntimeError("no CUDA device: iron_b200 buffers live in B200 HBM")
            self._dev = torch.zeros(self.nbytes, dtype=torch.uint8, device="cuda")
        return self._dev


class Tensor:
    """Explicit-sync host/HBM buffer (the XRTTensor surface on a B200)."""

    def __init__(self, shape, dtype=None, *, _storage=None, _offset=0):
        if dtype is None:
            dtype = _np_bf16
        self.dtype = np_dtype(dtype)
        self.shape = tuple(int(s) for s in (shape if isinstance(shape, (tuple, list)) else (shape,)))
        self._offset = int(_offset)
        self._nbytes = int(np.prod(self.shape, dtype=np.int64)) * self.dtype.itemsize
        self._storage = _storage if _storage is not None else _Storage(self._nbytes)
        if self._offset + self._nbytes > self._storage.nbytes:
            raise ValueError("subview exceeds its parent buffer")
        self.device = "cpu"

    # -- construction --------------------------------------------------------
    @classmethod
    def from_torch(cls, t: torch.Tensor) -> "Tensor":
        t = t.detach()
        out = cls(tuple(t.shape), np_dtype(t.dtype))
        out.torch_view().copy_(t.reshape(out.shape).cpu())
        if _cuda_ok():
            out.to("npu")
        return out

    def subview(self, byte_offset: int, shape, dtype) -> "Tensor":
        sub = Tensor(shape, dtype, _storage=self._storage, _offset=self._offset + int(byte_offset))
        sub.device = self.device
        return sub

    # -- views ---------------------------------------------------------------
    def _bytes(self, t: torch.Tensor) -> torch.Tensor:
        return t[self._offset : self._offset + self._nbytes]

    def torch_view(self) -> torch.Tensor:
        """Host view (what the next ``to("npu")`` uploads)."""
        return self._bytes(self._storage.host).view(torch_dtype(self.dtype)).view(self.shape)

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
        raw = self._bytes(self._storage.host).numpy()
        return raw.view(self.dtype).reshape(self.shape)

    # -- synchronisation -----------------------------------------------------
    def to(self, where: str) -> "Tensor":
        if where in ("npu", "cuda", "gpu"):
            self._bytes(self._storage.dev).copy_(self._bytes(self._storage.host), non_blocking=False)
            self.device = "npu"
        elif where == "cpu":
            src = self._bytes(self._storage.dev)
            self._bytes(self._storage.host).copy_(src, non_blocking=False)
            self.device = "cpu"
        else:
            raise ValueError(f"unknown location {where!r}")
        return self

    def to_torch(self) -> torch.Tensor:
        if self._storage._dev is not None:
            self.to("cpu")
        return self.torch_view().clone()

    def fill_(self, value) -> "Tensor":
        self.torch_view().fill_(value)
        if _cuda_ok():
            self.to("npu")
        return self

    def __repr__(self) -> str:
        return f"Tensor(shape={self.shape}, dtype={self.dtype}, device={self.device})"


XRTTensor = Tensor
DEFAULT_TENSOR_CLASS = Tensor
