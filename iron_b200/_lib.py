"""ctypes binding of libiron_b200.so (the C ABI declared in include/iron_b200.h).

Loading is lazy and loud: the first kernel call loads the in-tree library and
raises ``RuntimeError`` if it is missing or lacks a symbol. There is no CPU
fallback; every operator's ``get_callable()`` runs the CUDA kernels or fails.
"""

from __future__ import annotations

import ctypes
import threading
from ctypes import c_float, c_int, c_int64, c_uint, c_uint64, c_void_p, c_char_p, c_size_t
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libiron_b200.so"

IRON_OK = 0
IRON_FLAG_PDL = 0x1
IRON_FLAG_SWIGLU = 0x2
IRON_FLAG_X_READONLY = 0x4
(IRON_OK, IRON_ERR_NULL, IRON_ERR_SHAPE, IRON_ERR_ALIGN, IRON_ERR_UNSUPPORTED, IRON_ERR_CUDA,
 IRON_ERR_WORKSPACE, IRON_ERR_TIMEOUT, IRON_ERR_ARG) = (0, -1, -2, -3, -4, -5, -6, -7, -8)
IRON_EPI_NONE = 0
IRON_EPI_GELU = 1
IRON_GEMM_ROUND_FLOOR = 0x100
IRON_GEMM_EPI_SWIGLU = 4

P = c_void_p  # every tensor is passed as a raw device address

# name -> argtypes, in header order. Every function returns int (status) unless
# listed in _RESTYPES.
SIGNATURES: dict[str, list] = {
    "iron_strerror": [c_int],
    "iron_last_cuda_error": [],
    "iron_abi_version": [],
    "iron_gemv_bf16": [P, P, P, c_int, c_int, c_int64, c_int, c_int64, c_int64, c_int64,
                       c_int, P, c_int, c_uint, P],
    "iron_pack_int4g32": [P, P, P, c_int, c_int, P],
    "iron_gemv_int4g32": [P, P, P, c_int, c_int, c_int, P, c_uint, P],
    "iron_dequant_s4g32_rows": [P, P, P, c_int, c_int, P],
    "iron_dequant_u4": [P, P, c_int64, c_int, c_int, P],
    "iron_rmsnorm": [P, P, P, P, P, c_int, c_int, c_float, c_uint, P],
    "iron_rope": [P, P, P, P, c_int, c_int, c_int, P, c_int, c_uint, P],
    "iron_softmax": [P, P, c_int, c_int, c_int, P, c_uint, P],
    "iron_eltwise": [P, P, P, c_int64, c_int, c_uint, P],
    "iron_strided_copy": [P, P, c_int, c_int, P, P, c_int64, c_int, P, P, c_int64, c_int, P, P,
                          c_int64, c_int64, c_uint, P],
    "iron_repeat_interleave": [P, P, c_int64, c_int64, c_int, c_uint, P],
    "iron_transpose": [P, P, c_int, c_int, c_int, c_int, c_uint, P],
    "iron_attn_decode_workspace_bytes": [c_int, c_int, c_int, c_int],
    "iron_attn_decode_workspace_bytes_d": [c_int, c_int, c_int, c_int, c_int],
    "iron_attn_decode": [P, P, P, P, P, c_int, c_int, c_int, c_int, c_int, c_int64, c_int64,
                         c_float, P, c_size_t, c_uint, P],
    "iron_attn_decode_noalloc": [P, P, P, P, P, c_int, c_int, c_int, c_int, c_int, c_int64, c_int64,
                                 c_float, c_uint, P],
    "iron_rope_kv_append": [P, P, P, P, P, P, P, c_int, c_int, c_int, c_int, c_int64, c_int64,
                            c_uint, P],
    "iron_embed": [P, P, P, c_int, c_int, c_int, c_uint, P],
    "iron_argmax": [P, P, c_int, c_int, P, c_uint, P],
    "iron_gemm_bf16": [P, P, P, c_int, c_int, c_int, c_int64, c_int64, c_int64, P, c_int64, c_int, c_int,
                       c_float, c_float, c_int, c_uint, P],
    "iron_gemm_status": [c_int],
    "iron_unpack_int4g32": [P, P, c_int, c_int, P],
    "iron_gemv_int4g32_ex": [P, P, P, c_int, c_int, c_int, P, P, c_float, P, c_uint, P],
    "iron_argmax_finalize": [P, P, P, c_int, c_uint, P],
    "iron_sample_topk": [P, c_int, c_int, c_float, c_int, c_uint64, P, P, c_uint, P],
    "iron_gemv_int4g32_chain": [P, P, P, c_int, c_int, c_int, P, c_uint, P],
    "iron_pack_q4g32": [P, P, P, P, c_int, c_int, P],
    "iron_unpack_q4g32": [P, P, c_int, c_int, P],
    "iron_gemv_q4g32": [P, P, P, c_int, c_int, c_int, P, c_uint, P],
    "iron_embed_chain": [P, P, P, P, P, P, c_int, c_int, c_int, c_uint, P],
    "iron_l2_prefetch": [P, c_size_t, c_uint, P],
    "iron_attn_decode_kernels": [c_int, c_int, c_int, c_int],
    "iron_gemv_int4g32_allreduce": [P, P, P, c_int, c_int, c_int, P, P, c_uint, P],
    "iron_ipc_alloc": [c_size_t, P],
    "iron_ipc_free": [P],
    "iron_ipc_handle": [P, P],
    "iron_ipc_open": [P, P],
    "iron_ipc_close": [P],
    "iron_attn_decode_qkv_workspace_bytes": [c_int, c_int, c_int, c_int, c_int],
    "iron_attn_decode_qkv": [P, P, P, P, P, P, c_int, c_int, c_int, c_int, c_int, c_int64, c_int64, c_float, P,
                             c_size_t, c_uint, P],
    "iron_attn_prefill": [P, P, P, P, c_int, c_int, c_int, c_int, c_int, c_int, c_int, P, P, P, c_float, c_int,
                          c_uint, P],
}
_RESTYPES = {"iron_strerror": c_char_p, "iron_attn_decode_workspace_bytes": c_size_t,
             "iron_attn_decode_workspace_bytes_d": c_size_t,
             "iron_attn_decode_qkv_workspace_bytes": c_size_t}

class GemvChain(ctypes.Structure):
    """iron_gemv_chain (include/iron_b200.h): the decode-chain extras of
    iron_gemv_int4g32_chain (pointers as ints, NULL = off)."""

    _fields_ = [("residual", c_void_p), ("ss_in", c_void_p), ("eps", c_float), ("ss_out", c_void_p),
                ("y_weighted", c_void_p), ("weight", c_void_p), ("argmax_keys", c_void_p)]


_lock = threading.Lock()
_lib = None


def load() -> ctypes.CDLL:
    """Load libiron_b200.so once and bind every declared signature."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m iron_b200._build` "
                "(or __graft_entry__.build()). iron_b200 has no CPU fallback."
            )
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, argtypes in SIGNATURES.items():
            try:
                fn = getattr(lib, name)
            except AttributeError as e:  # pragma: no cover - build/header mismatch
                raise RuntimeError(f"{LIB_PATH} does not export {name}") from e
            fn.argtypes = argtypes
            fn.restype = _RESTYPES.get(name, c_int)
        _lib = lib
        return lib


def strerror(status: int) -> str:
    return load().iron_strerror(int(status)).decode()


def check(status: int, fn: str) -> None:
    """Map a non-zero C status to RuntimeError (IRON raises RuntimeError on a failed run)."""
    if status != IRON_OK:
        msg = f"{fn} failed: {strerror(status)} (status {status}"
        if status == -5:
            msg += f", cudaError {load().iron_last_cuda_error()}"
        raise RuntimeError(msg + ")")


def call(fn: str, *args) -> None:
    """Invoke C entry point `fn` and raise on a non-OK status."""
    check(getattr(load(), fn)(*args), fn)


def current_stream() -> int:
    import torch

    return torch.cuda.current_stream().cuda_stream


def dptr(t) -> int:
    """Device address of a CUDA torch tensor (or of an iron_b200 Tensor)."""
    dev = getattr(t, "device_tensor", None)
    if dev is not None:
        t = dev
    if t is None:
        return None
    if not getattr(t, "is_cuda", False):
        raise RuntimeError("iron_b200 kernels take CUDA tensors; got a host tensor")
    return t.data_ptr()
