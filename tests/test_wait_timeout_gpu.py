"""A bounded device-side wait that runs out, on one GPU, without faulting it.

The fused all-reduce GEMV (iron_gemv_int4g32_allreduce) waits for every rank's fp32
partial of each output tile in its own receive buffer. Launched here as rank 0 of a
world of 2 whose rank 1 never runs, rank 1's slots are never written: each wait gives
up after the caller's limit (iron_allreduce_peers.wait_us), sets the status word and
the kernel finishes with the values it has. The host reads the status the way the
tensor-parallel block does (TPDecoderBlock.check_status raises), and the context stays
usable. This is the analogue of IRON's failed-run check (iron/common/sequence.py:732-736:
a run that does not complete raises RuntimeError).
"""

import ctypes
import time
from types import SimpleNamespace

import pytest
import torch

pytestmark = pytest.mark.gpu

from iron_b200 import _lib
from iron_b200.applications.llama3_8b.tp_block import AllReducePeers, TPDecoderBlock, _DeviceBuffer
from iron_b200.applications.llama_3_2_1b.decode import Int4Matrix


def test_allreduce_wait_runs_out_and_reports():
    N, K, nv = 256, 512, 1
    g = torch.Generator(device="cuda").manual_seed(2)
    W = Int4Matrix(N, K, g, 0.001, 0.004)
    x = torch.randn(nv, K, device="cuda", generator=g).to(torch.bfloat16)
    y = torch.empty(nv, N, dtype=torch.bfloat16, device="cuda")
    y_plain = torch.empty_like(y)
    own = _DeviceBuffer((2, N, nv), "<u8", 8)    # rank 0's receive buffer, zero-filled
    other = _DeviceBuffer((2, N, nv), "<u8", 8)  # stands for rank 1's buffer: nobody reads it
    status = torch.zeros(4, dtype=torch.int32, device="cuda")
    peers = AllReducePeers()
    peers.world, peers.rank = 2, 0
    peers.recv[0], peers.recv[1] = own.ptr, other.ptr
    peers.status = status.data_ptr()
    peers.wait_us = 2000  # 2 ms per wait
    s = _lib.current_stream()
    try:
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        _lib.call("iron_gemv_int4g32_allreduce", W.packed.data_ptr(), x.data_ptr(), y.data_ptr(), N, K, nv, None,
                  ctypes.addressof(peers), 0, s)
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        assert int(status[0]) != 0, "the wait for the missing rank did not report"
        assert dt < 5.0, f"the kernel took {dt:.2f} s to give up"
        # with rank 1's partials missing (zero), each output is this rank's own partial:
        # bitwise the single-GPU GEMV of the same tile order
        _lib.call("iron_gemv_int4g32", W.packed.data_ptr(), x.data_ptr(), y_plain.data_ptr(), N, K, nv, None, 0, s)
        torch.cuda.synchronize()
        assert torch.equal(y, y_plain)
        # the slots the kernel consumed were cleared for the next use
        assert int(own.tensor.count_nonzero()) == 0
        # the host side of the tensor-parallel block reports the status as an error
        blk = object.__new__(TPDecoderBlock)
        blk.fused = True
        blk.site_o = SimpleNamespace(status=status)
        blk.site_d = SimpleNamespace(status=torch.zeros_like(status))
        with pytest.raises(RuntimeError, match="timed out"):
            blk.check_status()
        # the context is still usable: a healthy world-of-1 all-reduce completes with status 0
        status.zero_()
        peers.world = 1
        _lib.call("iron_gemv_int4g32_allreduce", W.packed.data_ptr(), x.data_ptr(), y.data_ptr(), N, K, nv, None,
                  ctypes.addressof(peers), 0, s)
        torch.cuda.synchronize()
        assert int(status[0]) == 0
        assert torch.equal(y, y_plain)
    finally:
        torch.cuda.synchronize()
        own.tensor = None
        other.tensor = None
        own.free()
        other.free()
