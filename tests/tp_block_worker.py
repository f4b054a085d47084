"""torchrun worker of tests/test_tp_block_gpu.py: the tensor-parallel block on
WORLD_SIZE GPUs against the single-GPU block on the same weights and inputs."""

import datetime
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), ".."))

from iron_b200.applications.llama3_8b.sharding import BlockShape  # noqa: E402
from iron_b200.applications.llama3_8b.tp_block import TPDecoderBlock  # noqa: E402


def _close(a, b, what, rtol=2e-2, atol=2e-2, max_mismatch_frac=0.0):
    """IRON's tolerance (|a-b| <= max(atol, rtol(|a|+|b|))) with a mismatch fraction.
    Returns the mismatches beyond the allowed fraction."""
    a, b = a.float(), b.float()
    bad = ~((a - b).abs() <= torch.maximum(torch.full_like(a, atol), rtol * (a.abs() + b.abs())))
    n = int(bad.sum())
    n = max(0, n - int(max_mismatch_frac * bad.numel()))
    if n:
        i = int(bad.flatten().nonzero()[0])
        print(f"rank {os.environ['RANK']} {what}: {n} mismatches, first at flat index {i}: "
              f"{float(a.flatten()[i])} vs {float(b.flatten()[i])}", flush=True)
    return n


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", int(os.environ["LOCAL_RANK"])))
    shape, B, L = BlockShape(), 2, 64
    g = torch.Generator(device="cuda").manual_seed(5)
    x0 = torch.randn(B, shape.hidden, device="cuda", generator=g).to(torch.bfloat16)
    kc = torch.randn(B, shape.n_kv, L, shape.head_dim, device="cuda", generator=g).to(torch.bfloat16)
    vc = torch.randn(B, shape.n_kv, L, shape.head_dim, device="cuda", generator=g).to(torch.bfloat16)
    pos = torch.tensor([5, 40], dtype=torch.int32, device="cuda")

    def run(tp, r, group, graph, fused=False):
        blk = TPDecoderBlock(shape, tp, r, B, L, seed=13, group=group, fused_allreduce=fused)
        blk.kc.copy_(kc[:, blk.sh.k0:blk.sh.k1])
        blk.vc.copy_(vc[:, blk.sh.k0:blk.sh.k1])
        blk.x.copy_(x0)
        blk.pos.copy_(pos)
        if graph:
            blk.capture()
        for _ in range(3):  # the peer buffers and flags are reused step after step
            blk.x.copy_(x0)
            blk.pos.copy_(pos)
            blk.step()
        torch.cuda.synchronize()
        blk.check_status()
        out = blk.x.clone()
        kcs = blk.kc.clone()
        blk.release()
        return out, kcs, blk.sh

    failures = 0
    out_1, kc_1, _ = run(1, 0, None, False)
    for graph in (False, True):
        for fused in (False, True):
            out_tp, kc_tp, sh = run(world, rank, None, graph, fused)
            what = f"graph={graph} fused={fused}"
            # NCCL sums bf16 partials ring-wise, rounding to bf16 at every hop (7 times at
            # tp = 8): a few outputs land an ulp or two past the bar, so that path may miss
            # on 0.1 % of them; the fused path sums fp32 partials in rank order, no misses
            failures += _close(out_tp, out_1, what + " out", max_mismatch_frac=0.0 if fused else 1e-3)
            failures += _close(kc_tp, kc_1[:, sh.k0:sh.k1], what + " k cache")
            if fused:  # every rank holds the same sum
                ref = out_tp.clone()
                dist.broadcast(ref, 0)
                n = int((ref != out_tp).sum())
                if n:
                    print(f"rank {rank} {what}: {n} elements differ from rank 0's", flush=True)
                failures += n
    other = torch.tensor([failures], device="cuda")
    dist.all_reduce(other)
    dist.destroy_process_group()
    if rank == 0:
        print(f"tp={world}: {int(other)} mismatching elements")
    sys.exit(0 if int(other) == 0 else 1)


if __name__ == "__main__":
    main()
