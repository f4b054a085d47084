#!/usr/bin/env python3
"""Benchmark of the IRON hot path on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload int4_gemv|bf16_gemv] [--n-vec B]

Workloads:
  int4_gemv (default, config 2): y = dequant(W) x, W [8192 x 2048] signed int4 with
      a bf16 scale per 32 k, x [B x 2048] bf16. One step = one GEMV call.
  bf16_gemv (config 1): W [2048 x 8192] bf16, x [8192].

Timing: W warm-up steps, then exactly K steps bracketed by a barrier and
cuda.synchronize, timed with CUDA events on the launching stream; the step loop
is a captured CUDA graph (one kernel per step, launched with programmatic
dependent launch so each GEMV streams its weights while the previous one
drains). Step i uses weight copy i mod R; the R copies span > 2x the 126 MB L2,
so every step reads its weights from HBM. With N > 1 (torchrun), every rank runs
the same workload on its own GPU (data-parallel replicas, no collective in the
step); value = all ranks' bytes / max-over-ranks time.

`--impl reference` times IRON's CPU path for the same workload on the host cores
(the oracle port of IRON's goldens: restated dequant, then torch `A @ B`).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np
import torch

REPO = Path(__file__).resolve().parent
L2_BYTES = 126 * 1024 * 1024
FALLBACK_HBM_GBS = 6650.0


def _args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20000)
    ap.add_argument("--warmup", type=int, default=200)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["int4_gemv", "bf16_gemv"], default="int4_gemv")
    ap.add_argument("--n-vec", type=int, default=1)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-pdl", action="store_true", help="launch without programmatic dependent launch")
    return ap.parse_args()


# ---- distributed plumbing ------------------------------------------------------
def _dist_init(n):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def _barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def _max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---- clocks during the timed region --------------------------------------------
class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.t0 = self.t1 = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._th = threading.Thread(target=self._read, daemon=True)
            self._th.start()
        except (OSError, FileNotFoundError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def mark(self, which):
        setattr(self, which, time.time())

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.12)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for ts, line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((ts, float(parts[1]), float(parts[2]), parts[5:9]))
            except ValueError:
                continue
        if not rows:
            return None
        inside = [r for r in rows if self.t0 is not None and self.t0 - 0.06 <= r[0] <= self.t1 + 0.06]
        use = inside or rows
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in use for n, v in zip(names, r[3]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[1] for r in use),
                "sm_max_mhz": max(r[2] for r in use), "reasons": reasons,
                "samples": len(use), "in_timed_region": bool(inside)}


def _peak_hbm():
    p = REPO / "MEASURED_PEAKS.json"
    try:
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def _profile_traffic(key: str):
    """DRAM bytes per launch from the committed ncu summary, if one exists."""
    p = REPO / "profiles" / "traffic.json"
    try:
        return json.loads(p.read_text()).get(key)
    except Exception:
        return None


# ---- workloads -------------------------------------------------------------------
class Int4Gemv:
    """signed int4 g32 W [N x K], x [B x K] -> y [B x N]."""

    N, K = 8192, 2048

    def __init__(self, n_vec: int, seed: int = 42):
        self.n_vec = n_vec
        self.bytes_per_step = self.N * self.K // 2 + self.N * (self.K // 32) * 2 + 2 * n_vec * (self.K + self.N)
        self.flops_per_step = 2 * self.N * self.K * n_vec
        self.weight_bytes = self.N * self.K // 2 + self.N * (self.K // 32) * 2
        self.seed = seed

    def config(self):
        return {"workload": "int4_gemv (BASELINE config 2)", "N": self.N, "K": self.K,
                "n_vec": self.n_vec, "group": 32, "weights": "signed int4 ~U{-8..7}, bf16 scales ~U[0.005,0.02]",
                "x": "bf16 ~N(0,1)"}

    def host_inputs(self):
        from oracle import quant  # bench's CPU legs only

        codes, sbits, _ = quant.make_s4g32(self.N, self.K, seed=self.seed)
        rng = np.random.default_rng(self.seed + 1)
        x = rng.standard_normal((self.n_vec, self.K)).astype(np.float32)
        return codes, sbits, x


def _make_int4_device(wl: Int4Gemv, copies: int):
    """R weight copies on the device, generated on the device (rotation for L2)."""
    g = torch.Generator(device="cuda")
    g.manual_seed(wl.seed)
    codes = torch.randint(0, 256, (copies, wl.N, wl.K // 2), dtype=torch.uint8, device="cuda", generator=g)
    s = torch.rand((copies, wl.N, wl.K // 32), device="cuda", generator=g) * 0.015 + 0.005
    scales = s.to(torch.bfloat16)
    x = torch.randn(wl.n_vec, wl.K, device="cuda", generator=g).to(torch.bfloat16)
    y = torch.empty(wl.n_vec, wl.N, dtype=torch.bfloat16, device="cuda")
    return codes, scales, x, y


def run_ours(args, world, rank, local):
    from iron_b200 import _lib
    from iron_b200.operators import GEMV

    lib = _lib.load()
    pdl_flag = 0 if args.no_pdl else _lib.IRON_FLAG_PDL
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    sp = stream.cuda_stream
    if args.workload == "int4_gemv":
        wl = Int4Gemv(args.n_vec)
        copies = max(2, -(-3 * L2_BYTES // wl.weight_bytes))
        codes, scales, x, y = _make_int4_device(wl, copies)
        N, K, nv = wl.N, wl.K, wl.n_vec
        packed = torch.stack([GEMV.pack_int4g32(codes[j], scales[j]) for j in range(copies)])
        pp, xp, yp = packed.data_ptr(), x.data_ptr(), y.data_ptr()
        pstride = packed[0].numel()

        def launch(i, flags=None):
            flags = pdl_flag if flags is None else flags
            j = i % copies
            return lib.iron_gemv_int4g32(pp + j * pstride, xp, yp, N, K, nv, None, flags, sp)

        kernel_key = "gemv_s4g32_stream_kernel"
    else:
        M, K = 2048, 8192
        wl = Int4Gemv(1)
        wl.bytes_per_step = 2 * M * K + 2 * K + 2 * M
        wl.flops_per_step = 2 * M * K
        wl.weight_bytes = 2 * M * K
        wl.config = lambda: {"workload": "bf16_gemv (BASELINE config 1)", "M": M, "K": K}
        copies = max(2, -(-3 * L2_BYTES // wl.weight_bytes))
        g = torch.Generator(device="cuda")
        g.manual_seed(42)
        W = (torch.randn(copies, M, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
        x = torch.randn(K, device="cuda", generator=g).to(torch.bfloat16)
        y = torch.empty(M, dtype=torch.bfloat16, device="cuda")
        wp, xp, yp, wst = W.data_ptr(), x.data_ptr(), y.data_ptr(), M * K * 2

        def launch(i, flags=None):
            flags = pdl_flag if flags is None else flags
            return lib.iron_gemv_bf16(wp + (i % copies) * wst, xp, yp, M, K, K, 1, 0, 0, 0, 1,
                                      None, 0, flags, sp)

        kernel_key = "gemv_bf16_kernel"

    # correctness guard on the exact bench inputs (first copy) before timing
    _check_first_copy(args, wl, locals())

    def capture(n):
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for i in range(n):
                st = launch(i)
                if st != 0:
                    raise RuntimeError(_lib.strerror(st))
        return graph

    per_graph = copies * max(1, 256 // copies)
    g_full = capture(per_graph)
    tail = args.steps % per_graph
    g_tail = capture(tail) if tail else None
    full_reps = args.steps // per_graph

    for _ in range(max(1, -(-args.warmup // per_graph))):
        g_full.replay()
    torch.cuda.synchronize()

    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    _barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if sampler:
        sampler.mark("t0")
    e0.record(stream)
    for _ in range(full_reps):
        g_full.replay()
    if g_tail is not None:
        g_tail.replay()
    e1.record(stream)
    e1.synchronize()
    if sampler:
        sampler.mark("t1")
    torch.cuda.synchronize()
    _barrier(world)
    ms = e0.elapsed_time(e1)
    ms_max = _max_over_ranks(ms, world)
    clocks = sampler.stop() if sampler else None

    # e2e: the public operator API with host buffers, copies inside the timed region
    e2e = _e2e(args, wl, locals())

    steps = args.steps
    per_step_ms = ms_max / steps
    value = wl.bytes_per_step * steps * world / (ms_max * 1e-3) / 1e9
    achieved = wl.bytes_per_step / (ms / steps * 1e-3) / 1e9
    peak, peak_kind = _peak_hbm()
    traffic = _profile_traffic(f"{kernel_key}:{args.workload}:nv{getattr(wl, 'n_vec', 1)}")
    line = {
        "metric": "int4 GEMV achieved HBM GB/s" if args.workload == "int4_gemv" else "bf16 GEMV achieved HBM GB/s",
        "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": steps,
        "warmup": args.warmup, "ms_per_step": per_step_ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16 (int4 weights dequantized exactly, fp32 accumulate)"
        if args.workload == "int4_gemv" else "bf16 (fp32 accumulate)",
        "data": "synthetic (seeded, on device)",
        "config": dict(wl.config(), l2="rotating %d weight copies (%.0f MB > 2x L2)" % (
            copies, copies * wl.weight_bytes / 1e6), parallelism=f"dp{world} (independent replicas)"),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": traffic,
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                     else "fallback 6650 GB/s", "algorithmic_bytes_per_launch": wl.bytes_per_step},
        "gpu_launches": steps,
        "e2e": e2e,
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args, wl, budget_s=10.0)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        del g_full, g_tail
        dist.destroy_process_group()


def _check_first_copy(args, wl, env):
    """Refuse to time a kernel whose output on the bench's own inputs is wrong."""
    from iron_b200 import _lib

    st = env["launch"](0, 0)
    if st != 0:
        raise RuntimeError(_lib.strerror(st))
    torch.cuda.synchronize()
    y = env["y"].float().cpu()
    if args.workload == "int4_gemv":
        codes = env["codes"][0]
        sc = env["scales"][0].float()
        c = codes.to(torch.int16)
        lo = ((c & 0xF) ^ 8) - 8
        hi = (((c >> 4) & 0xF) ^ 8) - 8
        q = torch.stack([lo, hi], -1).reshape(codes.shape[0], -1).float()
        W = (q * sc.repeat_interleave(32, dim=-1)).to(torch.bfloat16).float()
        ref = (env["x"].float() @ W.T).cpu()
    else:
        ref = (env["W"][0].float() @ env["x"].float()).cpu()
    err = (y - ref).abs().max().item()
    bound = 1e-2 + 2e-2 * ref.abs().max().item()
    if not err <= bound:
        raise RuntimeError(f"bench self-check failed: max |err| {err} > {bound}")


def _e2e(args, wl, env):
    """Same metric through the operator API: pinned host x in, host y out, per step."""
    from iron_b200.operators import GEMV

    steps = min(args.steps, 2000)
    if args.workload == "int4_gemv":
        op = GEMV(M=wl.N, K=wl.K, weight_dtype="int4g32", n_vec=wl.n_vec)
        fn = op.get_callable()
        packed = env["packed"]
        x_host = env["x"].cpu().pin_memory()
        y_host = torch.empty(tuple(env["y"].shape), dtype=torch.bfloat16).pin_memory()
        x_dev = torch.empty_like(env["x"])
        y_dev = torch.empty_like(env["y"])
        copies = packed.shape[0]

        def step(i):
            x_dev.copy_(x_host, non_blocking=True)
            j = i % copies
            fn(packed[j], x_dev if wl.n_vec > 1 else x_dev[0], y_dev if wl.n_vec > 1 else y_dev[0])
            y_host.copy_(y_dev, non_blocking=True)
    else:
        M, K = env["M"], env["K"]
        op = GEMV(M=M, K=K)
        fn = op.get_callable()
        W = env["W"]
        x_host = env["x"].cpu().pin_memory()
        y_host = torch.empty(M, dtype=torch.bfloat16).pin_memory()
        x_dev, y_dev = torch.empty_like(env["x"]), torch.empty_like(env["y"])

        def step(i):
            x_dev.copy_(x_host, non_blocking=True)
            fn(W[i % W.shape[0]], x_dev, y_dev)
            y_host.copy_(y_dev, non_blocking=True)

    for i in range(20):
        step(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(steps):
        step(i)
    e1.record()
    e1.synchronize()
    ms = e0.elapsed_time(e1)
    return {"value": round(wl.bytes_per_step * steps / (ms * 1e-3) / 1e9, 1), "unit": "GB/s",
            "h2d_bytes_per_step": int(x_host.numel() * 2), "d2h_bytes_per_step": int(y_host.numel() * 2),
            "steps": steps, "ms_per_step": ms / steps,
            "path": "iron_b200.operators.GEMV callable (ctypes C-ABI), pinned host buffers"}


# ---- CPU legs ----------------------------------------------------------------------
def _cpu_step_fn(args, wl):
    """IRON's CPU path for the workload: restated dequant (oracle) then torch A @ B."""
    from oracle import ops, quant

    if args.workload == "int4_gemv":
        codes, sbits, x = wl.host_inputs()
        xb = torch.from_numpy(x).to(torch.bfloat16)

        def step():
            W = torch.from_numpy(quant.dequant_s4g32(codes, sbits).view(np.int16)).view(torch.bfloat16)
            return ops.gemv_multi(W, xb)

        return step, "restated dequant (numpy) + torch fp32 matmul, config-2 shape, one GEMV per step"
    M, K = 2048, 8192
    g = torch.Generator()
    g.manual_seed(42)
    A = (torch.randn(M, K, generator=g) * 0.02).to(torch.bfloat16)
    B = torch.randn(K, generator=g).to(torch.bfloat16)

    def step():
        return A @ B  # gemv/reference.py:9-11

    return step, "iron gemv golden A @ B (torch bf16), config-1 shape, one GEMV per step"


def cpu_baseline(args, wl, budget_s=10.0):
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    step, desc = _cpu_step_fn(args, wl)
    step()
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < budget_s:
        step()
        n += 1
    dt = (time.perf_counter() - t0) / n
    return {"value": round(wl.bytes_per_step / dt / 1e9, 3), "unit": "GB/s", "cores": threads,
            "kind": "port", "sample": f"{n} steps in {budget_s:.0f} s: {desc}",
            "ms_per_step": dt * 1e3}


def run_reference(args, world, rank):
    if rank != 0:
        return
    wl = Int4Gemv(args.n_vec)
    if args.workload == "bf16_gemv":
        wl.bytes_per_step = 2 * 2048 * 8192 + 2 * 8192 + 2 * 2048
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    step, desc = _cpu_step_fn(args, wl)
    steps = max(1, min(args.steps, 20))
    for _ in range(max(1, min(args.warmup, 3))):
        step()
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    dt = (time.perf_counter() - t0) / steps
    value = round(wl.bytes_per_step / dt / 1e9, 3)
    line = {
        "impl": "reference",
        "metric": "int4 GEMV achieved HBM GB/s" if args.workload == "int4_gemv" else "bf16 GEMV achieved HBM GB/s",
        "value": value, "unit": "GB/s", "n_gpus": world, "steps": steps, "warmup": args.warmup,
        "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (seeded)",
        "config": wl.config() if args.workload == "int4_gemv" else {"workload": "bf16_gemv (BASELINE config 1)"},
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"{steps} steps (requested {args.steps}): {desc}"},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    args = _args()
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, world, rank)
        return
    world, rank, local = _dist_init(args.gpus)
    run_ours(args, world, rank, local)


if __name__ == "__main__":
    sys.path.insert(0, str(REPO))
    main()
