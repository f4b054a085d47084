"""bench.py's contract on the CPU: the reference arm (IRON's CPU path, timed on the host
cores) prints one JSON line with the keys the driver reads, only rank 0 prints under a
multi-rank launch, and fewer than 3 warm-up steps are refused; the GPU arms' block and
attention lines carry the contract keys (device timing stubbed); with two gloo ranks
every rank's reported time is the max over ranks."""

import json
import os
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
KEYS = {"impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
        "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"}


def _bench(*args, env=None, timeout=240):
    e = dict(os.environ, **(env or {}))
    return subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), *args], cwd=REPO, env=e,
                          capture_output=True, text=True, timeout=timeout)


@pytest.mark.parametrize("workload", ["decode", "bf16_gemv", "int4_gemv", "block", "attention", "tp_block"])
def test_reference_arm_prints_one_contract_line(workload):
    r = _bench("--impl", "reference", "--workload", workload, "--steps", "1", "--warmup", "3")
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    assert KEYS <= set(d), KEYS - set(d)
    assert d["impl"] == "reference" and d["value"] > 0 and d["higher_is_better"] is True
    assert d["cpu_baseline"]["kind"] in ("port", "reference") and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["e2e"]["value"] == d["value"] and d["e2e"]["unit"] == d["unit"]


def test_reference_arm_other_ranks_exit_quietly():
    r = _bench("--impl", "reference", "--workload", "bf16_gemv", "--steps", "1", "--warmup", "3",
               env={"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""


def test_fewer_than_three_warmup_steps_refused():
    r = _bench("--impl", "reference", "--workload", "bf16_gemv", "--steps", "1", "--warmup", "2")
    assert r.returncode != 0
    assert "warmup" in r.stderr


OURS_KEYS = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
             "scaling", "vs_baseline", "dtype", "data", "config", "roofline", "gpu_launches", "clocks", "e2e"}


def _run_line(fn, args, monkeypatch, capsys):
    import bench

    monkeypatch.setattr(bench, "ClockSampler", lambda local: None)
    fn(bench)(args, 1, 0, 0)
    return json.loads(capsys.readouterr().out.strip())


def test_attention_line_keys_and_scaled_traffic(monkeypatch, capsys):
    """The attention line's contract keys, with the device timing replaced by a stub: the
    headline is the last case, its traffic the profiled ratio times its bytes."""
    import bench

    def fake(B, L, args, max_alloc=0):
        return {"B": B, "L_max": L, "sum_len": 1, "us": 10.0, "gbs": 100.0, "bytes": 10 ** 9, "copies": 2,
                "calls_timed": 200}, 200

    monkeypatch.setattr(bench, "_time_attention", fake)
    args = type("A", (), {"attn_case": None, "no_pdl": False})()
    d = _run_line(lambda b: b.run_attention, args, monkeypatch, capsys)
    assert OURS_KEYS <= set(d), OURS_KEYS - set(d)
    assert len(d["cases"]) == 9 and d["config"]["headline_case"] == {"B": 64, "L_max": 32768}
    assert d["gpu_launches"] == 9 * 200 and d["steps"] == 200
    assert abs(d["roofline"]["traffic"] / 10 ** 9 - 1) < 1e-3  # the capture's traffic equals its bytes


def test_block_line_keys(monkeypatch, capsys):
    import bench

    def fake(args, world, local, full, pos, rank):
        return {"steps": 3000, "ms_per_step": 0.04, "bytes_per_step": 113260544,
                "kernels_per_step": 9 if full else 7, "clocks": None}

    monkeypatch.setattr(bench, "_time_block_form", fake)
    args = type("A", (), {"batch": 16, "no_cpu_baseline": True, "warmup": 30})()
    d = _run_line(lambda b: b.run_block, args, monkeypatch, capsys)
    assert OURS_KEYS <= set(d), OURS_KEYS - set(d)
    assert d["gpu_launches"] == 7 * 3000 and len(d["config"]["positions"]) == 16
    assert all(0 <= p < 4096 for p in d["config"]["positions"])
    assert abs(d["value"] - 113260544 / 40e-6 / 1e9) < 0.1


def _rank_max(rank, world, port, out):
    import torch.distributed as dist

    sys.path.insert(0, REPO)
    import bench

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        bench._barrier(world)
        out[rank] = bench._max_over_ranks(1.5 + rank, world)  # each rank's "device time"
        bench._barrier(world)
    finally:
        dist.destroy_process_group()


def test_multi_rank_time_is_the_max_over_ranks():
    """With N > 1 ranks the step time every rank reports is the slowest rank's (two gloo
    ranks standing in for the NCCL group of a GPU run)."""
    import socket

    import torch.multiprocessing as mp

    with socket.socket() as s_:
        s_.bind(("127.0.0.1", 0))
        port = s_.getsockname()[1]
    out = mp.get_context("spawn").Manager().dict()
    mp.spawn(_rank_max, args=(2, port, out), nprocs=2, join=True)
    assert dict(out) == {0: 2.5, 1: 2.5}
