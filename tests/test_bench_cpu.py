"""bench.py's contract on the CPU: the reference arm (IRON's CPU path, timed on the host
cores) prints one JSON line with the keys the driver reads, only rank 0 prints under a
multi-rank launch, and fewer than 3 warm-up steps are refused."""

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


@pytest.mark.parametrize("workload", ["decode", "bf16_gemv", "int4_gemv", "block", "attention"])
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
