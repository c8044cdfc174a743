"""The bench contract's reference arm on the CPU: `bench.py --impl reference` times the oracle (the
reference algorithm restated) and rank 0 prints exactly one JSON line on stdout with the keys the
driver reads; other ranks print nothing."""

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def run_bench(*args, env_extra=None):
    env = dict(os.environ, **(env_extra or {}))
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], cwd=ROOT, env=env,
                          capture_output=True, text=True, timeout=600)


def test_reference_arm_prints_one_json_line():
    res = run_bench("--impl", "reference", "--steps", "1", "--warmup", "3", "--config", "c2")
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [line for line in res.stdout.splitlines() if line.strip()]
    assert len(lines) == 1, res.stdout
    line = json.loads(lines[0])
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "higher_is_better", "cpu_baseline",
                "e2e", "config"):
        assert key in line, key
    assert line["impl"] == "reference" and line["value"] > 0 and line["unit"] == "TFLOP/s"
    assert line["cpu_baseline"]["cores"] >= 1 and line["cpu_baseline"]["kind"] == "port"
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0


def test_reference_arm_non_zero_ranks_print_nothing():
    res = run_bench("--impl", "reference", "--steps", "1", "--warmup", "3",
                    env_extra={"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert res.returncode == 0, res.stderr[-2000:]
    assert res.stdout.strip() == ""


def test_fewer_than_three_warmups_are_refused():
    res = run_bench("--impl", "reference", "--steps", "1", "--warmup", "1")
    assert res.returncode != 0
