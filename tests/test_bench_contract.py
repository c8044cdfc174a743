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


def _bench_module():
    import importlib.util
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_sharding_covers_every_work_unit_once():
    """bench.py's partition: for the layer configs at 1, 2, 4 and 8 ranks, the (KV group, tile
    range) shards cover every (group, tile) exactly once, and the exact-pair counts of the
    shards add up to the layer's (the oracle's accounting formula)."""
    import torch

    import oracle
    bench = _bench_module()
    g = torch.Generator().manual_seed(3)
    for kv_heads, group, blocks, length in ((4, 7, 256, 32768), (8, 5, 64, 8193), (4, 4, 17, 2177)):
        selected = torch.rand(1, blocks, blocks, kv_heads * group, generator=g) < 0.6
        selected &= torch.tril(torch.ones(blocks, blocks, dtype=torch.bool)).view(1, blocks, blocks, 1)
        total = bench.exact_pairs(selected, length, (0, kv_heads), (0, blocks), group)
        assert total == oracle.exact_token_pairs(selected, length)
        for world in (1, 2, 4, 8):
            if world > kv_heads and world % kv_heads:
                continue
            seen = torch.zeros(kv_heads, blocks, dtype=torch.int32)
            pairs = 0
            for rank in range(world):
                kv_range, tile_range = bench.partition(rank, world, kv_heads, blocks)
                seen[kv_range[0]:kv_range[1], tile_range[0]:tile_range[1]] += 1
                pairs += bench.exact_pairs(selected, length, kv_range, tile_range, group)
            assert bool((seen == 1).all()), (kv_heads, blocks, world)
            assert pairs == total


def test_world_sizes_that_leave_work_unowned_are_refused():
    """With 4 KV groups, 3, 5, 6 or 7 ranks would either leave a group unowned or index past
    the last group; partition refuses them instead of reporting work nobody did."""
    import pytest
    bench = _bench_module()
    for world in (3, 5, 6, 7):
        with pytest.raises(ValueError):
            bench.partition(0, world, 4, 256)


def test_tile_cut_fills_whole_waves():
    """Config 2 at 8 ranks (two ranks per KV group): the chosen cut is the one whose simulated
    CTA schedule ends first, so it finishes no later than the causal-work median cut (tile 181
    of 256); and the schedule walks exactly the exact kernel's grid (3 head pairs per tile and
    the odd head's CTA per two tiles)."""
    import torch
    bench = _bench_module()
    nb, group, heads = 256, 7, 28
    selected = torch.tril(torch.ones(nb, nb, dtype=torch.bool)).view(1, nb, nb, 1).expand(1, nb, nb, heads)
    costs = bench.cta_costs(selected.contiguous(), group)
    (_, _), (c0, c1) = bench.partition(0, 8, 4, nb, costs=costs, sms=148)
    assert c0 == 0
    span = lambda cut: max(bench.makespan(costs, (0, 1), (0, cut), 148), bench.makespan(costs, (0, 1), (cut, nb), 148))
    assert span(c1) <= span(181)
    assert span(c1) == min(span(cut) for cut in range(1, nb))
    for t0, t1 in ((0, nb), (c1, nb), (3, 8)):
        tiles = t1 - t0
        assert len(bench.launch_order(costs, (0, 4), (t0, t1))) == 4 * (3 * tiles + (tiles + 1) // 2)
    # the odd head's CTA holds tiles t and t - 1 (the union of their lists), and the lowest tile
    # of an odd range alone
    assert bench.launch_order(costs, (0, 1), (3, 6)) == [6.0] * 3 + [6.0] + [5.0] * 3 + [4.0] * 3 + [
        4.0 * bench.LONE_TILE_CTA_WEIGHT]
    # the two ranks of a group share its tiles exactly
    assert bench.partition(1, 8, 4, nb, costs=costs, sms=148) == ((0, 1), (c1, nb))
