"""The two multi-GPU splits compute what the unsplit path computes.

(a) The sharded layer (``bench.py --gpus N``): ``fpx_prefill_attention`` restricted to each
    rank's (KV group range, query-tile range) of ``bench.partition`` writes disjoint rows and
    heads; together, for N = 2, 4 and 8, the shards reassemble the unsharded output and LSE
    bit for bit. One GPU runs every shard in turn (the shards share nothing, so this is the
    same computation each rank does). So do ranges cut at odd tiles. Each shard's workspace
    starts as NaN bytes, as a rank's fresh workspace may hold anything.
(b) The tensor-parallel model (``exp3_b200.model``, ``evaluate.py:324-345`` for what is timed):
    TP = 2 against TP = 1 on the same seed, with one KV head over two ranks and a 3-head group
    split 2 + 1 (the split-group path that Qwen2.5-7B takes at 8 GPUs as 4 + 3). Last-token
    prefill logits and four teacher-forced decode steps agree within ``close()``, and the
    greedy tokens agree except at a near-tie of the TP = 1 logits.
"""

import datetime
import importlib.util
import os
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

from exp3_b200 import ops, synthetic
from exp3_b200._capi import STAGE_ROUTE

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]
two_gpus = pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                              reason="needs two GPUs (one process per rank)")


def _bench():
    spec = importlib.util.spec_from_file_location("bench_for_sharding", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.mark.parametrize("method", ["mean_native", "cgf_mean", "fp_v1_rescue"])
def test_layer_shards_reassemble_the_unsharded_output(method):
    bench = _bench()
    dev = torch.device("cuda", 0)
    length, heads, kv_heads, d = 8192, 28, 4, 128
    blocks, group, scale = length // 128, heads // kv_heads, d ** -0.5
    shape = synthetic.LayerShape(1, length, heads, kv_heads)
    q, k, v = synthetic.attention_inputs(shape, seed=21, needles=8, device=dev, structured_sigma=0.5)
    lse_full = torch.empty(1, length, heads, device=dev)
    # Every workspace starts as NaN bytes: no stage may read what it did not write in the same call.
    ws = torch.full((ops.workspace_bytes(method, 1, length, heads, kv_heads, d),), 0xFF, dtype=torch.uint8, device=dev)
    full = ops.prefill_attention(q, k, v, method, 0.08, scale, lse=lse_full, ws=ws)
    selected, _, _ = ops.export_routing(method, 1, length, heads, kv_heads, ws=ws, device=dev)
    density = float(selected.sum()) / (heads * blocks * (blocks + 1) / 2)
    assert density < 0.99  # the structured inputs drop blocks, so the tails run
    costs = bench.cta_costs(selected, group)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    for world in (2, 4, 8):
        out = torch.full_like(full, float("nan"))
        lse = torch.full_like(lse_full, float("nan"))
        for rank in range(world):
            kv_range, tile_range = bench.partition(rank, world, kv_heads, blocks, costs=costs, sms=sms)
            shard_ws = torch.full_like(ws, 0xFF)
            ops.prefill_attention(q, k, v, method, 0.08, scale, out=out, lse=lse, ws=shard_ws,
                                  kv_range=kv_range, tile_range=tile_range)
        torch.cuda.synchronize()
        assert torch.equal(out.view(torch.int16), full.view(torch.int16)), (world, _differs(out, full, lse, lse_full))
        assert torch.equal(lse, lse_full), (world, _differs(out, full, lse, lse_full))
    # Ranges of odd length, of one tile, and starting at an odd tile: the exact kernel pairs the
    # odd head's tiles from the top of each range, so each split pairs different tiles; a tile's
    # result does not depend on the tile it shares a CTA with.
    out = torch.full_like(full, float("nan"))
    lse = torch.full_like(lse_full, float("nan"))
    for tile_range in ((0, 37), (37, 38), (38, 41), (41, blocks)):
        shard_ws = torch.full_like(ws, 0xFF)
        ops.prefill_attention(q, k, v, method, 0.08, scale, out=out, lse=lse, ws=shard_ws,
                              kv_range=(0, kv_heads), tile_range=tile_range)
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), full.view(torch.int16)), _differs(out, full, lse, lse_full)
    assert torch.equal(lse, lse_full), _differs(out, full, lse, lse_full)
    # the routing of one shard alone equals the unsharded routing on its tiles and heads
    kv_range, tile_range = bench.partition(1, 8, kv_heads, blocks, costs=costs, sms=sms)
    shard_ws = torch.zeros_like(ws)
    ops.prefill_attention(q, k, v, method, 0.08, scale, out=torch.empty_like(full), ws=shard_ws,
                          kv_range=kv_range, tile_range=tile_range, stages=STAGE_ROUTE)
    sel_shard, _, _ = ops.export_routing(method, 1, length, heads, kv_heads, ws=shard_ws, device=dev)
    h0, h1 = kv_range[0] * group, kv_range[1] * group
    t0, t1 = tile_range
    assert torch.equal(sel_shard[:, t0:t1, :, h0:h1], selected[:, t0:t1, :, h0:h1])


def _differs(out, full, lse, lse_full):
    """Where a reassembled output differs from the unsharded one: (rows, query tiles, heads)."""
    rows = ((out.view(torch.int16) != full.view(torch.int16)).any(-1) | (lse != lse_full)).nonzero()
    return rows.shape[0], sorted({int(t) for t in rows[:, 1] // 128}), sorted({int(h) for h in rows[:, 2]})


def _close(a, b, rel=3e-2):
    err = (a - b).abs().max().item()
    scale = b.abs().max().item()
    cos = torch.nn.functional.cosine_similarity(a.flatten(), b.flatten(), dim=0).item()
    return err <= rel * scale + 1e-3 and cos > 0.999, (err, scale, cos)


def _same_token(a, b, err):
    """argmax(a) == argmax(b), or b's top two logits lie within the observed logit error."""
    if int(a.argmax()) == int(b.argmax()):
        return True
    top = b.topk(2).values
    return float(top[0] - top[1]) <= 2 * err


def _tp_rank(rank, world, port, q):
    import torch.distributed as dist

    from exp3_b200.model import AttentionSettings, Qwen2Config, Qwen2Model
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    result = None
    try:
        # one KV head, a 3-head group: at TP = 2 rank 0 holds query heads 0-1, rank 1 head 2
        cfg = Qwen2Config(vocab_size=512, hidden_size=384, intermediate_size=1024, num_hidden_layers=2,
                          num_attention_heads=3, num_key_value_heads=1)
        ids = torch.randint(0, cfg.vocab_size, (1500,), generator=torch.Generator().manual_seed(12)).to(dev)
        settings = AttentionSettings("mean_native", 0.08)
        single = Qwen2Model(cfg, device=dev, seed=13, attention=settings)
        checks = []
        # TP = 2 as one pass per layer, and as the 4-chunk pipeline with overlapped all-reduces
        for chunks in (1, 4):
            split = Qwen2Model(cfg, device=dev, seed=13, tp_rank=rank, tp_size=world, attention=settings)
            split.prefill_chunks = chunks
            assert split.qh == ([0, 1] if rank == 0 else [2])
            with torch.inference_mode():
                ref = single.prefill_logits(ids, max_new_tokens=8)
                got = split.prefill_logits(ids, max_new_tokens=8)
                for step in range(5):
                    ok, (err, _, _) = _close(got, ref)
                    checks.append((chunks, step, ok and _same_token(got, ref, err), err))
                    if step == 4:
                        break
                    token = ref.argmax().view(1)  # teacher-forced: both models decode the TP = 1 token
                    ref = single._forward(token, single.length, decoding=True)
                    single.length += 1
                    got = split._forward(token, split.length, decoding=True)
                    split.length += 1
        result = True if all(c[2] for c in checks) else checks
    except Exception as exc:  # reported to the parent, which fails the test
        result = repr(exc)
    finally:
        dist.destroy_process_group()
    q.put((rank, result))


@two_gpus
def test_tp2_model_matches_tp1_with_a_split_query_group():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_tp_rank, args=(r, 2, 29583, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert results == {0: True, 1: True}
