"""CPU checks of the full-model host logic: tensor-parallel partitions and weight sharding,
and (gloo, world size 2) that row-parallel partial outputs all-reduce to the full projection."""

import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from exp3_b200.model import QWEN25_7B, LayerWeights, Qwen2Config, ffn_partition, head_partition, synthetic_prompt

TINY = Qwen2Config(vocab_size=64, hidden_size=512, intermediate_size=256, num_hidden_layers=1,
                   num_attention_heads=12, num_key_value_heads=2)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_head_partition_covers_every_head_once(world):
    seen, kv_owners = [], {}
    for rank in range(world):
        kv, qh = head_partition(QWEN25_7B, rank, world)
        seen += qh
        for k in kv:
            kv_owners.setdefault(k, []).append(rank)
        group = QWEN25_7B.num_attention_heads // QWEN25_7B.num_key_value_heads
        assert all(h // group in kv for h in qh)  # a rank only holds query heads of its KV heads
    assert sorted(seen) == list(range(28))
    if world == 8:  # each KV head on two ranks, 7 query heads split 4 + 3
        assert all(len(r) == 2 for r in kv_owners.values())
        assert [len(head_partition(QWEN25_7B, r, 8)[1]) for r in range(8)] == [4, 3] * 4


def test_ffn_partition_and_uneven_splits():
    assert [ffn_partition(QWEN25_7B, r, 8) for r in (0, 7)] == [(0, 2368), (16576, 18944)]
    with pytest.raises(ValueError):
        head_partition(QWEN25_7B, 0, 3)


def test_sharded_weights_reassemble():
    full = LayerWeights(TINY, 0, 5, "cpu", [0, 1], list(range(12)), (0, 256))
    parts = [LayerWeights(TINY, 0, 5, "cpu", *head_partition(TINY, r, 4), ffn_partition(TINY, r, 4))
             for r in range(4)]
    d = 128
    q_full = full.w_qkv[: 12 * d]
    q_parts = torch.cat([p.w_qkv[: len(head_partition(TINY, r, 4)[1]) * d] for r, p in enumerate(parts)])
    assert torch.equal(q_parts, q_full)
    assert torch.equal(torch.cat([p.w_o for p in parts], dim=1), full.w_o)
    assert torch.equal(torch.cat([p.w_down for p in parts], dim=1), full.w_down)
    gate = torch.cat([p.w_gu[: p.w_gu.shape[0] // 2] for p in parts])
    assert torch.equal(gate, full.w_gu[:256])


def _row_parallel_rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        full = LayerWeights(TINY, 0, 5, "cpu", [0, 1], list(range(12)), (0, 256))
        kv, qh = head_partition(TINY, rank, world)
        mine = LayerWeights(TINY, 0, 5, "cpu", kv, qh, ffn_partition(TINY, rank, world))
        g = torch.Generator().manual_seed(0)
        attn = torch.randn(6, 12 * 128, generator=g)
        act = torch.randn(6, 256, generator=g)
        cols = torch.cat([torch.arange(h * 128, (h + 1) * 128) for h in qh])
        f0, f1 = ffn_partition(TINY, rank, world)
        o = attn[:, cols] @ mine.w_o.float().t()
        down = act[:, f0:f1] @ mine.w_down.float().t()
        dist.all_reduce(o)
        dist.all_reduce(down)
        ok = torch.allclose(o, attn @ full.w_o.float().t(), atol=1e-3) and \
            torch.allclose(down, act @ full.w_down.float().t(), atol=1e-3)
        q.put((rank, ok))
    finally:
        dist.destroy_process_group()


def test_row_parallel_allreduce_gloo_world2():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_row_parallel_rank, args=(r, 2, 29531, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert results == {0: True, 1: True}


def test_synthetic_prompt_plants_repeated_spans():
    ids = synthetic_prompt(4096, vocab=1000, spans=8, span_len=16, seed=1)
    assert ids.shape == (4096,) and int(ids.max()) < 1000
    assert torch.equal(ids, synthetic_prompt(4096, vocab=1000, spans=8, span_len=16, seed=1))



def test_vocab_sharded_lm_head_reassembles():
    """Under tensor parallelism each rank holds vocab / N rows of the LM head; the shards,
    concatenated in rank order (the all-gather's order), are the replicated head."""
    from exp3_b200.model import Qwen2Model
    full = Qwen2Model(TINY, device="cpu", seed=3)
    assert not full.vocab_sharded
    for world in (2, 4):
        shards = [Qwen2Model(TINY, device="cpu", seed=3, tp_rank=r, tp_size=world) for r in range(world)]
        assert all(m.vocab_sharded for m in shards)
        assert torch.equal(torch.cat([m.lm_head for m in shards]), full.lm_head)


@pytest.mark.parametrize("length,chunks", [(32640, 4), (1500, 4), (100, 4), (129, 8), (32640, 1)])
def test_prefill_pipeline_chunks_are_whole_tiles_covering_every_row(length, chunks):
    """The tensor-parallel prefill pipeline's row chunks: contiguous, in order, every boundary
    on a 128-row tile (so each chunk's attention is a tile range), together every row once."""
    from exp3_b200.model import Qwen2Model
    model = Qwen2Model.__new__(Qwen2Model)  # host logic only: no weights
    model.prefill_chunks = chunks
    bounds = model._chunk_bounds(length)
    tiles = (length + 127) // 128
    assert 1 <= len(bounds) <= min(chunks, tiles)
    assert bounds[0][0] == 0 and bounds[-1][1] == length
    for (a0, a1), (b0, b1) in zip(bounds, bounds[1:]):
        assert a1 == b0
    assert all(r0 % 128 == 0 and r0 < r1 for r0, r1 in bounds)
