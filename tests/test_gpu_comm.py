"""The one-shot peer-memory all-reduce (fpx_allreduce_bf16) used by the tensor-parallel decode.

On one GPU: a world of one is the identity, and a wait for a peer that never publishes gives
up after its bound, sets the buffer's error word and leaves the input as it was (the second
buffer's flag is simply never written: one kernel, nothing else waits on it). With two or more
GPUs: two ranks (one process each) sum in rank order, bit for bit equal to the fp32 sum rounded
once, also when the calls are captured in a CUDA graph and replayed, and a tensor-parallel
decode with the peer all-reduce yields the same tokens as with NCCL's.
"""

import ctypes
import datetime
import os

import pytest
import torch
import torch.multiprocessing as mp

from exp3_b200._capi import call, lib, ptr, stream

pytestmark = pytest.mark.gpu
two_gpus = pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                              reason="needs two GPUs (ranks that wait on each other never share one)")


def _buffer(max_elems):
    base = ctypes.c_void_p()
    handle = (ctypes.c_char * 64)()
    call("fpx_ar_create", ctypes.c_size_t(lib().fpx_ar_buffer_bytes(max_elems)), ctypes.byref(base), handle)
    return base.value


def test_world_of_one_is_identity_and_a_missing_peer_sets_the_error_word():
    max_elems = 1024
    own, other = _buffer(max_elems), _buffer(max_elems)
    try:
        x = torch.randn(512, device="cuda").bfloat16()
        y = x.clone()
        call("fpx_allreduce_bf16", ptr(y), y.numel(), (ctypes.c_void_p * 1)(own), 0, 1, max_elems, stream(y.device))
        torch.cuda.synchronize()
        assert torch.equal(x, y)
        code = ctypes.c_int(-1)
        call("fpx_ar_error", ctypes.c_void_p(own), ctypes.byref(code))
        assert code.value == 0
        # rank 0 of two; rank 1's flag (the second buffer) is never published
        bases = (ctypes.c_void_p * 2)(own, other)
        for _ in range(2):  # the second call sees the error word and returns at once
            call("fpx_allreduce_bf16", ptr(y), y.numel(), bases, 0, 2, max_elems, stream(y.device))
        torch.cuda.synchronize()
        call("fpx_ar_error", ctypes.c_void_p(own), ctypes.byref(code))
        assert code.value == 1
        assert torch.equal(x, y)
    finally:
        call("fpx_ar_destroy", ctypes.c_void_p(other))
        call("fpx_ar_destroy", ctypes.c_void_p(own))


def test_argument_checks():
    x = torch.zeros(12, device="cuda", dtype=torch.bfloat16)
    bases = (ctypes.c_void_p * 1)(ctypes.c_void_p(x.data_ptr()))
    # 12 values are not a whole number of 16-byte pieces; more ranks than the kernel takes
    assert lib().fpx_allreduce_bf16(ptr(x), 12, bases, 0, 1, 1024, stream(x.device)) != 0
    assert lib().fpx_allreduce_bf16(ptr(x), 8, bases, 0, 9, 1024, stream(x.device)) != 0
    assert lib().fpx_ar_buffer_bytes(12) == 0


def _expected(sizes, world, call_index):
    out = []
    for n in sizes:
        parts = [torch.randn(n, generator=torch.Generator().manual_seed(1000 * call_index + 10 * r + n % 7))
                 .bfloat16() for r in range(world)]
        acc = torch.zeros(n)
        for p in parts:
            acc += p.float()
        out.append((parts, acc.bfloat16()))
    return out


def _ar_rank(rank, world, port, q):
    from exp3_b200.comm import PeerAllReduce
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    ok = True
    try:
        ar = PeerAllReduce(None, dev, max_elems=4096)
        sizes = [8, 3584, 4096]
        for i in range(6):  # eager calls, sizes alternating, both slots used several times
            for parts, want in _expected(sizes, world, i):
                t = parts[rank].to(dev)
                ar.all_reduce_(t)
                ok &= torch.equal(t.cpu(), want)
        # three calls captured once, replayed four times on fresh inputs
        bufs = [torch.empty(n, device=dev, dtype=torch.bfloat16) for n in sizes]
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                for b in bufs:
                    ar.all_reduce_(b)
        torch.cuda.current_stream(dev).wait_stream(s)
        for i in range(10, 14):
            exp = _expected(sizes, world, i)
            for b, (parts, _) in zip(bufs, exp):
                b.copy_(parts[rank].to(dev))
            g.replay()
            torch.cuda.synchronize(dev)
            for b, (_, want) in zip(bufs, exp):
                ok &= torch.equal(b.cpu(), want)
        del g
        ok &= ar.error() == 0
        dist.barrier()
        ar.close()
    except Exception as exc:  # reported to the parent, which fails the test
        ok = repr(exc)
    finally:
        dist.destroy_process_group()
    q.put((rank, ok))


@two_gpus
def test_two_ranks_sum_in_rank_order_eager_and_graph():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_ar_rank, args=(r, 2, 29571, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert results == {0: True, 1: True}


def _tp_decode_rank(rank, world, port, q):
    import torch.distributed as dist
    from exp3_b200.model import AttentionSettings, Qwen2Config, Qwen2Model
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    result = None
    try:
        cfg = Qwen2Config(vocab_size=512, hidden_size=512, intermediate_size=1024, num_hidden_layers=2,
                          num_attention_heads=4, num_key_value_heads=2)
        ids = torch.randint(0, cfg.vocab_size, (600,), generator=torch.Generator().manual_seed(9)).to(dev)
        runs = []
        for peer in (False, True, True):  # NCCL eager, peer eager, peer graph
            m = Qwen2Model(cfg, device=dev, seed=11, tp_rank=rank, tp_size=world,
                           attention=AttentionSettings("mean_native", 0.08))
            m.peer_all_reduce = peer
            with torch.inference_mode():
                first = m.prefill(ids, max_new_tokens=8)
                if len(runs) < 2:
                    toks = [first]
                    for _ in range(7):
                        toks.append(m.decode_step(toks[-1]))
                    runs.append(torch.stack(toks).cpu())
                else:
                    runs.append(m.decode_graph(first, 8).cpu())
            if m._peer_ar is not None:
                assert m._peer_ar.error() == 0
                dist.barrier()
                m._peer_ar.close()
        result = bool(torch.equal(runs[0], runs[1]) and torch.equal(runs[0], runs[2]))
    except Exception as exc:
        result = repr(exc)
    finally:
        dist.destroy_process_group()
    q.put((rank, result))


@two_gpus
def test_tp_decode_with_peer_allreduce_matches_nccl():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_tp_decode_rank, args=(r, 2, 29573, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert results == {0: True, 1: True}
