"""Benchmark of the 32K Qwen2.5-7B-shape block-sparse prefill attention layer (config 2).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--method mean_native] [--alpha 0.08] [--variant iid|structured]
                    [--config c2|c4|c5] [--workload layer|model]

One step = one attention layer (route -> exact -> mean + merge) over B=1, L=32768,
H=28, Hkv=4, d=128 synthetic inputs (N(0,1) + RoPE theta 1e6 + 32 needles) already
resident in HBM; Q (235 MB) is larger than L2, so no flush is needed between steps.
``value`` is whole-job effective TFLOP/s = 4 d x exact token pairs (kernels.py:339-350)
over the max-over-ranks step time. With N GPUs (torchrun) the layer's independent work
units — (KV group, query-tile range) — are split across ranks with no collective in the
data path (strong scaling). ``--impl reference`` times the reference algorithm's CPU
restatement (oracle/) on this host's cores on a bounded sample of the same layer.
``--config c4|c5`` runs the 128K layer or the Qwen2.5-32B-shape (B=2, 64K) layer the same way;
``--workload model`` runs the full-model prefill + decode of config 3 (tensor parallel).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
os.environ.setdefault("NCCL_DEBUG", "WARN")

# Rank 0's stdout carries exactly one JSON line. Libraries print to file descriptor 1 on their
# own (NCCL announces its version there), so main() points descriptor 1 at stderr and the JSON
# line is written to a saved duplicate of the real stdout.
_JSON_OUT = None


def quiet_stdout():
    global _JSON_OUT
    sys.stdout.flush()
    _JSON_OUT = os.dup(1)
    os.dup2(2, 1)


def emit(line: dict):
    os.write(_JSON_OUT if _JSON_OUT is not None else 1, (json.dumps(line) + "\n").encode())

SCALE = 128 ** -0.5
# Layer workloads (--config): c2 is the headline; c4 / c5 are BASELINE.json's long-sequence and
# 32B-shape layers, sharded the same way.
LAYER_CONFIGS = {
    "c2": dict(batch=1, length=32768, heads=28, kv_heads=4,
               metric="effective TFLOP/s of the 32K Qwen2.5-7B-shape prefill attention layer",
               workload="config 2: one attention layer, B=1 L=32768 H=28 Hkv=4 d=128 bf16, synthetic N(0,1) "
                        "Q/K/V + RoPE(theta 1e6) + 32 needles"),
    "c4": dict(batch=1, length=131072, heads=28, kv_heads=4,
               metric="effective TFLOP/s of the 128K Qwen2.5-7B-shape prefill attention layer",
               workload="config 4: one attention layer, B=1 L=131072 H=28 Hkv=4 d=128 bf16, synthetic N(0,1) "
                        "Q/K/V + RoPE(theta 1e6) + 128 needles"),
    "c5": dict(batch=2, length=65536, heads=40, kv_heads=8,
               metric="effective TFLOP/s of the 64K Qwen2.5-32B-shape prefill attention layer",
               workload="config 5: one attention layer, B=2 L=65536 H=40 Hkv=8 d=128 bf16, synthetic N(0,1) "
                        "Q/K/V + RoPE(theta 1e6), K row norms log-normal(0, 0.5)"),
    # The reference's head-dim-256 path (check_qwen35_math.py: Qwen3.5-4B full-attention layers,
    # 16 query heads over 4 KV heads), run with fp_v1 as its Qwen3.5 drivers do.
    "q35": dict(batch=1, length=32768, heads=16, kv_heads=4, head_dim=256, method="fp_v1",
                metric="effective TFLOP/s of the 32K Qwen3.5-4B-shape (head dim 256) prefill attention layer",
                workload="head dim 256: one attention layer, B=1 L=32768 H=16 Hkv=4 d=256 bf16, synthetic N(0,1) "
                         "Q/K/V + RoPE(theta 1e6) + 32 needles"),
}
METRIC = LAYER_CONFIGS["c2"]["metric"]
WORKLOAD = LAYER_CONFIGS["c2"]["workload"]


def parse():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--method", default=None, help="default: mean_native (fp_v1 for q35)")
    ap.add_argument("--alpha", type=float, default=0.08)
    ap.add_argument("--variant", default="iid", choices=["iid", "structured"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--exact-kernel", default="tcgen05", choices=["tcgen05", "tcgen05_single", "mma"],
                    help="exact-attention kernel at head dim 128 (head dim 256 always runs tcgen05_single)")
    ap.add_argument("--config", default="c2", choices=sorted(LAYER_CONFIGS),
                    help="layer workload: c2 (32K, the headline), c4 (128K), c5 (32B shape, B=2, 64K), "
                         "q35 (head dim 256, 32K)")
    ap.add_argument("--workload", default="layer", choices=["layer", "model"],
                    help="layer: the 32K attention layer (default); model: full-model prefill + decode")
    ap.add_argument("--prompt-length", type=int, default=32640)
    ap.add_argument("--decode-tokens", type=int, default=128)
    args = ap.parse_args()
    if args.method is None:
        args.method = LAYER_CONFIGS[args.config].get("method", "mean_native")
    return args


def peaks():
    try:
        data = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
        return data["bf16_tflops"], data.get("bf16_tflops_sustained"), data["hbm_gbs"], "measured"
    except (OSError, KeyError, ValueError):
        return 1590.0, 1400.0, 6650.0, "fallback"


def inputs(variant, device, config="c2"):
    from exp3_b200 import synthetic
    kw = {"structured_sigma": 0.5} if variant == "structured" else {}
    return synthetic.config_inputs(config, seed=0, device=device, **kw)


def partition(rank, world, kv_heads, blocks):
    """Rank's (kv_range, tile_range): KV groups first, then causal-work-balanced tile ranges."""
    if world <= kv_heads:
        per = kv_heads // world
        return (rank * per, (rank + 1) * per), (0, blocks)
    parts = world // kv_heads
    kv = rank // parts
    j = rank % parts
    # tile t costs ~ (t + 1): cut where the cumulative causal work reaches j / parts
    cut = lambda i: min(blocks, int(round(blocks * math.sqrt(i / parts))))
    return (kv, kv + 1), (cut(j), cut(j + 1))


def exact_pairs(selected, length, kv_range, tile_range, group, block=128):
    """4 d x pairs numerator (kernels.py:339-350) over the rank's heads and tiles."""
    blocks = selected.shape[1]
    counts = torch.full((blocks,), block, dtype=torch.int64, device=selected.device)
    counts[-1] = length - (blocks - 1) * block
    q_ids = torch.arange(blocks, device=selected.device).view(blocks, 1)
    k_ids = torch.arange(blocks, device=selected.device).view(1, blocks)
    weights = torch.where(k_ids < q_ids, counts.view(-1, 1) * counts.view(1, -1),
                          torch.where(k_ids == q_ids, (counts * (counts + 1) // 2).view(-1, 1), 0))
    h0, h1 = kv_range[0] * group, kv_range[1] * group
    t0, t1 = tile_range
    sub = selected[:, t0:t1, :, h0:h1].to(torch.int64)
    return int((sub * weights[t0:t1].view(1, t1 - t0, blocks, 1)).sum())


class ClockSampler:
    """SM clock and throttle-reason samples taken during the timed region (read only).

    NVML is read every ~2 ms from a thread, so even a region of a few milliseconds gets
    samples; without NVML it falls back to `nvidia-smi -lms 100`. One sample is also taken
    synchronously when the region opens (`mark()`)."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, index):
        self.index, self.rows, self.proc, self.nvml, self.max_mhz = index, [], None, None, None
        self.stop = threading.Event()
        self.opened = False

    def open(self):
        """NVML start-up and a few discarded reads, before the warm-up steps: the first reads of
        a fresh process are slow and must not fall inside the timed region."""
        if self.opened:
            return self
        self.opened = True
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nvml = pynvml
            self.handle = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM))
            for _ in range(3):
                self._nvml_sample()
            self.rows.clear()
        except Exception:
            self.nvml = None
        return self

    def _nvml_sample(self):
        n = self.nvml
        mhz = n.nvmlDeviceGetClockInfo(self.handle, n.NVML_CLOCK_SM)
        bits = n.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
        masks = (n.nvmlClocksEventReasonHwSlowdown, n.nvmlClocksEventReasonHwThermalSlowdown,
                 n.nvmlClocksEventReasonSwThermalSlowdown, n.nvmlClocksEventReasonSwPowerCap)
        self.rows.append((float(mhz), {name for name, m in zip(self.REASONS, masks) if bits & m}))

    def _nvml_loop(self):
        while not self.stop.wait(0.005):
            try:
                self._nvml_sample()
            except Exception:  # a failed read only loses a sample
                pass

    def __enter__(self):
        self.open()
        if self.nvml:
            self.thread = threading.Thread(target=self._nvml_loop, daemon=True)
            self.thread.start()
            return self
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._smi_read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def mark(self):
        if self.nvml:
            try:
                self._nvml_sample()
            except Exception:
                pass

    def _smi_read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9 and parts[1].replace(".", "").isdigit():
                if self.max_mhz is None and parts[2].replace(".", "").isdigit():
                    self.max_mhz = float(parts[2])
                self.rows.append((float(parts[1]), {name for name, val in zip(self.REASONS, parts[5:9])
                                                    if val.lower().startswith("active")}))

    def __exit__(self, *exc):
        self.stop.set()
        if self.nvml:
            self.thread.join(timeout=1)
            try:
                self.nvml.nvmlShutdown()
            except Exception:
                pass
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return None
        reasons = set().union(*(r for _, r in self.rows))
        return {"sm_mhz": statistics.median(m for m, _ in self.rows), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(self.rows),
                "source": "nvml" if self.nvml else "nvidia-smi"}


def cpu_sample_tiles(blocks):
    # a late, a middle and an early tile: the routing + exact + mean work of the whole layer
    # is ~ sum_t (t + 1); these three cover the range of per-tile costs.
    return [blocks - 1, blocks // 2, blocks // 8]


def cpu_baseline(method, alpha, q, k, v, budget_s=15.0, config="c2"):
    """Times the oracle (the reference algorithm restated on the CPU, fp32 like the reference's
    torch code) with all host threads on a bounded sample of query tiles."""
    import oracle
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    blocks = oracle.num_blocks(q.shape[1])
    tiles = cpu_sample_tiles(blocks)
    flops = 0
    elapsed = 0.0
    runs = 0
    while runs == 0 or (elapsed < budget_s and runs < 20):
        t0 = time.perf_counter()
        d = q.shape[-1]
        outs, sel, _ = oracle.prefill_attention_tiles(method, q, k, v, d ** -0.5, alpha, tiles=tiles)
        elapsed += time.perf_counter() - t0
        flops += 4 * d * oracle.exact_token_pairs(sel, q.shape[1])
        runs += 1
    return {"value": flops / elapsed / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"query tiles {tiles} of the {config} layer (L={q.shape[1]}), all {q.shape[2]} heads, "
                      f"{runs} pass(es), {elapsed:.1f} s, oracle/ fp32 torch on {threads} threads"}


def run_reference(args, rank, world):
    if rank != 0:
        return
    q, k, v = inputs(args.variant, "cpu", args.config)
    for _ in range(args.warmup):
        cpu_baseline(args.method, args.alpha, q, k, v, budget_s=0.0, config=args.config)
    values = [cpu_baseline(args.method, args.alpha, q, k, v, budget_s=0.0, config=args.config)
              for _ in range(args.steps)]
    cfg = LAYER_CONFIGS[args.config]
    value = statistics.median(v["value"] for v in values)
    line = {"impl": "reference", "metric": cfg["metric"], "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
            "config": {"workload": cfg["workload"], "method": args.method, "alpha": args.alpha,
                       "variant": args.variant},
            "cpu_baseline": {**values[0], "value": value},
            "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    emit(line)


def run_model(args, rank, world, local):
    """Config 3: random-init Qwen2.5-7B, 32640-token prompt (uniform ids + 64 planted 16-token
    key -> value spans), sparse prefill then 128 dense greedy decode tokens; tensor parallel on N GPUs."""
    import datetime

    import torch.distributed as dist
    from exp3_b200.model import QWEN25_7B, AttentionSettings, Qwen2Model, synthetic_prompt

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)
    model = Qwen2Model(QWEN25_7B, device=dev, seed=0, tp_rank=rank, tp_size=world,
                       attention=AttentionSettings(args.method, args.alpha))
    ids_host = synthetic_prompt(args.prompt_length, QWEN25_7B.vocab_size).pin_memory()
    ids = ids_host.to(dev)
    clocks = ClockSampler(local).open()
    for _ in range(args.warmup):
        model.prefill(ids, args.decode_tokens)
    torch.cuda.synchronize()

    def timed(fn, n):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(n):
            fn()
        b.record()
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / n
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t)
        return ms

    with clocks:
        prefill_ms = timed(lambda: model.prefill(ids, args.decode_tokens), args.steps)
    first = model.prefill(ids, args.decode_tokens)

    def decode_eager():
        model.length = args.prompt_length
        tok = first
        for _ in range(args.decode_tokens - 1):
            tok = model.decode_step(tok)

    def decode_graph():
        model.length = args.prompt_length
        model.decode_graph(first, args.decode_tokens)

    # Per token over the decode_tokens - 1 steps after the prefill's token (evaluate.py:384-400);
    # the graph run includes its one eager warm-up step and the capture.
    decode_eager_ms = timed(decode_eager, 1) / max(1, args.decode_tokens - 1)
    decode_ms = timed(decode_graph, 1) / max(1, args.decode_tokens - 1)
    replay_ms = model.replay_ms_per_token()
    if world > 1 and replay_ms is not None:
        t = torch.tensor([replay_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        replay_ms = float(t)
    # End to end (evaluate.prefill): token ids from pinned host memory, prefill, first token to host.
    result = torch.empty(1, dtype=torch.int64).pin_memory()

    def e2e():
        ids.copy_(ids_host, non_blocking=True)
        result.copy_(model.prefill(ids, args.decode_tokens).view(1), non_blocking=True)

    e2e_ms = timed(e2e, args.steps)
    flops = model.prefill_flops(args.prompt_length)  # linear + all causal attention pairs
    if rank == 0:
        line = {"metric": "full-model prefill latency, Qwen2.5-7B shape, 32640 tokens", "value": prefill_ms,
                "unit": "ms", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": prefill_ms,
                "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic (random-init weights, seeded prompt)",
                "config": {"workload": "config 3: random-init Qwen2.5-7B (28 layers, hidden 3584, 28/4 heads, "
                                       "FFN 18944, vocab 152064), prompt 32640 ids with 64 planted 16-token spans",
                           "method": args.method, "alpha": args.alpha,
                           "parallelism": f"tp{world} (heads / FFN sharded, NCCL all-reduce after o_proj and down)",
                           "prefill_tflops_dense_equivalent": flops / (prefill_ms * 1e-3) / 1e12,
                           "decode_ms_per_token": decode_ms, "decode_ms_per_token_eager": decode_eager_ms,
                           "decode_replay_ms_per_token": replay_ms,
                           "decode": "CUDA-graph steps (Model.decode_graph); decode_ms_per_token includes the "
                                     "eager warm-up step and the capture, decode_replay_ms_per_token is the "
                                     "steady-state replay",
                           "decode_comm": "one-shot peer-memory all-reduce (exp3_b200.comm)" if world > 1 else None,
                           "decode_tokens": args.decode_tokens},
                "e2e": {"value": e2e_ms, "unit": "ms", "h2d_bytes_per_step": ids_host.numel() * 8,
                        "d2h_bytes_per_step": 8},
                "clocks": clocks.summary()}
        emit(line)
    if world > 1:
        model.close_comm()
        dist.barrier()
        dist.destroy_process_group()


def main():
    args = parse()
    quiet_stdout()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", args.gpus))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if args.warmup < 3:
        raise SystemExit("at least 3 warm-up steps")
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if args.workload == "model":
        return run_model(args, rank, world, local)

    import torch.distributed as dist
    from exp3_b200 import ops
    from exp3_b200._capi import STAGE_EXACT, STAGE_MEAN, STAGE_ROUTE
    from exp3_b200.attention import AttentionBackend

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    from exp3_b200 import _capi
    _capi.set_exact_kernel(args.exact_kernel)
    cfg = LAYER_CONFIGS[args.config]
    b, length, heads, kv_heads, d = cfg["batch"], cfg["length"], cfg["heads"], cfg["kv_heads"], cfg.get("head_dim", 128)
    scale = d ** -0.5
    group = heads // kv_heads
    blocks = length // 128
    q, k, v = inputs(args.variant, dev, args.config)
    kv_range, tile_range = partition(rank, world, kv_heads, blocks)
    method, alpha = args.method, args.alpha
    nbytes = ops.workspace_bytes(method, b, length, heads, kv_heads, d)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    out = torch.empty(b, length, heads, d, dtype=torch.bfloat16, device=dev)

    # Selected work of this rank (routing of the full layer, untimed).
    ops.prefill_attention(q, k, v, method, alpha, scale, out=out, ws=ws, stages=STAGE_ROUTE)
    selected, _, _ = ops.export_routing(method, b, length, heads, kv_heads, head_dim=d, ws=ws, device=dev)
    pairs = exact_pairs(selected, length, kv_range, tile_range, group)
    all_pairs = exact_pairs(selected, length, (0, kv_heads), (0, blocks), group)
    density = float(selected.sum()) / (b * heads * blocks * (blocks + 1) / 2)
    flops = 4 * d * pairs
    total_flops = 4 * d * all_pairs
    del selected

    def step(events=None):
        common = dict(out=out, ws=ws, kv_range=kv_range, tile_range=tile_range)
        if events is None:
            ops.prefill_attention(q, k, v, method, alpha, scale, **common)
            return
        events[0].record()
        ops.prefill_attention(q, k, v, method, alpha, scale, stages=STAGE_ROUTE, **common)
        events[1].record()
        ops.prefill_attention(q, k, v, method, alpha, scale, stages=STAGE_EXACT, **common)
        events[2].record()
        ops.prefill_attention(q, k, v, method, alpha, scale, stages=STAGE_MEAN, **common)
        events[3].record()

    clocks = ClockSampler(local).open()
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with clocks:
        start.record()
        for i in range(args.steps):
            step(ev[i])
        clocks.mark()  # the steps are queued: the GPU is running them now
        end.record()
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms_total = start.elapsed_time(end)
    route_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in ev)
    exact_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in ev)
    mean_ms = statistics.mean(e[2].elapsed_time(e[3]) for e in ev)
    ms_step = ms_total / args.steps
    if world > 1:
        t = torch.tensor([ms_step], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_step = float(t)

    # End to end through the public API (AttentionBackend.forward, the attention.py call site)
    # with pinned host buffers: every step copies this rank's Q/K/V in (H2D), runs the layer and
    # reads its output rows back (D2H), all inside the timed region. The steps are pipelined as
    # a serving loop runs them: two device input slots, step i+1's H2D on a copy stream while
    # step i computes, and step i's D2H on a second copy stream while step i+1 computes.
    h0, h1 = kv_range[0] * group, kv_range[1] * group
    t0, t1 = tile_range
    # The pipeline streams work units: one per KV group this rank owns when it owns whole groups
    # (each group is an independent attention problem: its query heads, its K and V), else the
    # rank's tile shard. Per unit, the H2D of the next unit overlaps this unit's compute and the
    # D2H of the previous one, so only one unit's copies are left outside the overlap.
    full_tiles = tile_range == (0, blocks)
    units = [(g, g + 1) for g in range(kv_range[0], kv_range[1])] if full_tiles else [tuple(kv_range)]
    host = [tuple(x.contiguous().cpu().pin_memory() for x in (q[:, :, a * group:c * group], k[:, :, a:c], v[:, :, a:c]))
            for a, c in units]
    slots = 2
    o_hs = [[torch.empty(b, (t1 - t0) * 128, (c - a) * group, d, dtype=torch.bfloat16).pin_memory() for a, c in units]
            for _ in range(slots)]
    dev_in = [[[torch.empty_like(x, device=dev) for x in unit] for unit in host] for _ in range(slots)]
    backend = AttentionBackend(alpha=alpha)
    backend.configure(method)
    compute = torch.cuda.current_stream(dev)
    h2d_stream, d2h_stream = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    class Layer:
        layer_idx = 0

    def e2e_run(n, start=None, end=None):
        in_free = [[None] * len(units) for _ in range(slots)]  # compute has finished reading the slot
        with torch.cuda.stream(h2d_stream):
            if start is not None:
                start.record(h2d_stream)
        for i in range(n):
            sl = i % slots
            for u in range(len(units)):
                qd, kd, vd = dev_in[sl][u]
                with torch.cuda.stream(h2d_stream):
                    if in_free[sl][u] is not None:
                        h2d_stream.wait_event(in_free[sl][u])
                    for dst, src in zip(dev_in[sl][u], host[u]):
                        dst.copy_(src, non_blocking=True)
                    ready = torch.cuda.Event()
                    ready.record(h2d_stream)
                compute.wait_event(ready)
                if full_tiles:
                    o, _ = backend.forward(Layer(), qd.transpose(1, 2), kd.transpose(1, 2), vd.transpose(1, 2), None,
                                           scale)
                else:  # a tile shard: the same fused op with this rank's tile range
                    o = ops.prefill_attention(qd, kd, vd, method, alpha, scale, tile_range=tile_range)
                done = torch.cuda.Event()
                done.record(compute)
                in_free[sl][u] = done
                with torch.cuda.stream(d2h_stream):
                    d2h_stream.wait_event(done)
                    o_hs[sl][u].copy_(o[:, t0 * 128:t1 * 128], non_blocking=True)
                o.record_stream(d2h_stream)
        if end is not None:
            end.record(d2h_stream)

    e2e_run(args.warmup)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2e_run(args.steps, s2, e2)
    torch.cuda.synchronize()
    e2e_ms = s2.elapsed_time(e2) / args.steps
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t)
    h2d = sum(x.numel() * x.element_size() for unit in host for x in unit)
    d2h = sum(o.numel() * o.element_size() for o in o_hs[0])
    if world > 1:
        counts = torch.tensor([float(h2d), float(d2h)], device=dev)
        dist.all_reduce(counts)
        h2d, d2h = int(counts[0]), int(counts[1])

    peak, peak_sus, hbm, peak_kind = peaks()
    achieved = flops / (exact_ms * 1e-3) / 1e12
    traffic = None
    traffic_file = ROOT / "profiles" / "exact_attention_traffic.json"
    if traffic_file.exists():
        try:
            traffic = json.loads(traffic_file.read_text()).get(f"bytes_per_launch_{args.config}")
        except ValueError:
            traffic = None
    launches_per_step = {"dense": 2, "fp_v1": 3}.get(method, 4)
    if method in ("mean_balanced", "cgf_mean", "dispersion_mean") and alpha == 0:
        launches_per_step = 4

    line = None
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline and args.config in ("c2", "q35"):
            qc, kc, vc = q.cpu(), k.cpu(), v.cpu()
            cpu = cpu_baseline(method, alpha, qc, kc, vc, config=args.config)
        line = {
            "metric": cfg["metric"], "value": total_flops / (ms_step * 1e-3) / 1e12, "unit": "TFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": cfg["workload"], "method": method, "alpha": alpha, "variant": args.variant,
                       "exact_kernel": "tcgen05_single" if d == 256 else args.exact_kernel, "ms_per_layer": ms_step, "density": density, "exact_token_pairs": all_pairs,
                       "l2": f"no flush: Q ({q.numel() * 2 / 1e6:.0f} MB) and O are larger than the 126 MB L2",
                       "parallelism": f"{world} rank(s): (KV group x query-tile range) shards, no collective",
                       "stage_ms_rank0": {"route": route_ms, "exact": exact_ms, "mean_merge": mean_ms}},
            "roofline": {"bound": "tensor", "kernel": "exact attention (sparse FA)" + (", d=256" if d == 256 else ""), "achieved": achieved,
                         "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                         "peak_kind": f"{peak_kind} burst bf16", "frac_of_sustained":
                             achieved / peak_sus if peak_sus else None, "traffic": traffic},
            "cpu_baseline": cpu,
            "e2e": {"value": total_flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "pipeline": f"{len(units)} unit(s) per step (KV groups, or the rank's tile shard), 2 input "
                                "slots per unit; H2D / compute / D2H of successive units overlap on 3 streams"},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clocks.summary(),
        }
        emit(line)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
