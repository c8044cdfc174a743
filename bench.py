"""Benchmark of the 32K Qwen2.5-7B-shape block-sparse prefill attention layer (config 2).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--method mean_native] [--alpha 0.08] [--variant iid|structured]
                    [--config c2|c4|c5|q35] [--workload layer|model]
                    [--no-structured] [--no-model] [--no-reference-gpu] [--no-cpu-baseline]

One step = one attention layer (route -> exact -> mean + merge) over B=1, L=32768,
H=28, Hkv=4, d=128 synthetic inputs (N(0,1) + RoPE theta 1e6 + 32 needles) already
resident in HBM; Q (235 MB) is larger than L2, so no flush is needed between steps.
``value`` is whole-job effective TFLOP/s = 4 d x exact token pairs (kernels.py:339-350)
over the max-over-ranks step time. With N GPUs (torchrun) the layer's independent work
units — (KV group, query-tile range) — are split across ranks with no collective in the
data path (strong scaling). ``--impl reference`` times the reference algorithm's CPU
restatement (oracle/) on this host's cores on a bounded sample of the same layer.

The default config-2 line also carries three sub-records:
- ``structured``: the same layer on the block-structured inputs (sigma 0.5), where the
  routing drops blocks and the block-mean tail does real work;
- ``model``: config 3, the full-model 32640-token prefill (tensor parallel over the N
  GPUs) with its end-to-end latency and graphed decode;
- ``reference_gpu`` (N=1): the reference's own bf16 path (its Triton kernels and torch code,
  installed in baseline/_ref) timed on the same GPU as a black box, beside torch's dense SDPA.
``--config c4|c5|q35`` runs the 128K layer, the Qwen2.5-32B-shape (B=2, 64K) layer or the
head-dim-256 layer the same way; ``--workload model`` prints the full-model line alone.
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
import typing
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
    ap.add_argument("--no-structured", action="store_true", help="skip the structured-inputs sub-record")
    ap.add_argument("--no-model", action="store_true", help="skip the full-model sub-record")
    ap.add_argument("--no-reference-gpu", action="store_true",
                    help="skip timing the reference's own Triton path on the GPU")
    ap.add_argument("--time-reference-gpu", action="store_true", help=argparse.SUPPRESS)
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


# A CTA of the two-tile exact kernel that holds one tile alone (the last tile of a shard's range
# for the odd head of a group, the pairing of that head running tiles t and t - 1 together) runs
# the same per-block chain as a pair: measured at about this fraction of a pair's time.
LONE_TILE_CTA_WEIGHT = 0.94
# Per-CTA set-up and epilogue (TMEM allocation, block-list union, Q load, O store), in blocks.
CTA_OVERHEAD_BLOCKS = 1.0


class CtaCosts(typing.NamedTuple):
    """Costs of the exact kernel's CTAs, in K/V blocks run (CPU float64).

    ``units``: [B, Hkv, U, nb], the CTA of unit u at query tile t: a head pair's union (the
    two-tile kernel, U = G // 2) or one head (the one-tile kernel, U = G). ``odd_own`` and
    ``odd_union``: [B, Hkv, nb] for the two-tile kernel when G is odd, the last head's block
    count at tile t and the union of its tiles t and t - 1 (the CTA that runs both), else None.
    """
    units: torch.Tensor
    odd_own: typing.Optional[torch.Tensor] = None
    odd_union: typing.Optional[torch.Tensor] = None


def cta_costs(selected, group, paired=True):
    """``CtaCosts`` of ``selected`` [B, nb, nb, H] (the routed block mask). ``paired``: the
    two-tile kernel (csrc/attn_tc.cu: head pairs of a KV group at one tile, and the odd head
    at two neighbouring tiles); else one head per CTA (csrc/attn_tc1.cu)."""
    b, nb, _, heads = selected.shape
    hkv = heads // group
    sel = selected.view(b, nb, nb, hkv, group)
    per_tile = lambda m: m.sum(2).to(torch.float64).cpu()  # [B, nb, Hkv]
    if not paired:
        return CtaCosts(sel.sum(2).permute(0, 2, 3, 1).to(torch.float64).cpu())
    units = torch.zeros(b, hkv, group // 2, nb, dtype=torch.float64)
    for j in range(group // 2):
        units[:, :, j, :] = per_tile(sel[..., 2 * j] | sel[..., 2 * j + 1]).permute(0, 2, 1)
    if group % 2 == 0:
        return CtaCosts(units)
    last = sel[..., group - 1]  # [B, nb (query tile), nb (key block), Hkv]
    prev = torch.cat([torch.zeros_like(last[:, :1]), last[:, :-1]], dim=1)  # tile t - 1's row at t
    return CtaCosts(units, per_tile(last).permute(0, 2, 1), per_tile(last | prev).permute(0, 2, 1))


def launch_order(costs, kv_range, tile_range):
    """The exact kernel's CTA costs for one shard in launch order (csrc/attn_tc.cu
    ``exact_unit``; batch slowest, then the tiles longest first, then KV group and unit)."""
    t0, t1 = tile_range
    kv0, kv1 = kv_range
    tiles = list(range(t1 - 1, t0 - 1, -1))
    out = []
    for b in range(costs.units.shape[0]):
        unit_rows = costs.units[b, kv0:kv1].permute(2, 0, 1).reshape(costs.units.shape[3], -1).tolist()
        if costs.odd_own is None:
            for t in tiles:
                out += unit_rows[t]
            continue
        own = costs.odd_own[b, kv0:kv1].t().tolist()
        union = costs.odd_union[b, kv0:kv1].t().tolist()
        for y in range(0, len(tiles), 2):
            ta = tiles[y]
            out += unit_rows[ta]
            if y + 1 < len(tiles):
                out += union[ta]
                out += unit_rows[tiles[y + 1]]
            else:
                out += [c * LONE_TILE_CTA_WEIGHT for c in own[ta]]
    return out


def makespan(costs, kv_range, tile_range, sms):
    """List-schedules the exact kernel's grid on ``sms`` SMs, one CTA per SM, in launch order
    and returns when the last CTA ends, in blocks."""
    import heapq
    if tile_range[1] <= tile_range[0]:
        return 0.0
    free = [0.0] * sms
    for w in launch_order(costs, kv_range, tile_range):
        heapq.heappush(free, heapq.heappop(free) + w + CTA_OVERHEAD_BLOCKS)
    return max(free)


def tile_cuts(costs, kv, parts, blocks, sms):
    """Query-tile cuts [0 = c0 < c1 < ... < c_parts = blocks] of KV group ``kv`` over ``parts``
    ranks. Two parts: the cut that minimises the slower rank's simulated makespan (so the late,
    long tiles fill whole waves of CTAs instead of leaving a near-empty last wave), and among
    those the one that leaves the two ranks closest; more parts: equal shares of the summed
    cost."""
    per_tile = costs.units[:, kv].sum(dim=(0, 1))
    if costs.odd_own is not None:
        per_tile = per_tile + costs.odd_own[:, kv].sum(0)
    if parts == 2:
        best = None
        for cut in range(1, blocks):
            early = makespan(costs, (kv, kv + 1), (0, cut), sms)
            late = makespan(costs, (kv, kv + 1), (cut, blocks), sms)
            key = (max(early, late), abs(early - late))
            if best is None or key < best[0]:
                best = (key, cut)
        return [0, best[1], blocks]
    cum = per_tile.cumsum(0)
    total = float(cum[-1])
    cuts = [0]
    for j in range(1, parts):
        cuts.append(max(cuts[-1] + 1, int(torch.searchsorted(cum, total * j / parts)) + 1))
    cuts.append(blocks)
    if any(b <= a for a, b in zip(cuts, cuts[1:])):
        raise ValueError(f"{blocks} tiles do not split over {parts} ranks")
    return cuts


def partition(rank, world, kv_heads, blocks, costs=None, sms=148):
    """Rank's (kv_range, tile_range): whole KV groups when ``world`` divides Hkv, else
    (``world`` a multiple of Hkv) one KV group split into query-tile ranges at cuts chosen from
    ``costs`` (``cta_costs``; all-causal costs when None). Other world sizes would leave work
    unowned or index past Hkv, so they are refused."""
    if world <= kv_heads:
        if kv_heads % world:
            raise ValueError(f"{kv_heads} KV groups do not split over {world} ranks")
        per = kv_heads // world
        return (rank * per, (rank + 1) * per), (0, blocks)
    if world % kv_heads:
        raise ValueError(f"{world} ranks do not split {kv_heads} KV groups evenly")
    parts = world // kv_heads
    kv = rank // parts
    j = rank % parts
    if costs is None:
        costs = CtaCosts(torch.arange(1, blocks + 1, dtype=torch.float64).expand(1, kv_heads, 1, blocks))
    cuts = tile_cuts(costs, kv, parts, blocks, sms)
    return (kv, kv + 1), (cuts[j], cuts[j + 1])


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


def _max_over_ranks(x, world, dev):
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([float(x)], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t)


def _gather(values, world, dev):
    """[world][len(values)] of every rank's values (all ranks take part)."""
    if world == 1:
        return [list(values)]
    import torch.distributed as dist
    mine = torch.tensor([float(x) for x in values], device=dev)
    out = torch.empty(world * len(values), device=dev)
    dist.all_gather_into_tensor(out, mine)
    return out.view(world, len(values)).tolist()


def _timed(fn, n, world, dev):
    """Mean CUDA-event time of ``fn`` over ``n`` calls on the current stream, max over ranks."""
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(n):
        fn()
    b.record()
    torch.cuda.synchronize()
    return _max_over_ranks(a.elapsed_time(b) / n, world, dev)


def model_measure(args, rank, world, local, dev, steps):
    """Config 3: random-init Qwen2.5-7B, 32640-token prompt (uniform ids + 64 planted 16-token
    key -> value spans), sparse prefill then 128 dense greedy decode tokens; tensor parallel on
    the N GPUs (the caller has set up the process group). Times are max over ranks."""
    from exp3_b200.model import QWEN25_7B, AttentionSettings, Qwen2Model, synthetic_prompt

    model = Qwen2Model(QWEN25_7B, device=dev, seed=0, tp_rank=rank, tp_size=world,
                       attention=AttentionSettings(args.method, args.alpha))
    ids_host = synthetic_prompt(args.prompt_length, QWEN25_7B.vocab_size).pin_memory()
    ids = ids_host.to(dev)
    clocks = ClockSampler(local).open()
    for _ in range(args.warmup):
        model.prefill(ids, args.decode_tokens)
    torch.cuda.synchronize()
    # Tensor parallel: the prefill runs as one pass per layer or as the 4-chunk pipeline that
    # overlaps its all-reduces (Qwen2Model._forward_pipelined); both are timed after the warm-up
    # (max over ranks, so every rank makes the same choice) and the faster one is used and reported.
    by_chunks = {}
    if world > 1:
        for chunks in (1, 4):
            model.prefill_chunks = chunks
            model.prefill(ids, args.decode_tokens)
            by_chunks[chunks] = _timed(lambda: model.prefill(ids, args.decode_tokens), 2, world, dev)
        model.prefill_chunks = min(by_chunks, key=by_chunks.get)
    with clocks:
        prefill_ms = _timed(lambda: model.prefill(ids, args.decode_tokens), steps, world, dev)
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
    decode_eager_ms = _timed(decode_eager, 1, world, dev) / max(1, args.decode_tokens - 1)
    decode_ms = _timed(decode_graph, 1, world, dev) / max(1, args.decode_tokens - 1)
    replay_ms = model.replay_ms_per_token()
    replay_ms = _max_over_ranks(replay_ms, world, dev) if replay_ms is not None else None
    # End to end (evaluate.prefill): token ids from pinned host memory, prefill, first token to host.
    result = torch.empty(1, dtype=torch.int64).pin_memory()

    def e2e():
        ids.copy_(ids_host, non_blocking=True)
        result.copy_(model.prefill(ids, args.decode_tokens).view(1), non_blocking=True)

    e2e_ms = _timed(e2e, steps, world, dev)
    flops = model.prefill_flops(args.prompt_length)  # linear + all causal attention pairs
    model_chunks = model.prefill_chunks
    if world > 1:
        model.close_comm()
    del model
    torch.cuda.empty_cache()
    return {"prefill_ms": prefill_ms, "e2e_ms": e2e_ms, "tp": world, "prefill_chunks": model_chunks,
            "prefill_ms_by_chunks": by_chunks or None,
            "prefill_tflops_dense_equivalent": flops / (prefill_ms * 1e-3) / 1e12,
            "decode_ms_per_token": decode_ms, "decode_ms_per_token_eager": decode_eager_ms,
            "decode_replay_ms_per_token": replay_ms, "steps": steps,
            "h2d_bytes_per_step": ids_host.numel() * 8, "d2h_bytes_per_step": 8,
            "clocks": clocks.summary()}


MODEL_WORKLOAD = ("config 3: random-init Qwen2.5-7B (28 layers, hidden 3584, 28/4 heads, FFN 18944, "
                  "vocab 152064), prompt 32640 ids with 64 planted 16-token spans")


def run_model(args, rank, world, local):
    """``--workload model``: the full-model line alone (value = prefill latency)."""
    import datetime

    import torch.distributed as dist

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)
    m = model_measure(args, rank, world, local, dev, args.steps)
    if rank == 0:
        line = {"metric": "full-model prefill latency, Qwen2.5-7B shape, 32640 tokens", "value": m["prefill_ms"],
                "unit": "ms", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": m["prefill_ms"], "higher_is_better": False, "scaling": "strong", "vs_baseline": None,
                "dtype": "bf16", "data": "synthetic (random-init weights, seeded prompt)",
                "config": {"workload": MODEL_WORKLOAD, "method": args.method, "alpha": args.alpha,
                           "parallelism": f"tp{world} (heads / FFN sharded, NCCL all-reduce after o_proj and down)",
                           **{k: m[k] for k in ("prefill_tflops_dense_equivalent", "decode_ms_per_token",
                                                "decode_ms_per_token_eager", "decode_replay_ms_per_token")},
                           "decode": "CUDA-graph steps (Model.decode_graph); decode_ms_per_token includes the "
                                     "eager warm-up step and the capture, decode_replay_ms_per_token is the "
                                     "steady-state replay",
                           "decode_comm": "one-shot peer-memory all-reduce (exp3_b200.comm)" if world > 1 else None,
                           "decode_tokens": args.decode_tokens},
                "e2e": {"value": m["e2e_ms"], "unit": "ms", "h2d_bytes_per_step": m["h2d_bytes_per_step"],
                        "d2h_bytes_per_step": m["d2h_bytes_per_step"]},
                "clocks": m["clocks"]}
        emit(line)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_reference_gpu(args):
    """Child process of the N=1 bench: the reference's own prefill attention (exp3
    ``AttentionBackend.forward``, attention.py:154-339: its Triton kernels, torch.compile'd
    selection and torch tail) on the same layer and GPU, timed as a black box with CUDA events,
    and torch's dense causal SDPA beside it. Prints one JSON line."""
    ref_root = ROOT / "baseline" / "_ref"
    sys.path.insert(0, str(ref_root))
    try:
        from exp3 import attention as ref_attention
    except Exception as exc:  # noqa: BLE001 - any import failure means "not installed here"
        emit({"unavailable": f"the reference is not importable from baseline/_ref ({type(exc).__name__}: {exc})"})
        return
    import torch.nn.functional as F
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = LAYER_CONFIGS[args.config]
    d = cfg.get("head_dim", 128)
    scale = d ** -0.5
    q, k, v = inputs(args.variant, dev, args.config)
    qh, kh, vh = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)  # HF's [B, H, L, d] views

    class Layer:
        layer_idx = 0

    backend = ref_attention.AttentionBackend(alpha=args.alpha)
    backend.configure(args.method, args.alpha)
    t0 = time.perf_counter()
    for _ in range(args.warmup):  # the first call autotunes the Triton kernels and compiles
        backend.forward(Layer(), qh, kh, vh, None, scale)
    torch.cuda.synchronize()
    warm_s = time.perf_counter() - t0
    ms = _timed(lambda: backend.forward(Layer(), qh, kh, vh, None, scale), args.steps, 1, dev)
    backend.start_profile()
    backend.forward(Layer(), qh, kh, vh, None, scale)
    row = backend.finish_profile()[0]
    pairs = int(row.get("exact_token_pairs") or 0)
    stages = {name: row[f"{name}_ms"] for name in ("descriptor", "selector", "indices", "exact", "mean", "merge")}
    sdpa = lambda: F.scaled_dot_product_attention(qh, kh, vh, is_causal=True, scale=scale, enable_gqa=True)
    for _ in range(args.warmup):
        sdpa()
    sdpa_ms = _timed(sdpa, args.steps, 1, dev)
    b, length, heads = q.shape[0], q.shape[1], q.shape[2]
    causal = b * heads * length * (length + 1) // 2
    try:
        import triton
        triton_version = triton.__version__
    except Exception:  # noqa: BLE001
        triton_version = None
    emit({"ms_per_layer": ms, "effective_tflops": 4 * d * pairs / (ms * 1e-3) / 1e12 if pairs else None,
          "exact_token_pairs": pairs, "density": pairs / causal if pairs else None,
          "stage_ms": stages, "exact_tflops": 4 * d * pairs / (stages["exact"] * 1e-3) / 1e12
          if pairs and stages["exact"] else None,
          "tiles": {"q_tile": row.get("q_tile_size"), "k_tile": row.get("k_tile_size"),
                    "score_k_tile": row.get("score_k_tile_size")},
          "warmup_s": warm_s, "steps": args.steps, "triton": triton_version,
          "path": "exp3 AttentionBackend.forward from baseline/_ref (unmodified reference): Triton "
                  "compute_mean_vector / compute_block_score / _flash_forward (autotuned on this GPU), "
                  "torch.compile'd selection, torch fp32 mean tail and merge",
          "sdpa_dense": {"ms": sdpa_ms, "tflops_all_causal_pairs": 4 * d * causal / (sdpa_ms * 1e-3) / 1e12,
                         "call": "torch.nn.functional.scaled_dot_product_attention(is_causal=True, "
                                 "enable_gqa=True), bf16"}})


def reference_gpu_record(args, timeout_s=600):
    """Runs ``run_reference_gpu`` in a child process (its autotuning, torch.compile and the
    global attention registration stay out of this process) and returns its record."""
    cmd = [sys.executable, str(ROOT / "bench.py"), "--time-reference-gpu", "--config", args.config,
           "--method", args.method, "--alpha", str(args.alpha), "--variant", args.variant,
           "--steps", str(args.steps), "--warmup", str(args.warmup)]
    env = dict(os.environ, CUDA_VISIBLE_DEVICES=os.environ.get("CUDA_VISIBLE_DEVICES", "0").split(",")[0])
    for key in ("RANK", "WORLD_SIZE", "LOCAL_RANK", "MASTER_ADDR", "MASTER_PORT"):
        env.pop(key, None)
    try:
        res = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=timeout_s)
    except subprocess.TimeoutExpired:
        return {"unavailable": f"timed out after {timeout_s} s"}
    lines = [line for line in res.stdout.splitlines() if line.strip().startswith("{")]
    if res.returncode != 0 or not lines:
        tail = " | ".join(res.stderr.strip().splitlines()[-3:])[-400:]
        return {"unavailable": f"exit {res.returncode}: {tail}"}
    return json.loads(lines[-1])


def layer_measure(args, variant, dev, rank, world, local, with_e2e):
    """One layer workload on this rank's shard: routing of the full layer (untimed) for the
    work accounting and the partition, then ``args.steps`` timed steps (route -> exact -> mean +
    merge, CUDA events per stage), and the end-to-end leg through the public API."""
    import torch.distributed as dist
    from exp3_b200 import ops
    from exp3_b200._capi import STAGE_EXACT, STAGE_MEAN, STAGE_ROUTE
    from exp3_b200.attention import AttentionBackend

    cfg = LAYER_CONFIGS[args.config]
    b, length, heads, kv_heads, d = cfg["batch"], cfg["length"], cfg["heads"], cfg["kv_heads"], cfg.get("head_dim", 128)
    scale = d ** -0.5
    group = heads // kv_heads
    blocks = length // 128
    q, k, v = inputs(variant, dev, args.config)
    method, alpha = args.method, args.alpha
    nbytes = ops.workspace_bytes(method, b, length, heads, kv_heads, d)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    out = torch.empty(b, length, heads, d, dtype=torch.bfloat16, device=dev)

    # Routing of the full layer (untimed): the selected work and the shard cuts.
    ops.prefill_attention(q, k, v, method, alpha, scale, out=out, ws=ws, stages=STAGE_ROUTE)
    selected, _, _ = ops.export_routing(method, b, length, heads, kv_heads, head_dim=d, ws=ws, device=dev)
    paired = d == 128 and args.exact_kernel == "tcgen05"
    costs = cta_costs(selected, group, paired=paired)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    kv_range, tile_range = partition(rank, world, kv_heads, blocks, costs=costs, sms=sms)
    pairs = exact_pairs(selected, length, kv_range, tile_range, group)
    all_pairs = exact_pairs(selected, length, (0, kv_heads), (0, blocks), group)
    density = float(selected.sum()) / (b * heads * blocks * (blocks + 1) / 2)
    flops = 4 * d * pairs
    total_flops = 4 * d * all_pairs
    del selected
    if world > 1:  # every unit of the layer is owned by exactly one rank
        summed = torch.tensor([pairs], dtype=torch.int64, device=dev)
        dist.all_reduce(summed)
        if int(summed) != all_pairs:
            raise RuntimeError(f"shards cover {int(summed)} exact pairs of the layer's {all_pairs}")

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
    ms_rank = start.elapsed_time(end) / args.steps
    route_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in ev)
    exact_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in ev)
    mean_ms = statistics.mean(e[2].elapsed_time(e[3]) for e in ev)
    per_rank = _gather([ms_rank, route_ms, exact_ms, mean_ms, flops], world, dev)
    ms_step = max(r[0] for r in per_rank)
    stages = {name: {"max": max(r[i] for r in per_rank), "min": min(r[i] for r in per_rank)}
              for i, name in ((1, "route"), (2, "exact"), (3, "mean_merge"))}
    slowest = max(range(world), key=lambda i: per_rank[i][0])
    # the exact kernel's rate on the slowest rank's own selected pairs
    exact_rate_slowest = per_rank[slowest][4] / (per_rank[slowest][2] * 1e-3) / 1e12
    result = {"ms_step": ms_step, "route_ms": route_ms, "exact_ms": exact_ms, "mean_ms": mean_ms,
              "flops": flops, "total_flops": total_flops, "all_pairs": all_pairs, "density": density,
              "kv_range": kv_range, "tile_range": tile_range, "stages": stages, "slowest_rank": slowest,
              "per_rank_ms": [r[0] for r in per_rank], "exact_tflops_slowest_rank": exact_rate_slowest,
              "clocks": clocks.summary(), "q": q, "k": k, "v": v}
    if not with_e2e:
        return result

    # End to end through the public API (AttentionBackend.forward, the attention.py call site)
    # with pinned host buffers: every step copies this rank's inputs in (H2D), runs the layer
    # and reads its output rows back (D2H), all inside the timed region. A whole-group shard
    # copies its groups' Q, K and V; a tile shard copies only its query rows of Q and the K/V
    # rows up to its last tile (the rows its work reads). The steps are pipelined as a serving
    # loop runs them: per unit, the H2D of the next unit overlaps this unit's compute and the
    # D2H of the previous one, so only one unit's copies are left outside the overlap.
    t0, t1 = tile_range
    full_tiles = tile_range == (0, blocks)
    r0, r1 = t0 * 128, min(length, t1 * 128)
    units = [(g, g + 1) for g in range(kv_range[0], kv_range[1])] if full_tiles else [tuple(kv_range)]
    host = [tuple(x.contiguous().cpu().pin_memory() for x in
                  (q[:, r0:r1, a * group:c * group], k[:, :r1, a:c], v[:, :r1, a:c])) for a, c in units]
    slots = 2
    o_hs = [[torch.empty(b, r1 - r0, (c - a) * group, d, dtype=torch.bfloat16).pin_memory() for a, c in units]
            for _ in range(slots)]
    dev_in = [[(torch.empty(b, length, (c - a) * group, d, dtype=torch.bfloat16, device=dev),
                torch.empty(b, length, c - a, d, dtype=torch.bfloat16, device=dev),
                torch.empty(b, length, c - a, d, dtype=torch.bfloat16, device=dev)) for a, c in units]
              for _ in range(slots)]
    for sl in dev_in:  # rows outside the shard are never read; keep them finite all the same
        for unit in sl:
            for x in unit:
                x.zero_()
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
                    qd[:, r0:r1].copy_(host[u][0], non_blocking=True)
                    kd[:, :r1].copy_(host[u][1], non_blocking=True)
                    vd[:, :r1].copy_(host[u][2], non_blocking=True)
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
                    o_hs[sl][u].copy_(o[:, r0:r1], non_blocking=True)
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
    e2e_ms = _max_over_ranks(s2.elapsed_time(e2) / args.steps, world, dev)
    h2d = sum(x.numel() * x.element_size() for unit in host for x in unit)
    d2h = sum(o.numel() * o.element_size() for o in o_hs[0])
    if world > 1:
        counts = torch.tensor([float(h2d), float(d2h)], device=dev)
        dist.all_reduce(counts)
        h2d, d2h = int(counts[0]), int(counts[1])
    result.update(e2e_ms=e2e_ms, h2d=h2d, d2h=d2h, units=len(units))
    return result


def main():
    args = parse()
    quiet_stdout()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", args.gpus))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if args.warmup < 3:
        raise SystemExit("at least 3 warm-up steps")
    if args.time_reference_gpu:
        return run_reference_gpu(args)
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if args.workload == "model":
        return run_model(args, rank, world, local)

    import torch.distributed as dist

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)
    from exp3_b200 import _capi
    _capi.set_exact_kernel(args.exact_kernel)
    cfg = LAYER_CONFIGS[args.config]
    d = cfg.get("head_dim", 128)
    headline = args.config == "c2"

    lay = layer_measure(args, args.variant, dev, rank, world, local, with_e2e=True)
    q, k, v = lay.pop("q"), lay.pop("k"), lay.pop("v")
    peak, peak_sus, hbm, peak_kind = peaks()
    achieved = lay["flops"] / (lay["exact_ms"] * 1e-3) / 1e12
    traffic = None
    traffic_file = ROOT / "profiles" / "exact_attention_traffic.json"
    if traffic_file.exists():
        try:
            traffic = json.loads(traffic_file.read_text()).get(f"bytes_per_launch_{args.config}")
        except ValueError:
            traffic = None
    launches_per_step = {"dense": 2, "fp_v1": 3}.get(args.method, 4)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.config in ("c2", "q35"):
        cpu = cpu_baseline(args.method, args.alpha, q.cpu(), k.cpu(), v.cpu(), config=args.config)
    del q, k, v
    torch.cuda.empty_cache()

    structured = None
    if headline and args.variant == "iid" and not args.no_structured:
        st = layer_measure(args, "structured", dev, rank, world, local, with_e2e=False)
        for key in ("q", "k", "v"):
            st.pop(key)
        torch.cuda.empty_cache()
        structured = {
            "variant": "structured (block offsets sigma 0.5; synthetic.attention_inputs)",
            "density": st["density"], "ms_per_layer": st["ms_step"],
            "effective_tflops": st["total_flops"] / (st["ms_step"] * 1e-3) / 1e12,
            "exact_token_pairs": st["all_pairs"], "stage_ms": st["stages"],
            "exact": {"achieved_tflops": st["flops"] / (st["exact_ms"] * 1e-3) / 1e12,
                      "frac": st["flops"] / (st["exact_ms"] * 1e-3) / 1e12 / peak,
                      "on": "the selected pairs of rank 0's shard"},
            "tail_merge_ms": st["stages"]["mean_merge"]["max"], "route_ms": st["stages"]["route"]["max"],
            "clocks": st["clocks"]}

    model = None
    if headline and not args.no_model and args.method == "mean_native":
        try:
            model = model_measure(args, rank, world, local, dev, steps=min(args.steps, 5))
        except ValueError as exc:  # a world size the tensor-parallel split refuses
            model = {"unavailable": str(exc)}

    reference_gpu = None
    if rank == 0 and world == 1 and headline and not args.no_reference_gpu:
        reference_gpu = reference_gpu_record(args)

    if rank == 0:
        ms_step = lay["ms_step"]
        line = {
            "metric": cfg["metric"], "value": lay["total_flops"] / (ms_step * 1e-3) / 1e12, "unit": "TFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": cfg["workload"], "method": args.method, "alpha": args.alpha,
                       "variant": args.variant,
                       "exact_kernel": "tcgen05_single" if d == 256 else args.exact_kernel, "ms_per_layer": ms_step,
                       "density": lay["density"], "exact_token_pairs": lay["all_pairs"],
                       "l2": f"no flush: Q ({cfg['batch'] * cfg['length'] * cfg['heads'] * d * 2 / 1e6:.0f} MB) "
                             "and O are larger than the 126 MB L2",
                       "parallelism": f"{world} rank(s): (KV group x query-tile range) shards, no collective; "
                                      "tile cuts by simulated CTA waves of the selected work",
                       "rank0_shard": {"kv_range": list(lay["kv_range"]), "tile_range": list(lay["tile_range"])},
                       "stage_ms_over_ranks": lay["stages"], "per_rank_ms": lay["per_rank_ms"],
                       "slowest_rank": lay["slowest_rank"],
                       "stage_ms_rank0": {"route": lay["route_ms"], "exact": lay["exact_ms"],
                                          "mean_merge": lay["mean_ms"]}},
            "roofline": {"bound": "tensor", "kernel": "exact attention (sparse FA)" + (", d=256" if d == 256 else ""),
                         "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                         "peak_kind": f"{peak_kind} burst bf16",
                         "frac_of_sustained": achieved / peak_sus if peak_sus else None, "traffic": traffic,
                         "on": "rank 0's selected pairs over rank 0's exact-kernel CUDA-event time",
                         "slowest_rank_achieved": lay["exact_tflops_slowest_rank"]},
            "cpu_baseline": cpu,
            "e2e": {"value": lay["total_flops"] / (lay["e2e_ms"] * 1e-3) / 1e12, "unit": "TFLOP/s",
                    "ms_per_step": lay["e2e_ms"], "h2d_bytes_per_step": lay["h2d"], "d2h_bytes_per_step": lay["d2h"],
                    "pipeline": f"{lay['units']} unit(s) per step (KV groups, or the rank's tile shard), 2 input "
                                "slots per unit; H2D / compute / D2H of successive units overlap on 3 streams; "
                                "a tile shard copies only the rows it reads"},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": lay["clocks"],
        }
        if structured is not None:
            line["structured"] = structured
        if model is not None:
            line["model"] = {"workload": MODEL_WORKLOAD, "method": args.method, "alpha": args.alpha,
                             "parallelism": f"tp{world}", **model}
        if reference_gpu is not None:
            line["reference_gpu"] = reference_gpu
        emit(line)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
