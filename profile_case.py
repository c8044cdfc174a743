"""Runs the fused prefill attention layer a few times on one shape: the command profiled by ncu.

    python profile_case.py [--length 32768] [--head-dim 128|256] [--method mean_native] [--alpha 0.08]
                           [--repeats 3] [--variant iid|structured] [--kernel tcgen05|tcgen05_single|mma]

Exits 0 after printing per-stage CUDA-event times of the last repeat; it is meant to be run
once plainly and then under ``ncu -k regex:<kernel> -s <skip> -c <count>``.
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parent))

from exp3_b200 import _capi, ops, synthetic  # noqa: E402
from exp3_b200._capi import STAGE_EXACT, STAGE_MEAN, STAGE_ROUTE  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--length", type=int, default=32768)
    ap.add_argument("--heads", type=int, default=28)
    ap.add_argument("--kv-heads", type=int, default=4)
    ap.add_argument("--head-dim", type=int, default=128, choices=[128, 256])
    ap.add_argument("--method", default="mean_native")
    ap.add_argument("--alpha", type=float, default=0.08)
    ap.add_argument("--repeats", type=int, default=3)
    ap.add_argument("--variant", default="iid", choices=["iid", "structured"])
    ap.add_argument("--kernel", default="tcgen05", choices=["tcgen05", "tcgen05_single", "mma"])
    ap.add_argument("--emulate", type=int, default=0, choices=[0, 2, 3])
    args = ap.parse_args()
    dev = torch.device("cuda", 0)
    shape = synthetic.LayerShape(1, args.length, args.heads, args.kv_heads, args.head_dim)
    q, k, v = synthetic.attention_inputs(shape, seed=0, needles=32, device=dev,
                                         structured_sigma=0.5 if args.variant == "structured" else 0.0)
    _capi.set_exact_kernel(args.kernel)
    _capi.set_exp_emulation(args.emulate)
    out = torch.empty_like(q)
    scale = args.head_dim ** -0.5
    times = {}
    for _ in range(args.repeats):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        ev[0].record()
        ops.prefill_attention(q, k, v, args.method, args.alpha, scale, out=out, stages=STAGE_ROUTE)
        ev[1].record()
        ops.prefill_attention(q, k, v, args.method, args.alpha, scale, out=out, stages=STAGE_EXACT)
        ev[2].record()
        ops.prefill_attention(q, k, v, args.method, args.alpha, scale, out=out, stages=STAGE_MEAN)
        ev[3].record()
        torch.cuda.synchronize()
        times = {"route_ms": ev[0].elapsed_time(ev[1]), "exact_ms": ev[1].elapsed_time(ev[2]),
                 "mean_ms": ev[2].elapsed_time(ev[3])}
    if _capi.device_error() != 0:
        raise SystemExit("a kernel reported a timed-out wait")
    print(times)


if __name__ == "__main__":
    main()
