"""Summarises an ncu CSV launch list (``--metrics gpu__time_duration.sum --csv``) per kernel.

    python ncu_summary.py launches.csv [--top 12]

Prints launches, total device time and share per kernel name. ncu serialises launches
and runs them cold, so compare shares, not absolute times, with a bench run.
"""

from __future__ import annotations

import argparse
import collections
import csv

UNIT_US = {"nsecond": 1e-3, "ns": 1e-3, "usecond": 1.0, "us": 1.0, "msecond": 1e3, "ms": 1e3}


def summarise(path: str, metric: str = "gpu__time_duration.sum"):
    rows = [r for r in csv.reader(open(path)) if len(r) > 10]
    header, body = rows[0], rows[1:]
    ki, mi, vi, ui = (header.index(x) for x in ("Kernel Name", "Metric Name", "Metric Value", "Metric Unit"))
    agg = collections.OrderedDict()
    for r in body:
        if r[mi] != metric:
            continue
        name = r[ki].split("(")[0].strip()
        entry = agg.setdefault(name, [0, 0.0])
        entry[0] += 1
        entry[1] += float(r[vi].replace(",", "")) * UNIT_US.get(r[ui], 1.0)
    total = sum(v[1] for v in agg.values()) or 1.0
    return sorted(((n, c, t, t / total) for n, (c, t) in agg.items()), key=lambda x: -x[2])


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("csv")
    ap.add_argument("--top", type=int, default=12)
    args = ap.parse_args()
    print(f"{'launches':>8} {'total ms':>10} {'share':>7}  kernel")
    for name, count, us, share in summarise(args.csv)[: args.top]:
        print(f"{count:8d} {us / 1e3:10.3f} {100 * share:6.2f}%  {name[:90]}")


if __name__ == "__main__":
    main()
