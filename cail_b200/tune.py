"""Measures the auto-dispatch crossovers of this box and writes a CAIL_TUNE_FILE.

    python -m cail_b200.tune --ranks 2,4,8 --out cail.tune [--nvls] [--ce]

For every rank count it runs ``cail_bench`` under ``cail-mpirun`` with each
algorithm forced (one_shot and two_shot over 32 KiB .. 8 MiB; with --nvls or
--ce also nvls / ce_two_shot against two_shot over 1 MiB .. 1 GiB) and keeps,
per size, the p50 latency (max over ranks).  The file then holds, per rank
count, the largest size up to which one_shot never loses
(``oneshot_max``) and the smallest size from which nvls or ce_two_shot never
loses any more (``nvls_min``, ``ce_min``; omitted when they never win).  The
library reads it with ``CAIL_TUNE_FILE=cail.tune``; environment variables of
the same meaning still take precedence.
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys
import time
from typing import Dict, List, Optional

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "build", "bin")
LIB = os.path.join(ROOT, "build", "lib")

Sweep = Dict[int, float]  # bytes -> p50 microseconds


def parse_bench(text: str) -> Sweep:
    """p50 per size from cail_bench's CSV (bytes,algo,p50_us,p99_us,mean_us,busbw)."""
    out: Sweep = {}
    for line in text.splitlines():
        f = line.strip().split(",")
        if len(f) >= 3 and f[0].isdigit():
            out[int(f[0])] = float(f[2])
    return out


def last_win(small: Sweep, big: Sweep) -> Optional[int]:
    """Largest size s such that `small` is no slower than `big` at s and at
    every smaller size measured for both; None if it loses at the smallest."""
    best = None
    for b in sorted(set(small) & set(big)):
        if small[b] <= big[b]:
            best = b
        else:
            break
    return best


def first_lasting_win(new: Sweep, old: Sweep) -> Optional[int]:
    """Smallest size s from which `new` is no slower than `old` at s and at
    every larger size measured for both; None if it loses at the largest."""
    best = None
    for b in sorted(set(new) & set(old), reverse=True):
        if new[b] <= old[b]:
            best = b
        else:
            break
    return best


def tune_line(nranks: int, one: Sweep, two: Sweep, nvls: Optional[Sweep] = None,
              two_big: Optional[Sweep] = None, ce: Optional[Sweep] = None) -> str:
    parts = [f"nranks={nranks}"]
    om = last_win(one, two)
    if om is not None:
        parts.append(f"oneshot_max={om}")
    if nvls is not None and two_big is not None:
        nm = first_lasting_win(nvls, two_big)
        if nm is not None:
            parts.append(f"nvls_min={nm}")
    if ce is not None and two_big is not None:
        cm = first_lasting_win(ce, two_big)
        if cm is not None:
            parts.append(f"ce_min={cm}")
    return " ".join(parts)


def measure(nranks: int, algo: str, lo: int, hi: int, iters: int, timeout: int) -> Sweep:
    env = {k: v for k, v in os.environ.items() if not k.startswith("CAIL_")}
    env.update({"CAIL_ALGO": algo, "CAIL_MIN_MSG_SIZE": "0"})
    cmd = [os.path.join(BIN, "cail-mpirun"), "-np", str(nranks), "--timeout", str(timeout), "-x",
           "LD_PRELOAD=" + os.path.join(LIB, "libcail.so"), os.path.join(BIN, "cail_bench"), "-b", str(lo),
           "-e", str(hi), "-i", str(iters), "-w", "10"]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=timeout + 30)
    if r.returncode != 0:
        raise RuntimeError(f"cail_bench np={nranks} {algo} failed:\n{r.stdout[-2000:]}{r.stderr[-2000:]}")
    return parse_bench(r.stdout)


def main(argv: Optional[List[str]] = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--ranks", default="2,4,8", help="comma-separated rank counts (one GPU per rank)")
    ap.add_argument("--out", default="cail.tune")
    ap.add_argument("--nvls", action="store_true", help="also place the nvls crossover")
    ap.add_argument("--ce", action="store_true", help="also place the ce_two_shot crossover")
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--timeout", type=int, default=300, help="seconds per cail_bench run")
    a = ap.parse_args(argv)
    lines = [f"# CAIL_TUNE_FILE written by cail_b200.tune on {time.strftime('%Y-%m-%d %H:%M:%S')}"]
    for n in [int(x) for x in a.ranks.split(",") if x]:
        one = measure(n, "one_shot", 32 << 10, 8 << 20, a.iters, a.timeout)
        two = measure(n, "two_shot", 32 << 10, 8 << 20, a.iters, a.timeout)
        nvls = two_big = ce = None
        if a.nvls or a.ce:
            two_big = measure(n, "two_shot", 1 << 20, 1 << 30, a.iters, a.timeout)
        if a.nvls:
            nvls = measure(n, "nvls", 1 << 20, 1 << 30, a.iters, a.timeout)
        if a.ce:
            ce = measure(n, "ce_two_shot", 1 << 20, 1 << 30, a.iters, a.timeout)
        line = tune_line(n, one, two, nvls, two_big, ce)
        print(line, flush=True)
        lines.append(line)
    with open(a.out, "w") as f:
        f.write("\n".join(lines) + "\n")
    print(f"wrote {a.out}", file=sys.stderr)
    return 0


if __name__ == "__main__":
    sys.exit(main())
