"""One-GPU kernel benchmark (the test-only libcail_kbench.so harness).

Times one of cail's kernels on the current GPU with every peer of a P-rank
communicator emulated by a buffer of the same GPU, so the kernel can be
timed and profiled without NVLink:

    python -m cail_b200.kbench KERNEL [--ranks P] [--bytes N] [--iters K]

KERNEL: one_shot, two_shot_zerocopy, fold, bulk_copy, push (the push
two-shot of P emulated ranks in one cooperative launch), copy, reduce_local.
Prints one line: kernel, ranks, bytes, mean ms per launch, and the bytes the
kernel moves through DRAM per launch divided by that time (the copy and
reduce kernels' algorithmic traffic; for the emulated collectives, the
local-memory traffic that replaces NVLink).
"""
from __future__ import annotations

import argparse
import ctypes
import sys

from . import _lib

KERNELS = {"one_shot": 0, "two_shot_zerocopy": 1, "fold": 2, "bulk_copy": 3, "push": 4, "copy": 5,
           "reduce_local": 6}


def dram_bytes(kernel: str, P: int, nbytes: int) -> int:
    """Algorithmic DRAM bytes per launch (reads + writes)."""
    if kernel in ("copy", "bulk_copy"):
        return 2 * nbytes
    if kernel == "reduce_local":
        return 3 * nbytes                       # read in, read io, write io
    if kernel == "fold":
        return (P + 1) * nbytes                 # P sources, one output
    if kernel == "one_shot":
        return nbytes + P * nbytes + P * nbytes + nbytes   # read src, push P slots, fold P, write dst
    if kernel == "two_shot_zerocopy":
        return 2 * nbytes                       # its slice of P inputs read, of P outputs written (x P / P)
    if kernel == "push":
        # all P ranks: push (P-1)/P N, fold reads N and writes N/P + (P-1)/P N,
        # copy-out reads and writes (P-1)/P N -- per rank; times P ranks
        per = nbytes * ((P - 1) / P * 2 + 1 + 1 / P + (P - 1) / P + 2 * (P - 1) / P)
        return int(per * P)
    raise ValueError(kernel)


def run(kernel: str, P: int, nbytes: int, iters: int) -> float:
    ctypes.CDLL(_lib.lib_path("libmpi.so"), mode=ctypes.RTLD_GLOBAL)
    ctypes.CDLL(_lib.lib_path("libcail.so"), mode=ctypes.RTLD_GLOBAL)
    k = ctypes.CDLL(_lib.lib_path("libcail_kbench.so"))
    k.cail_bench_kernel_local.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_size_t, ctypes.c_int,
                                          ctypes.POINTER(ctypes.c_float)]
    ms = ctypes.c_float(0)
    rc = k.cail_bench_kernel_local(KERNELS[kernel], P, nbytes, iters, ctypes.byref(ms))
    if rc != 0:
        raise RuntimeError(f"cail_bench_kernel_local({kernel}) returned {rc}")
    return ms.value


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("kernel", choices=sorted(KERNELS))
    ap.add_argument("--ranks", type=int, default=8)
    ap.add_argument("--bytes", type=int, default=64 << 20)
    ap.add_argument("--iters", type=int, default=20)
    a = ap.parse_args()
    ms = run(a.kernel, a.ranks, a.bytes, a.iters)
    gbs = dram_bytes(a.kernel, a.ranks, a.bytes) / (ms * 1e-3) / 1e9
    print(f"{a.kernel} ranks={a.ranks} bytes={a.bytes} ms={ms:.4f} dram_GBps={gbs:.1f}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
