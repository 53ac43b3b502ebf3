"""One-GPU kernel benchmark (the test-only libcail_kbench.so harness).

Times one of cail's kernels on the current GPU with every peer of a P-rank
communicator emulated by a buffer of the same GPU, so the kernel can be
timed and profiled without NVLink:

    python -m cail_b200.kbench KERNEL [--ranks P] [--bytes N] [--iters K]
    python -m cail_b200.kbench reduce_local --impl reference [--bytes N] [--iters K]
    python -m cail_b200.kbench noalloc [--ranks S] [--bytes N] [--iters K]

KERNEL: one_shot, two_shot_zerocopy, fold, bulk_copy, push (the push
two-shot of P emulated ranks in one cooperative launch), copy, reduce_local.
noalloc times cail_reduce_sources_noalloc() folding S sources of N bytes
(at most 8 x 256 KiB, its fixed scratch) on the current stream.

--impl reference (reduce_local only) times the reference library's own
cail_gpu_reduce_local() (its float4 SUM kernel plus its stream synchronise,
built from the unmodified sources into baseline/_ref) against the same
entry point of libcail (--impl ours): inout += in over float buffers of
--bytes bytes, CUDA events around --iters calls.

Prints one line: kernel, ranks, bytes, mean ms per launch, and the bytes the
kernel moves through DRAM per launch divided by that time (the copy and
reduce kernels' algorithmic traffic; for the emulated collectives, the
local-memory traffic that replaces NVLink).
"""
from __future__ import annotations

import argparse
import ctypes
import os
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
        # all P emulated ranks: each reads its input once, stores it into
        # P - 1 peers' slots, folds P copies and writes its output
        return P * (2 * P + 1) * nbytes
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


def run_entry(impl: str, nbytes: int, iters: int) -> float:
    """Mean ms per cail_gpu_reduce_local(in, io, n, CAIL_FLOAT, CAIL_SUM)
    call of the chosen library (each call returns after its kernel)."""
    import torch

    ctypes.CDLL(_lib.lib_path("libmpi.so"), mode=ctypes.RTLD_GLOBAL)
    path = _lib.lib_path("libcail.so") if impl == "ours" else os.path.join(_lib.REF_LIB_DIR, "libcail.so")
    lib = ctypes.CDLL(path)
    lib.cail_gpu_reduce_local.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int,
                                          ctypes.c_int]
    if impl == "reference":
        lib.cail_gpu_init()
    n = nbytes // 4
    x = torch.rand(n, device="cuda")
    io = torch.rand(n, device="cuda")
    torch.cuda.synchronize()
    for _ in range(3):
        assert lib.cail_gpu_reduce_local(x.data_ptr(), io.data_ptr(), n, 3, 0) == 0
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        lib.cail_gpu_reduce_local(x.data_ptr(), io.data_ptr(), n, 3, 0)
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters


def run_noalloc(nsrc: int, nbytes: int, iters: int) -> float:
    import torch

    ctypes.CDLL(_lib.lib_path("libmpi.so"), mode=ctypes.RTLD_GLOBAL)
    lib = ctypes.CDLL(_lib.lib_path("libcail.so"))
    vp = ctypes.c_void_p
    lib.cail_reduce_sources_noalloc.argtypes = [ctypes.POINTER(vp), ctypes.c_int, vp, ctypes.c_size_t, ctypes.c_int,
                                                ctypes.c_int, vp]
    n = nbytes // 4
    srcs = [torch.rand(n, device="cuda") for _ in range(nsrc)]
    out = torch.empty(n, device="cuda")
    arr = (vp * nsrc)(*[t.data_ptr() for t in srcs])
    stream = torch.cuda.current_stream().cuda_stream
    H = _lib.H
    for _ in range(3):
        assert lib.cail_reduce_sources_noalloc(arr, nsrc, out.data_ptr(), n, H["MPI_FLOAT"], H["MPI_SUM"], stream) == 0
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        lib.cail_reduce_sources_noalloc(arr, nsrc, out.data_ptr(), n, H["MPI_FLOAT"], H["MPI_SUM"], stream)
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("kernel", choices=sorted(KERNELS) + ["noalloc"])
    ap.add_argument("--ranks", type=int, default=8)
    ap.add_argument("--bytes", type=int, default=64 << 20)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--impl", choices=["harness", "ours", "reference"], default="harness",
                    help="reduce_local only: time a library's cail_gpu_reduce_local entry point")
    a = ap.parse_args()
    if a.impl != "harness":
        if a.kernel != "reduce_local":
            ap.error("--impl ours|reference applies to reduce_local")
        ms = run_entry(a.impl, a.bytes, a.iters)
        gbs = dram_bytes("reduce_local", 1, a.bytes) / (ms * 1e-3) / 1e9
        print(f"reduce_local impl={a.impl} bytes={a.bytes} ms={ms:.4f} dram_GBps={gbs:.1f}")
        return 0
    if a.kernel == "noalloc":
        ms = run_noalloc(a.ranks, a.bytes, a.iters)
        # read every source twice (push, fold), write scratch once and the output once
        gbs = (2 * a.ranks * a.bytes + a.ranks * a.bytes + a.bytes) / (ms * 1e-3) / 1e9
        print(f"noalloc sources={a.ranks} bytes={a.bytes} ms={ms:.4f} moved_GBps={gbs:.1f}")
        return 0
    ms = run(a.kernel, a.ranks, a.bytes, a.iters)
    gbs = dram_bytes(a.kernel, a.ranks, a.bytes) / (ms * 1e-3) / 1e9
    print(f"{a.kernel} ranks={a.ranks} bytes={a.bytes} ms={ms:.4f} dram_GBps={gbs:.1f}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
