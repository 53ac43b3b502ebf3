#!/usr/bin/env python
"""Allreduce benchmark: bus bandwidth and p50 latency of MPI_Allreduce.

Headline (one JSON line on rank 0): MPI_FLOAT SUM of a 1 GiB buffer per
rank, separate send/recv buffers, inputs normal(0,1) seeded per rank; K
timed calls after W warm-up calls, bracketed by a barrier and
torch.cuda.synchronize() on both sides, timed with CUDA events, max over
ranks.  1 GiB inputs exceed the 126 MB L2, so no flush is needed.  The
JSON also carries the size sweep 32 KiB .. 1 GiB (busbw and p50 latency per
size, max over ranks) and an end-to-end number through the public API that
includes the host->device copy of each step's input from pinned memory and
the device->host copy of its result.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference|nccl|pmpi]
    torchrun --nproc-per-node N bench.py --gpus N ...   (one rank per GPU)

--impl reference runs the unmodified reference library (baseline/_ref,
built by baseline/build_reference.py) through its own public API,
MPI_Allreduce, on the same MPI; --impl nccl runs torch.distributed NCCL
all_reduce; --impl pmpi runs the MPI's own PMPI_Allreduce (no interposer).

busbw = 2 (P-1)/P * bytes / t (nccl-tests convention).  With one GPU that
factor is 0, so the N=1 value is algbw = bytes / t of the single-rank call
(a device copy through cail's kernels).

--workload ddp runs the data-parallel GPT-2-medium step instead (tokens/s and
exposed communication): gradients in 25 MB buckets all-reduced through the
interposer (ours, reference, pmpi), or PyTorch's DistributedDataParallel
over NCCL with the same bucket size (--impl nccl).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import time

METRIC = "allreduce busbw GB/s & p50 latency vs msg size at 2/4/8 B200 (max over ranks)"
GIB = 1 << 30


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def busbw(nbytes: int, t_s: float, p: int) -> float:
    alg = nbytes / t_s / 1e9
    return alg * 2 * (p - 1) / p if p > 1 else alg


def unavailable(reason: str) -> None:
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps({"impl": "reference", "unavailable": reason}), flush=True)
    sys.exit(0)


class Comm:
    """Barrier / max-over-ranks for either MPI (ours, reference, pmpi) or NCCL."""

    def __init__(self, impl: str, rank: int, size: int):
        self.impl = impl
        self.rank = rank
        self.size = size

    def barrier(self):
        if self.impl == "nccl":
            if self.size == 1:  # one rank: no process group is created
                return
            import torch.distributed as dist
            dist.barrier()
        else:
            import cail_b200
            cail_b200.barrier()

    def max(self, v: float) -> float:
        if self.impl == "nccl":
            if self.size == 1:
                return v
            import torch
            import torch.distributed as dist
            t = torch.tensor([v], dtype=torch.float64, device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return float(t.item())
        import cail_b200
        return cail_b200.host_max(v)


def run_ddp(args, rank: int, world: int, local: int, comm: "Comm") -> dict:
    """Data-parallel GPT-2-medium step: fp32, micro-batch 8 x 1024 tokens per
    GPU, gradients in 25 MB buckets all-reduced through the interposer while
    backward runs.  Exposed communication = step time with communication
    minus step time of the same loop with the allreduces switched off."""
    import torch

    from cail_b200.models import GPT2, GPT2Config
    from cail_b200.parallel import BucketedAllreduce

    cfg = GPT2Config.medium()
    mb, seq = args.micro_batch, cfg.n_ctx
    torch.manual_seed(0)
    model = GPT2(cfg).cuda()
    opt = torch.optim.AdamW(model.parameters(), lr=1e-4, fused=True)
    ddp = BucketedAllreduce(model, world, bucket_bytes=25 << 20)
    g = torch.Generator().manual_seed(4242 + rank)
    host_x = torch.randint(0, cfg.vocab, (mb, seq), generator=g).pin_memory()
    host_y = torch.randint(0, cfg.vocab, (mb, seq), generator=g).pin_memory()
    x = torch.empty_like(host_x, device="cuda")
    y = torch.empty_like(host_y, device="cuda")
    on = ddp.enabled

    def step():
        ddp.zero_grad()
        x.copy_(host_x, non_blocking=True)
        y.copy_(host_y, non_blocking=True)
        loss = model(x, y)
        loss.backward()
        ddp.finish()
        opt.step()
        return loss.item()  # device->host read of the step's result

    def timed(enabled: bool) -> float:
        ddp.enabled = enabled and on
        comm.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            step()
        torch.cuda.synchronize()
        return comm.max((time.perf_counter() - t0) / args.steps)

    for _ in range(args.warmup):
        step()
    ddp.check_views(model)
    t_compute = timed(False)
    t_full = timed(True)
    ddp.close()
    tokens = world * mb * seq
    return {
        "metric": "DDP GPT-2-medium training throughput (tokens/s, fp32 grads, 25 MB buckets)",
        "value": round(tokens / t_full, 1),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(t_full * 1e3, 3),
        "compute_only_ms_per_step": round(t_compute * 1e3, 3),
        "exposed_comm_ms": round((t_full - t_compute) * 1e3, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "dtype": "fp32",
        "data": "synthetic token ids uniform over the vocabulary; random-init weights",
        "config": {"model": "GPT-2 medium (24L, d1024, 16H, MLP 4096, vocab 50257)", "global_batch": world * mb,
                   "seq_len": seq, "parallelism": f"dp{world}", "buckets": ddp.num_buckets,
                   "params": model.num_params()},
        "impl": args.impl,
    }


def run_ddp_nccl(args, rank: int, world: int, local: int, comm: "Comm") -> dict:
    """The same GPT-2-medium step under PyTorch's DistributedDataParallel over
    NCCL (25 MB buckets, gradients as bucket views): the NCCL baseline of the
    data-parallel workload.  Compute-only time runs the loop under no_sync()."""
    import contextlib

    import torch
    from torch.nn.parallel import DistributedDataParallel as DDP

    from cail_b200.models import GPT2, GPT2Config

    cfg = GPT2Config.medium()
    mb, seq = args.micro_batch, cfg.n_ctx
    torch.manual_seed(0)
    model = GPT2(cfg).cuda()
    net = DDP(model, device_ids=[local], bucket_cap_mb=25, gradient_as_bucket_view=True) if world > 1 else model
    opt = torch.optim.AdamW(model.parameters(), lr=1e-4, fused=True)
    g = torch.Generator().manual_seed(4242 + rank)
    host_x = torch.randint(0, cfg.vocab, (mb, seq), generator=g).pin_memory()
    host_y = torch.randint(0, cfg.vocab, (mb, seq), generator=g).pin_memory()
    x = torch.empty_like(host_x, device="cuda")
    y = torch.empty_like(host_y, device="cuda")

    def step(sync: bool):
        opt.zero_grad(set_to_none=False)
        x.copy_(host_x, non_blocking=True)
        y.copy_(host_y, non_blocking=True)
        ctx = contextlib.nullcontext() if (sync or world == 1) else net.no_sync()
        with ctx:
            loss = net(x, y)
            loss.backward()
        opt.step()
        return loss.item()  # device->host read of the step's result

    def timed(sync: bool) -> float:
        comm.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            step(sync)
        torch.cuda.synchronize()
        return comm.max((time.perf_counter() - t0) / args.steps)

    for _ in range(args.warmup):
        step(True)
    t_compute = timed(False)
    t_full = timed(True)
    tokens = world * mb * seq
    return {
        "metric": "DDP GPT-2-medium training throughput (tokens/s, fp32 grads, 25 MB buckets)",
        "value": round(tokens / t_full, 1),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(t_full * 1e3, 3),
        "compute_only_ms_per_step": round(t_compute * 1e3, 3),
        "exposed_comm_ms": round((t_full - t_compute) * 1e3, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "dtype": "fp32",
        "data": "synthetic token ids uniform over the vocabulary; random-init weights",
        "config": {"model": "GPT-2 medium (24L, d1024, 16H, MLP 4096, vocab 50257)", "global_batch": world * mb,
                   "seq_len": seq, "parallelism": f"dp{world}", "buckets": "torch DDP, bucket_cap_mb=25",
                   "params": model.num_params()},
        "impl": "nccl",
    }


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--workload", default="allreduce", choices=["allreduce", "ddp"])
    ap.add_argument("--micro-batch", type=int, default=8)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference", "nccl", "pmpi"])
    ap.add_argument("--bytes", type=int, default=GIB, help="headline message size per rank")
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--sweep-min", type=int, default=32 << 10)
    ap.add_argument("--sweep-max", type=int, default=GIB)
    ap.add_argument("--sweep-iters", type=int, default=100)
    ap.add_argument("--sweep-warmup", type=int, default=20)
    ap.add_argument("--no-e2e", action="store_true")
    args = ap.parse_args()

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        log(f"bench: WORLD_SIZE={world} but --gpus {args.gpus}; launch with torchrun --nproc-per-node {args.gpus}")
        sys.exit(2)
    if args.warmup < 3:
        log("bench: at least 3 warm-up steps are required; using 3")
        args.warmup = 3

    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    import torch

    if args.impl == "reference":
        from cail_b200 import _lib
        if not os.path.exists(os.path.join(_lib.REF_LIB_DIR, "libcail.so")):
            unavailable("reference library not built: run python baseline/build_reference.py "
                        "(the reference is a C/autotools library with no Python packaging)")
    torch.cuda.set_device(local)
    torch.cuda.init()
    dev = torch.device("cuda", local)

    if args.impl == "nccl":
        import torch.distributed as dist
        from datetime import timedelta
        if world > 1:
            dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
        comm = Comm("nccl", rank, world)

        # torch.distributed has no out-of-place all_reduce: the timed calls
        # reduce dst in place (NCCL's own cost, no extra copy); the result
        # check and the end-to-end loop below put the input into dst first
        def allreduce(src, dst):
            if world > 1:
                dist.all_reduce(dst)
            else:
                dst.copy_(src)
    else:
        import cail_b200
        from cail_b200 import _lib
        impl = {"ours": "ours", "reference": "reference", "pmpi": "none"}[args.impl]
        cail_b200.init(impl)
        comm = Comm(args.impl, cail_b200.rank(), cail_b200.world_size())
        H = _lib.H
        # MPI_Allreduce of the loaded library (ours, the reference or the
        # MPI's own) called through ctypes, which releases the GIL; both arms
        # take this same call path and load no Python extension of this repo
        mpi_allreduce = _lib.loaded().cail.MPI_Allreduce
        dt, op, cw = H["MPI_FLOAT"], H["MPI_SUM"], H["MPI_COMM_WORLD"]

        def allreduce(src, dst):
            rc = mpi_allreduce(src.data_ptr(), dst.data_ptr(), src.numel(), dt, op, cw)
            if rc != 0:
                raise RuntimeError(f"MPI_Allreduce returned {rc}")

    P = world
    if args.workload == "ddp":
        if args.impl == "nccl":
            out = run_ddp_nccl(args, rank, world, local, comm)
            if rank == 0:
                print(json.dumps(out), flush=True)
            if world > 1:
                import torch.distributed as dist
                dist.destroy_process_group()
            return
        out = run_ddp(args, rank, world, local, comm)
        if rank == 0:
            print(json.dumps(out), flush=True)
        import cail_b200
        cail_b200.finalize()
        return
    count = args.bytes // 4
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)
    send = torch.randn(count, device=dev, generator=gen)
    recv = torch.empty_like(send)
    torch.cuda.synchronize()

    def stats_launches():
        if args.impl != "ours":
            return None
        import cail_b200
        return cail_b200.stats().launches

    # ---------------- headline: K timed steps of the full message
    # nvidia-smi samples every 100 ms from before the warm-up to the end of
    # the sweep, a window that contains the (short) timed region
    from cail_b200.utils import ClockSampler
    clocks = ClockSampler(local, period_ms=100).__enter__()
    time.sleep(0.3)
    for _ in range(args.warmup):
        allreduce(send, recv)
    comm.barrier()
    torch.cuda.synchronize()
    l0 = stats_launches()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.steps):
        allreduce(send, recv)
    end.record()
    torch.cuda.synchronize()
    comm.barrier()
    l1 = stats_launches()
    t_step = comm.max(start.elapsed_time(end) / 1e3 / args.steps)
    value = busbw(args.bytes, t_step, P)
    algo = None
    if args.impl == "ours":
        import cail_b200
        algo = cail_b200.last_algorithm()

    # ---------------- result check: every rank regenerates all P inputs from
    # their seeds and folds them in rank order in fp32 (the oracle); the
    # NVLink kernels fold in the same order, so floats must match bit for bit
    def rank_order_fold() -> "torch.Tensor":
        g = torch.Generator(device=dev)
        acc = None
        for r in range(P):
            g.manual_seed(1234 + r)
            x = torch.randn(count, device=dev, generator=g)
            acc = x if acc is None else acc.add_(x)
            del x
        return acc

    if args.impl == "nccl" and world > 1:
        recv.copy_(send)
        allreduce(recv, recv)
        torch.cuda.synchronize()
    expect = rank_order_fold()
    mismatches = comm.max(float((expect != recv).sum().item()))
    max_err = comm.max(float((expect - recv).abs().max().item()))
    # relative to 1 + |expected|, as the repository's checker does
    rel_err = comm.max(float(((expect - recv).abs() / (1.0 + expect.abs())).max().item()))
    del expect
    if mismatches == 0:
        check = "bit_exact"
    else:
        reassociating = args.impl == "nccl" or algo == "nvls"
        check = {"mismatches": int(mismatches), "max_abs_err": max_err, "max_rel_err": rel_err,
                 "within_tolerance_1e-4": bool(rel_err <= 1e-4),
                 "note": ("NCCL reduces in its own order" if args.impl == "nccl" else
                          "NVLS: the NVSwitch adds the ranks' values in its own order" if reassociating else
                          "differs from the rank-order fold")}

    # ---------------- end to end through the public API, host data
    e2e = None
    if not args.no_e2e:
        if args.impl == "nccl":
            public = allreduce
        else:
            from cail_b200.ops import allreduce as public  # the tensor API over MPI_Allreduce
        h_in = torch.empty(count, dtype=torch.float32, pin_memory=True)
        h_in.copy_(send.cpu())
        h_out = torch.empty(count, dtype=torch.float32, pin_memory=True)
        # (NCCL reduces in place: its input goes straight into recv)
        inp = recv if args.impl == "nccl" and world > 1 else send
        for _ in range(2):
            inp.copy_(h_in, non_blocking=True)
            torch.cuda.synchronize()
            public(inp, recv)
            h_out.copy_(recv, non_blocking=True)
            torch.cuda.synchronize()
        comm.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            inp.copy_(h_in, non_blocking=True)
            torch.cuda.synchronize()
            public(inp, recv)
            h_out.copy_(recv, non_blocking=True)
            torch.cuda.synchronize()
        t_e2e = comm.max((time.perf_counter() - t0) / args.steps)
        e2e = {"value": busbw(args.bytes, t_e2e, P), "unit": "GB/s", "ms_per_step": t_e2e * 1e3,
               "h2d_bytes_per_step": count * 4, "d2h_bytes_per_step": count * 4,
               "api": "torch.distributed.all_reduce" if args.impl == "nccl" else "cail_b200.ops.allreduce"}
        del h_in, h_out

    # ---------------- sweep
    def run_sweep(lo: int, hi: int) -> list:
        rows = []
        nbytes = lo
        while nbytes <= hi:
            n = nbytes // 4
            s, r = send[:n], recv[:n]
            iters = args.sweep_iters
            for _ in range(args.sweep_warmup):
                allreduce(s, r)
            comm.barrier()
            torch.cuda.synchronize()
            evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iters)]
            for a, b in evs:
                a.record()
                allreduce(s, r)
                b.record()
            torch.cuda.synchronize()
            ts = [a.elapsed_time(b) / 1e3 for a, b in evs]
            p50 = comm.max(statistics.median(ts))
            p99 = comm.max(sorted(ts)[min(len(ts) - 1, int(math.ceil(0.99 * len(ts))) - 1)])
            mean = comm.max(sum(ts) / len(ts))
            row = {"bytes": nbytes, "busbw": round(busbw(nbytes, mean, P), 2), "p50_us": round(p50 * 1e6, 2),
                   "p99_us": round(p99 * 1e6, 2), "iters": iters}
            if args.impl == "ours":
                import cail_b200
                row["algo"] = cail_b200.last_algorithm()
            rows.append(row)
            nbytes *= 2
        return rows

    sweep, sweep_ordered = [], []
    if not args.no_sweep:
        sweep = run_sweep(args.sweep_min, min(args.sweep_max, args.bytes))
        if args.impl == "ours" and P > 1:
            # small messages again with stream-ordered completion (the call
            # returns once queued, like NCCL's): the same events then time the
            # device work instead of the host round trip of a blocking call
            import cail_b200
            prev = cail_b200.set_stream_ordered(True)
            sweep_ordered = run_sweep(args.sweep_min, min(512 << 10, args.sweep_max, args.bytes))
            cail_b200.set_stream_ordered(bool(prev))
    clocks.__exit__(None, None, None)
    clock_summary = clocks.summary()
    if clock_summary is not None:
        clock_summary["window"] = "warm-up + timed region + e2e + sweep"

    out = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": P,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(t_step * 1e3, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "fp32",
        "data": "synthetic: normal(0,1) per element, seeded per rank",
        "impl": args.impl,
        "config": {
            "model": "MPI_Allreduce MPI_FLOAT MPI_SUM (collective library; no model)",
            "global_batch": count,
            "seq_len": None,
            "parallelism": f"allreduce over {P} rank(s), one per GPU",
            "msg_bytes": args.bytes,
            "buffers": "separate send/recv",
            "l2": "inputs (1 GiB) larger than the 126 MB L2; sweep sizes below 128 MB are L2-warm",
            "value_definition": ("busbw = 2(P-1)/P*bytes/t" if P > 1 else "algbw = bytes/t (busbw factor is 0 at P=1)"),
            "timing": "CUDA events around K calls, barrier+synchronize both sides, max over ranks",
        },
        "clocks": clock_summary,
        "e2e": e2e,
        "gpu_launches": (l1 - l0) if (l0 is not None and l1 is not None) else None,
        "check": check,
        "algorithm": algo,
        "sweep": sweep,
        "sweep_stream_ordered": sweep_ordered,
    }
    if rank == 0:
        print(json.dumps(out), flush=True)

    if args.impl == "nccl":
        import torch.distributed as dist
        if world > 1:
            dist.destroy_process_group()
    else:
        import cail_b200
        cail_b200.finalize()


if __name__ == "__main__":
    main()
