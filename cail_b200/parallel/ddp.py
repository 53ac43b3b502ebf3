"""Data-parallel gradient allreduce with bucketing and backward overlap.

Gradients live in flat fp32 bucket buffers of ~25 MB (each parameter's
``.grad`` is a view into its bucket, so autograd accumulates straight into
them).  Buckets are formed in reverse parameter order, the order in which
backward produces gradients.  When every gradient of a bucket has been
accumulated (post-accumulate-grad hooks) an event is recorded on the
compute stream and the bucket is queued to a communication thread, which
waits for the event and calls MPI_Allreduce(MPI_IN_PLACE, bucket, MPI_FLOAT,
MPI_SUM) through the cail_torch extension with the GIL released.  cail runs
the reduction on its own CUDA stream, so it overlaps the rest of backward.
``finish()`` waits for all buckets and averages them.
"""
from __future__ import annotations

import queue
import threading
from typing import Dict, List

import torch

from .. import _lib


class BucketedAllreduce:
    def __init__(self, model: torch.nn.Module, world_size: int, bucket_bytes: int = 25 << 20,
                 comm: int | None = None, enabled: bool = True):
        self.world = world_size
        self.enabled = enabled and world_size > 1
        self.comm = _lib.H["MPI_COMM_WORLD"] if comm is None else comm
        params = [p for p in model.parameters() if p.requires_grad]
        if any(p.dtype != torch.float32 for p in params):
            raise TypeError("the harness reduces fp32 gradients (MPI_FLOAT)")
        groups: List[List[torch.nn.Parameter]] = [[]]
        size = 0
        for p in reversed(params):
            groups[-1].append(p)
            size += p.numel() * 4
            if size >= bucket_bytes:
                groups.append([])
                size = 0
        groups = [g for g in groups if g]
        self.flats: List[torch.Tensor] = []
        self.bucket_of: Dict[int, int] = {}
        self.sizes = [len(g) for g in groups]
        dev = params[0].device
        for b, g in enumerate(groups):
            flat = torch.zeros(sum(p.numel() for p in g), dtype=torch.float32, device=dev)
            off = 0
            for p in g:
                p.grad = flat[off:off + p.numel()].view_as(p)
                off += p.numel()
                self.bucket_of[id(p)] = b
                p.register_post_accumulate_grad_hook(self._ready)
            self.flats.append(flat)
        self.remaining = list(self.sizes)
        self.done = [threading.Event() for _ in groups]
        self.errors: List[str] = []
        self.q: "queue.Queue" = queue.Queue()
        self.thread = None
        if self.enabled:
            from ..ops import ext

            self.ext = ext.get()
            libs = _lib.loaded()
            if libs.impl == "ours":
                # each bucket's producer event is waited for before its call,
                # so cail need not order itself after the legacy stream (which
                # would make it wait for the whole queued backward)
                libs.cail.cail_set_stream_sync(0)
            self.thread = threading.Thread(target=self._worker, daemon=True)
            self.thread.start()

    @property
    def num_buckets(self) -> int:
        return len(self.flats)

    def _ready(self, p: torch.Tensor) -> None:
        b = self.bucket_of[id(p)]
        self.remaining[b] -= 1
        if self.remaining[b] == 0:
            if not self.enabled:
                self.done[b].set()
                return
            ev = torch.cuda.Event() if p.is_cuda else None
            if ev is not None:
                ev.record()
            self.q.put((b, ev))

    def _worker(self) -> None:
        dt, op = _lib.H["MPI_FLOAT"], _lib.H["MPI_SUM"]
        # A new thread starts on device 0.  CUDA-aware MPIs (the reference
        # among them) allocate scratch and launch on the calling thread's
        # current device, so it must be the buckets' device.
        if self.flats and self.flats[0].is_cuda:
            torch.cuda.set_device(self.flats[0].device)
        while True:
            item = self.q.get()
            if item is None:
                return
            b, ev = item
            if ev is not None:
                ev.synchronize()
            rc = self.ext.allreduce_inplace(self.flats[b], dt, op, self.comm)
            if rc != 0:
                self.errors.append(f"bucket {b}: MPI_Allreduce returned {rc}")
            self.done[b].set()

    def zero_grad(self) -> None:
        for f in self.flats:
            f.zero_()
        self.remaining = list(self.sizes)
        for d in self.done:
            d.clear()

    def check_views(self, model: torch.nn.Module) -> None:
        """Asserts that autograd accumulated into the bucket views."""
        for p in model.parameters():
            if p.requires_grad:
                flat = self.flats[self.bucket_of[id(p)]]
                base = flat.data_ptr()
                if not (base <= p.grad.data_ptr() < base + flat.numel() * 4):
                    raise RuntimeError("a gradient left its bucket view")

    def finish(self) -> None:
        """Waits for every bucket and averages the gradients."""
        for d in self.done:
            d.wait()
        if self.errors:
            raise RuntimeError("; ".join(self.errors))
        if self.enabled:
            for f in self.flats:
                f.mul_(1.0 / self.world)

    def close(self) -> None:
        if self.thread is not None:
            self.q.put(None)
            self.thread.join()
            self.thread = None
