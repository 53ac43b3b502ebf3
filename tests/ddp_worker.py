"""Worker for test_ddp.py: one rank of a data-parallel step of a tiny GPT-2.

Every rank builds the same model (same seed), runs forward/backward on its
own synthetic batch with gradients bucketed and all-reduced through the
interposed MPI_Allreduce, then checks the averaged gradients against a
single-process reference that sees all ranks' batches.
"""
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import cail_b200 as cail  # noqa: E402
from cail_b200.models import GPT2, GPT2Config  # noqa: E402
from cail_b200.parallel import BucketedAllreduce  # noqa: E402


def batch(r, c):
    g = torch.Generator().manual_seed(100 + r)
    idx = torch.randint(0, c.vocab, (2, c.n_ctx), generator=g)
    tgt = torch.randint(0, c.vocab, (2, c.n_ctx), generator=g)
    return idx, tgt


def main():
    device = sys.argv[1] if len(sys.argv) > 1 else "cpu"
    rank = cail.init("ours", host=(device == "cpu"))
    P = cail.world_size()
    if device == "cuda":
        torch.cuda.set_device(int(os.environ.get("CMPI_LOCAL_RANK", rank)) % torch.cuda.device_count())
    c = GPT2Config.tiny()
    torch.manual_seed(0)
    model = GPT2(c).to(device)
    ref = GPT2(c).to(device)
    ref.load_state_dict(model.state_dict())
    ddp = BucketedAllreduce(model, P, bucket_bytes=64 << 10)
    assert ddp.num_buckets > 1
    for step in range(2):
        ddp.zero_grad()
        idx, tgt = batch(rank + 10 * step, c)
        model(idx.to(device), tgt.to(device)).backward()
        ddp.finish()
        ddp.check_views(model)
        ref.zero_grad()
        loss = sum(ref(*(t.to(device) for t in batch(r + 10 * step, c))) for r in range(P)) / P
        loss.backward()
        worst = max((p.grad - q.grad).abs().max().item() for p, q in zip(model.parameters(), ref.parameters()))
        if worst > 1e-5:
            print(f"rank {rank}: step {step} gradient mismatch {worst:.3e}", flush=True)
            sys.exit(1)
    ddp.close()
    if rank == 0:
        print(f"DDP OK P={P} buckets={ddp.num_buckets}", flush=True)
    cail.finalize()


if __name__ == "__main__":
    main()
