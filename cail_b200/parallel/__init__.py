"""Data parallelism on top of the interposed MPI_Allreduce."""
from .ddp import BucketedAllreduce

__all__ = ["BucketedAllreduce"]
