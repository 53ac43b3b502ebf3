"""Collective operations on tensors (the interposed MPI_Allreduce)."""
from .allreduce import allreduce, allreduce_, mpi_datatype, mpi_op

__all__ = ["allreduce", "allreduce_", "mpi_datatype", "mpi_op"]
