"""Utilities: clock sampling, launching minimpi jobs."""
from .clocks import ClockSampler

__all__ = ["ClockSampler"]
