"""Models used by the benchmarks."""
from .gpt2 import GPT2, GPT2Config

__all__ = ["GPT2", "GPT2Config"]
