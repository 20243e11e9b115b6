"""AdamW branch (CUDA multi-tensor kernel); the class keeps the reference's name."""

from .cuda_adam import TritonAdamW

__all__ = ["TritonAdamW"]
