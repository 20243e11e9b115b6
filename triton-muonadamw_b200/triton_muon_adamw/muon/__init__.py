"""Muon branch (tcgen05 Newton-Schulz kernels); the class keeps the reference's name."""

from .cuda_muon import TritonMuon

__all__ = ["TritonMuon"]
