"""Back-compatible import path: ``from MuonAdamW import MuonAdamW, ...``.

Mirrors the reference's top-level shim (``MuonAdamW package/MuonAdamW.py``).
"""

from triton_muon_adamw import AdamConfig, MuonAdamW, MuonConfig, PyTorchMuonAdamW

__all__ = ["AdamConfig", "MuonAdamW", "MuonConfig", "PyTorchMuonAdamW"]
