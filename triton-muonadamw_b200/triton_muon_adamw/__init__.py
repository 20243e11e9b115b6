"""B200-native MuonAdamW: drop-in replacement of the ``triton_muon_adamw`` package.

Exports the reference package's four names (``AdamConfig``, ``MuonAdamW``,
``MuonConfig``, ``PyTorchMuonAdamW``); the optimizer step runs as hand-written
sm_100a CUDA kernels behind a C ABI (``include/muon_adamw_b200.h``).
"""

from .optimizer import AdamConfig, MuonAdamW, MuonConfig, PyTorchMuonAdamW

__all__ = [
    "AdamConfig",
    "MuonAdamW",
    "MuonConfig",
    "PyTorchMuonAdamW",
]
