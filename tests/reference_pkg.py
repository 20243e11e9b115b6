"""Import the unmodified reference package for side-by-side GPU tests.

The reference (Mithun-033/Triton-MuonAdamW, ``MuonAdamW package/``) is
installed unmodified under ``baseline/_ref`` (a pure-Python wheel of its
``triton_muon_adamw/`` files, installed with ``pip --target``).  Its package
has the same import name as ours, ``triton_muon_adamw``, so it is loaded here
under the alias ``ref_triton_muon_adamw``; its modules use relative imports
only, so nothing of it resolves to our package.  Test infrastructure only.
"""

from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

REF_ROOT = Path(__file__).resolve().parent.parent / "baseline" / "_ref"
ALIAS = "ref_triton_muon_adamw"


def load_reference():
    """The reference package (``MuonAdamW``, ``PyTorchMuonAdamW``, configs; ``.muon.TritonMuon``)."""
    if ALIAS in sys.modules:
        return sys.modules[ALIAS]
    init = REF_ROOT / "triton_muon_adamw" / "__init__.py"
    if not init.exists():
        raise FileNotFoundError(
            f"{init} is missing: install the reference package into baseline/_ref "
            "(pip install --no-deps --target baseline/_ref) before running the reference parity tests")
    spec = importlib.util.spec_from_file_location(ALIAS, init, submodule_search_locations=[str(init.parent)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[ALIAS] = mod
    try:
        spec.loader.exec_module(mod)
    except BaseException:
        del sys.modules[ALIAS]
        raise
    importlib.import_module(f"{ALIAS}.muon.triton_muon")
    importlib.import_module(f"{ALIAS}.adamw.triton_adam")
    return mod
