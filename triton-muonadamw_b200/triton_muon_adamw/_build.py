"""Build the CUDA library in-tree for sm_100a.

    python -m triton_muon_adamw._build

compiles ``../csrc/*.cu`` with nvcc into ``libmuonadamw_b200.so`` next to this
file.  nvcc cross-compiles, so no GPU is needed.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE.parent / "csrc"
INCLUDE = HERE.parent.parent / "include"
OUT = HERE / "libmuonadamw_b200.so"
SOURCES = ["capi.cu", "adamw.cu", "muon_prep.cu", "ns_gemm.cu", "muon_plan.cu", "muon_noalloc.cu", "p2p.cu", "patch.cu"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise FileNotFoundError("nvcc not found")


def needs_rebuild() -> bool:
    if not OUT.exists():
        return True
    t = OUT.stat().st_mtime
    deps = [CSRC / s for s in SOURCES] + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h"))
    deps.append(INCLUDE / "muon_adamw_b200.h")
    return any(d.exists() and d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not needs_rebuild():
        return OUT
    tmp = OUT.with_suffix(".so.tmp")
    cmd = [nvcc_path(), *ARCH_FLAGS, "-lineinfo", "-O3", "-std=c++17", f"-I{INCLUDE}", "-Xcompiler", "-fPIC", "-shared",
           "-o", str(tmp), *[str(CSRC / s) for s in SOURCES]]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
