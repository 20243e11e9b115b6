"""CPU checks of the C-ABI library and the host-side Python layer (no GPU needed).

No compute call is made here: only loading, symbol export, argument
validation (which fails before any CUDA call) and plan sizing.
"""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest
import torch
import torch.nn as nn

from conftest import REPO

HEADER = REPO / "include" / "muon_adamw_b200.h"


def header_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(mad_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    from triton_muon_adamw import _lib
    lib = _lib.load()
    declared = header_functions()
    assert len(declared) >= 14
    for name in declared:
        assert hasattr(lib, name), f"{name} declared in {HEADER.name} but not exported"
    assert set(declared) == set(_lib.SIGNATURES), "ctypes signatures must cover exactly the header"
    assert lib.mad_abi_version() == 4


def test_invalid_arguments_fail_before_any_cuda_call():
    from triton_muon_adamw import _lib
    lib = _lib.load()
    rc = lib.mad_adamw_step(None, None, None, None, -1, 1e-3, 0.1, 0.1, 0.9, 0.999, 0.0, 1e-8, None)
    assert rc == 1 and b"negative numel" in lib.mad_last_error()
    rc = lib.mad_adamw_step(None, None, None, None, 10, 1e-3, 0.1, 0.1, 0.9, 0.999, 0.0, 1e-8, None)
    assert rc == 1 and b"null pointer" in lib.mad_last_error()
    # zero elements is a no-op, not an error
    assert lib.mad_adamw_step(None, None, None, None, 0, 1e-3, 0.1, 0.1, 0.9, 0.999, 0.0, 1e-8, None) == 0
    info = _lib.MuonPlanInfo()
    bad = (_lib.MuonMatrix * 1)(_lib.MuonMatrix(8, 8, 8, 0, 4, 1.0))
    assert lib.mad_muon_plan_size(bad, 1, ctypes.byref(info)) == 1
    assert b"shape" in lib.mad_last_error()
    assert lib.mad_muon_step_multi(ctypes.byref(info), None, 0.95, 1, 3.4, -4.7, 2.0, 0, 1e-7, 1e-3, 0.1, None) == 1


def test_plan_sizes_for_the_8b_shapes():
    """Tile counts of the plan follow from the shapes alone (upper-triangle tiles only)."""
    from oracle.muon_adamw_oracle import llama_8b_shapes
    from triton_muon_adamw import _lib
    lib = _lib.load()
    _, muon = llama_8b_shapes()
    arr = (_lib.MuonMatrix * len(muon))()
    for i, (r, c) in enumerate(muon):
        arr[i] = _lib.MuonMatrix(16, 16, 16, r, c, 1.0)     # fake, aligned, never dereferenced
    info = _lib.MuonPlanInfo()
    _lib.check(lib.mad_muon_plan_size(arr, len(muon), ctypes.byref(info)))

    def tri(m):           # 256 x 256 pair tiles on or above the diagonal
        t = -(-m // 256)
        return t * (t + 1) // 2

    counts = {}
    for s in muon:
        counts[s] = counts.get(s, 0) + 1
    exp_gram = sum(cnt * tri(min(s)) for s, cnt in counts.items())
    exp_upd = sum(cnt * (-(-min(s) // 256)) * (-(-max(s) // 256)) for s, cnt in counts.items())
    assert info.gram_tiles == exp_gram == info.poly_tiles
    assert info.update_tiles == exp_upd
    # bf16 workspaces: 2 iterates (m x n) + A, B (m x m), rows padded to 64
    exp_work = sum(cnt * (2 * min(s) * max(s) * 2 + 2 * min(s) ** 2 * 2) for s, cnt in counts.items())
    assert info.work_bytes == exp_work
    assert info.table_bytes < 64 << 20


class Tiny(nn.Module):
    def __init__(self, tied=True):
        super().__init__()
        self.emb = nn.Embedding(32, 8)
        self.l1 = nn.Linear(8, 16)
        self.ln = nn.LayerNorm(16)
        self.l2 = nn.Linear(16, 8, bias=False)
        self.head = nn.Linear(8, 32, bias=False)
        if tied:
            self.head.weight = self.emb.weight
        self.frozen = nn.Parameter(torch.zeros(4, 4), requires_grad=False)

    def get_input_embeddings(self):
        return self.emb

    def get_output_embeddings(self):
        return self.head


@pytest.mark.parametrize("tied", [True, False])
def test_auto_split_matches_reference_routing(tied):
    from oracle.muon_adamw_oracle import split_params
    from triton_muon_adamw.optimizer import split_parameters
    m = Tiny(tied)
    adam, muon = split_parameters(m, "auto")
    ref_adam, ref_muon = split_params(model=m)
    assert [id(p) for p in adam] == [id(p) for p in ref_adam]
    assert [id(p) for p in muon] == [id(p) for p in ref_muon]
    assert [tuple(p.shape) for p in muon] == [(16, 8), (8, 16)]
    assert sum(p is m.emb.weight for p in adam) == 1


def test_split_errors_match_reference():
    from triton_muon_adamw.optimizer import split_parameters
    with pytest.raises(ValueError, match="explicit"):
        split_parameters(Tiny(), "explicit")
    with pytest.raises(ValueError, match="auto"):
        split_parameters({"adam": [], "muon": []}, "auto")
    with pytest.raises(AttributeError):
        split_parameters(nn.Linear(2, 2), "auto")


def test_configs_match_reference_defaults():
    """Field names, order and defaults of optimizer.py:14-67 in the reference."""
    from dataclasses import fields
    from triton_muon_adamw import AdamConfig, MuonConfig
    assert [(f.name, f.default) for f in fields(AdamConfig)] == [
        ("lr", 1e-3), ("betas", (0.9, 0.999)), ("eps", 1e-7), ("weight_decay", 0.01)]
    assert [(f.name, f.default) for f in fields(MuonConfig)] == [
        ("lr", 1e-3), ("beta", 0.95), ("eps", 1e-7), ("weight_decay", 0.1), ("coeffs", (3.445, -4.775, 2.0315)),
        ("nesterov", True), ("ns_steps", 5), ("adjust_lr_fn", "original")]


def test_bad_adjust_lr_fn_raises_assertion():
    from triton_muon_adamw import MuonAdamW, MuonConfig
    with pytest.raises(AssertionError):
        MuonAdamW({"adam": [], "muon": []}, muon_config=MuonConfig(adjust_lr_fn="bogus"), parameter_split="explicit")


def test_product_path_refuses_cpu_tensors():
    """There is no CPU implementation: a CPU parameter fails loudly at step()."""
    from triton_muon_adamw import MuonAdamW
    m = Tiny()
    for p in m.parameters():
        p.grad = torch.zeros_like(p)
    opt = MuonAdamW(m)
    with pytest.raises(ValueError, match="CUDA"):
        opt.step()


def test_lr_scale_matches_oracle():
    from oracle.muon_adamw_oracle import scaled_lr
    from triton_muon_adamw.muon.cuda_muon import lr_scale
    for fn in ("original", "match_rms_adamw", "spectral_unclamped"):
        for shape in [(4096, 1024), (1024, 4096), (7, 7), (14336, 4096)]:
            assert 1e-3 * lr_scale(shape, fn) == pytest.approx(scaled_lr(1e-3, shape, fn), rel=1e-15)


def test_state_dict_layout_matches_torch_wrapper():
    """state_dict() of MuonAdamW has the layout of PyTorchMuonAdamW.state_dict() (CPU, before any step)."""
    from triton_muon_adamw import MuonAdamW, PyTorchMuonAdamW
    m = Tiny()
    ours = MuonAdamW(m).state_dict()
    ref = PyTorchMuonAdamW(Tiny()).state_dict()
    assert set(ours) == set(ref) == {"adam", "muon"}
    for k in ("adam", "muon"):
        assert set(ours[k]) == set(ref[k])
        og, rg = ours[k]["param_groups"][0], ref[k]["param_groups"][0]
        assert og["params"] == rg["params"]
        for key in ("lr", "weight_decay"):
            assert og[key] == rg[key]
    assert set(ours["muon"]["state"][0]) == {"momentum_buffer"}


def test_table_layout_constants_match_the_device_structs():
    """Tests that read the device plan table directly use these sizes; plan.cuh pins them with static_asserts."""
    import re
    from pathlib import Path

    from test_gpu_parity import INV_NORM_OFFSET, MATDESC_BYTES
    src = (Path(__file__).resolve().parent.parent / "triton-muonadamw_b200" / "csrc" / "plan.cuh").read_text()
    assert re.search(r"sizeof\(MatDesc\) == (\d+)", src).group(1) == str(MATDESC_BYTES)
    body = src[src.index("struct MatDesc {"):src.index("float inv_norm;")]
    off = 0
    for line in body.splitlines()[1:]:
        decl = line.split("//")[0].strip().rstrip(";")
        if not decl:
            continue
        names = [n.strip() for n in decl.split(None, 1)[1].split(",")] if "*" not in decl else [decl.split("*")[1]]
        size = 8 if ("*" in decl or decl.startswith(("double", "int64_t"))) else 4
        for n in names:
            m = re.search(r"\[(\d+)\]", n)
            off += size * (int(m.group(1)) if m else 1)
    assert off == INV_NORM_OFFSET


def test_ctypes_structures_match_the_c_header(tmp_path):
    """Every struct of include/muon_adamw_b200.h, compiled by gcc, has the ctypes binding's size and offsets."""
    import shutil
    import subprocess
    from pathlib import Path

    from triton_muon_adamw import _lib
    if shutil.which("gcc") is None:
        pytest.skip("gcc not available")
    include = Path(__file__).resolve().parent.parent / "include"
    structs = {"mad_adamw_tensor": _lib.AdamWTensor, "mad_muon_matrix": _lib.MuonMatrix,
               "mad_muon_plan_info": _lib.MuonPlanInfo, "mad_muon_buffers": _lib.MuonBuffers,
               "mad_grad_reduce": _lib.GradReduce, "mad_peer_set": _lib.PeerSet}
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "muon_adamw_b200.h"', "int main(void) {"]
    for cname, cls in structs.items():
        lines.append(f'printf("{cname} size %zu\\n", sizeof({cname}));')
        for field, _ in cls._fields_:
            lines.append(f'printf("{cname} {field} %zu\\n", offsetof({cname}, {field}));')
    lines += ['printf("MAD_MAX_RANKS %d\\n", MAD_MAX_RANKS);', 'printf("MAD_IPC_HANDLE_BYTES %d\\n", MAD_IPC_HANDLE_BYTES);',
              'printf("MAD_DTYPE_F32_MASTER %d\\n", (int)MAD_DTYPE_F32_MASTER);', "return 0; }"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c11", "-I", str(include), str(src), "-o", str(exe)], check=True)
    out = dict(line.rsplit(" ", 1) for line in subprocess.run([str(exe)], check=True, capture_output=True,
                                                               text=True).stdout.splitlines())
    for cname, cls in structs.items():
        assert int(out[f"{cname} size"]) == ctypes.sizeof(cls), cname
        for field, _ in cls._fields_:
            assert int(out[f"{cname} {field}"]) == getattr(cls, field).offset, (cname, field)
    assert int(out["MAD_MAX_RANKS"]) == _lib.MAX_RANKS
    assert int(out["MAD_IPC_HANDLE_BYTES"]) == _lib.IPC_HANDLE_BYTES
    assert int(out["MAD_DTYPE_F32_MASTER"]) == _lib.DTYPE_F32_MASTER


def test_muonadamw_rejects_bad_options_before_touching_the_gpu():
    """Argument errors surface at construction, on any device (construction makes no CUDA call)."""
    from triton_muon_adamw import MuonAdamW
    params = {"adam": [nn.Parameter(torch.zeros(4))], "muon": [nn.Parameter(torch.zeros(4, 4))]}
    with pytest.raises(ValueError):
        MuonAdamW(params, parameter_split="explicit", peer_push="bogus")
    with pytest.raises(ValueError):
        MuonAdamW(params, parameter_split="explicit", reduce_grads="max")
    with pytest.raises(TypeError):
        MuonAdamW(params, parameter_split="explicit", master_weights=True)     # float32 parameters
    opt = MuonAdamW({k: [nn.Parameter(p.detach().to(torch.bfloat16)) for p in v] for k, v in params.items()},
                    parameter_split="explicit", master_weights=True)
    assert all(m.dtype == torch.float32 for m in opt.muon.masters.values())
    assert all(m.dtype == torch.float32 for m in opt.muon.momentum.values())


@pytest.mark.parametrize("bad_delta", [8, 4, -24, 1])
def test_gradient_reduction_rejects_unaligned_peer_deltas_before_any_launch(bad_delta):
    """Peer copies are read with 16-byte vector loads at g + delta[k]: a delta off that grid is refused."""
    from triton_muon_adamw import _lib
    lib = _lib.load()
    red = _lib.GradReduce(2, 0.5)
    red.delta[0], red.delta[1] = 0, 1 << 20
    red.delta[1] += bad_delta
    fake_table = ctypes.c_void_p(0x10000)      # never dereferenced: the check fails first
    rc = lib.mad_adamw_step_multi_reduce(fake_table, 1, 1e-3, 0.9, 0.999, 1e-8, 0.01, 0.1, 0.1,
                                         ctypes.byref(red), None)
    assert rc == 2 and b"not a multiple of 16" in lib.mad_last_error()
    info = _lib.MuonPlanInfo()
    info.n_mats = 1
    rc = lib.mad_muon_prep_reduce(ctypes.byref(info), fake_table, 0.95, 1, 1e-7, ctypes.byref(red), None)
    assert rc == 2 and b"not a multiple of 16" in lib.mad_last_error()
    rc = lib.mad_muon_step_multi_reduce(ctypes.byref(info), fake_table, 0.95, 1, 3.4, -4.7, 2.0, 5, 1e-7, 1e-3,
                                        0.1, ctypes.byref(red), None)
    assert rc == 2 and b"not a multiple of 16" in lib.mad_last_error()


def test_reference_install_is_importable_beside_ours():
    """The unmodified reference under baseline/_ref loads under its alias without shadowing our package."""
    import triton_muon_adamw as ours
    from reference_pkg import load_reference
    R = load_reference()
    assert R.__name__ == "ref_triton_muon_adamw" and R.MuonAdamW is not ours.MuonAdamW
    assert "baseline" in R.__file__ and "baseline" not in ours.__file__
    assert hasattr(R.muon.triton_muon, "TritonMuon") and hasattr(R, "PyTorchMuonAdamW")
