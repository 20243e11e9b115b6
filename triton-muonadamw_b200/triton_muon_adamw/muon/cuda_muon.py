"""Muon branch of MuonAdamW on the B200: prep + ns_steps x (Gram, polynomial, update).

Replaces the reference's ``TritonMuon`` (triton_muon.py:375-457), keeping its
name, constructor, attributes (``model_params``, ``momentum``, ``a``, ``b``,
``c``, ``beta``, ``lr``, ``weight_decay``, ``steps``, ``eps``,
``is_nesterov``, ``adjust_lr_fn``) and behaviour: momentum buffers in the
parameter dtype allocated at construction, parameters whose ``grad`` is
``None`` skipped, ``AssertionError`` for an unknown ``adjust_lr_fn`` or a
non-2-D parameter.

The reference runs ~27 launches per matrix; ``step()`` runs 2 + 3*ns_steps
launches for all matrices together (``mad_muon_step_multi``), over a plan
(tensor maps, tile lists, bf16 workspaces) built once and rebuilt only when a
tensor's storage changes.
"""

from __future__ import annotations

import ctypes
import math
from collections.abc import Iterable
from typing import Literal

import torch
import torch.nn as nn

from .. import _lib
from ..adamw.cuda_adam import dtype_code, entry_dtype

ADJUST_LR_FNS = ("original", "match_rms_adamw", "spectral_unclamped")


def lr_scale(shape, adjust_lr_fn: str) -> float:
    """Shape factor of the Muon learning rate, ``scaled_lr = lr * lr_scale`` (triton_muon.py:424-431).

    ``match_rms_adamw`` follows torch's definition ``0.2*sqrt(max(rows, cols))``;
    the reference's own expression raises a ``TypeError`` (``max`` of an int).
    """
    rows, cols = int(shape[0]), int(shape[1])
    if adjust_lr_fn == "original":
        return math.sqrt(max(1, rows / cols))
    if adjust_lr_fn == "match_rms_adamw":
        return 0.2 * math.sqrt(max(rows, cols))
    return math.sqrt(rows / cols)


class MuonPlan:
    """Device plan for a fixed list of (param, grad, momentum[, shadow]) matrices.

    Each matrix is float32 or bf16 throughout, or a float32 master (and
    momentum) with a bf16 grad and a bf16 shadow written with the update.
    """

    def __init__(self):
        self.key = None
        self.grads = None
        self.replans = 0
        self.info = _lib.MuonPlanInfo()
        self.table = None
        self.work = None
        self.buffers = None
        self.n_mats = 0
        self.shapes = []

    def ensure(self, triples, adjust_lr_fn, device) -> None:
        """Plan (or keep) the plan for these matrices.

        Gradient addresses are not part of the key: when only they changed,
        ``mad_muon_set_grads`` rewrites them in place on the stream (old and
        new addresses all 16-byte aligned) -- no tensor-map encodes, no upload,
        no synchronisation.
        """
        triples = [tuple(t) + (None,) * (4 - len(t)) for t in triples]
        key = (adjust_lr_fn,) + tuple((p.data_ptr(), m.data_ptr(), tuple(p.shape), p.dtype, g.dtype,
                                       sh.data_ptr() if sh is not None else 0) for p, g, m, sh in triples)
        grads = tuple(t[1].data_ptr() for t in triples)
        if key == self.key:
            if grads == self.grads:
                return
            if all(a % 16 == 0 for a in grads) and all(a % 16 == 0 for a in self.grads):
                lib = _lib.load()
                arr = (ctypes.c_void_p * max(1, len(grads)))(*grads)
                _lib.check(lib.mad_muon_set_grads(ctypes.byref(self.info), self.table.data_ptr(), arr,
                                                  _lib.stream_handle()), "mad_muon_set_grads")
                self.grads = grads
                return
        lib = _lib.load()
        n = len(triples)
        arr = (_lib.MuonMatrix * max(1, n))()
        for i, (p, g, m, sh) in enumerate(triples):
            arr[i] = _lib.MuonMatrix(p.data_ptr(), g.data_ptr(), m.data_ptr(), p.shape[0], p.shape[1],
                                     lr_scale(p.shape, adjust_lr_fn), entry_dtype(p, g, sh, "Muon parameter"), 0,
                                     sh.data_ptr() if sh is not None else None)
        info = _lib.MuonPlanInfo()
        _lib.check(lib.mad_muon_plan_size(arr, n, ctypes.byref(info)), "mad_muon_plan_size")
        self.table = torch.empty(max(1, info.table_bytes), dtype=torch.uint8, device=device)
        # 1024-byte aligned view of the work buffer (TMA swizzle atoms).
        raw = torch.empty(info.work_bytes + 1024, dtype=torch.uint8, device=device)
        off = (-raw.data_ptr()) % 1024
        self._work_raw = raw
        self.work = raw[off:off + info.work_bytes]
        bufs = (_lib.MuonBuffers * max(1, n))()
        _lib.check(lib.mad_muon_plan(arr, n, self.table.data_ptr(), self.work.data_ptr() if n else None,
                                     ctypes.byref(info), bufs, _lib.stream_handle()), "mad_muon_plan")
        self.info = info
        self.buffers = bufs
        self.n_mats = n
        self.shapes = [tuple(t[0].shape) for t in triples]
        self.key = key
        self.grads = grads
        self.replans += 1

    def read_status(self, clear=True) -> int:
        st = ctypes.c_uint32(0)
        if self.n_mats:
            lib = _lib.load()
            _lib.check(lib.mad_muon_read_status(ctypes.byref(self.info), self.table.data_ptr(), ctypes.byref(st),
                                                1 if clear else 0, _lib.stream_handle()), "mad_muon_read_status")
        return st.value


def run_muon_plan(plan: MuonPlan, *, beta, nesterov, a, b, c, ns_steps, eps, lr, weight_decay, timer=None,
                  stream=None, reduce=None, reserve_sms: int = 0) -> None:
    """Launch the whole Muon branch for a plan on the current (or given) stream.

    Without a timer this is one C call (``mad_muon_step_multi``); with one,
    the same launches are issued phase by phase with a CUDA event between
    them so each kernel can be timed on its launching stream.  ``reduce`` (a
    ``GradReduce``) makes the prep sum each gradient over ranks;
    ``reserve_sms`` SMs are left free by the GEMMs (``mad_set_gemm_sm_reserve``).
    """
    if plan.n_mats == 0:
        return
    lib = _lib.load()
    _lib.check(lib.mad_set_gemm_sm_reserve(int(reserve_sms)), "mad_set_gemm_sm_reserve")
    info, tab, st = ctypes.byref(plan.info), plan.table.data_ptr(), _lib.stream_handle(stream)
    nest = 1 if nesterov else 0
    if timer is None:
        if reduce is None:
            _lib.check(lib.mad_muon_step_multi(info, tab, beta, nest, a, b, c, ns_steps, eps, lr, weight_decay, st),
                       "mad_muon_step_multi")
        else:
            _lib.check(lib.mad_muon_step_multi_reduce(info, tab, beta, nest, a, b, c, ns_steps, eps, lr,
                                                      weight_decay, ctypes.byref(reduce), st),
                       "mad_muon_step_multi_reduce")
        return
    timer.mark("prep")
    if reduce is None:
        _lib.check(lib.mad_muon_prep(info, tab, beta, nest, eps, st), "mad_muon_prep")
    else:
        _lib.check(lib.mad_muon_prep_reduce(info, tab, beta, nest, eps, ctypes.byref(reduce), st),
                   "mad_muon_prep_reduce")
    for it in range(ns_steps):
        timer.mark("gram")
        _lib.check(lib.mad_ns_gram(info, tab, it, st), "mad_ns_gram")
        timer.mark("poly")
        _lib.check(lib.mad_ns_poly(info, tab, it, b, c, st), "mad_ns_poly")
        last = it == ns_steps - 1
        timer.mark("update_last" if last else "update")
        _lib.check(lib.mad_ns_update(info, tab, it, 1 if last else 0, a, lr, weight_decay, st), "mad_ns_update")
    timer.mark(None)


class TritonMuon:
    """Muon over float32 or bf16 CUDA matrices with hand-written sm_100a kernels.

    The name is the reference's (``triton_muon_adamw.muon.TritonMuon``) so
    imports keep working; there is no Triton code behind it.
    """

    def __init__(
        self,
        params: Iterable[nn.Parameter] | list[nn.Parameter],
        lr: float = 1e-3,
        weight_decay: float = 0.1,
        coeffs: tuple[float, float, float] = (3.445, -4.775, 2.0315),
        nesterov: bool = True,
        beta: float = 0.95,
        ns_steps: int = 5,
        eps: float = 1e-7,
        adjust_lr_fn: Literal["original", "match_rms_adamw", "spectral_unclamped"] = "original",
    ):
        if adjust_lr_fn not in ADJUST_LR_FNS:
            raise AssertionError(f"Invalid adjust_lr_fn: {adjust_lr_fn}")
        self.model_params = list(params)
        self.a = coeffs[0]
        self.b = coeffs[1]
        self.c = coeffs[2]
        self.is_nesterov = nesterov
        self.beta = beta
        self.lr = lr
        self.adjust_lr_fn = adjust_lr_fn
        self.weight_decay = weight_decay
        self.steps = ns_steps
        self.eps = eps
        self.momentum = {}
        for param in self.model_params:
            self.momentum[param] = torch.zeros_like(param, device=param.device, dtype=param.dtype)
        self.masters = None  # {param: float32 master} in mixed-precision mode (MuonAdamW(master_weights=True))
        self._plan = MuonPlan()

    def _active(self, only=None):
        triples = []
        for p in (self.model_params if only is None else only):
            if p.grad is None:
                continue
            if p.ndim != 2:
                raise AssertionError("Muon only supports 2D tensors")
            for t, what in ((p, "Muon parameter"), (p.grad, "Muon gradient")):
                if not t.is_cuda:
                    raise ValueError(f"{what} must be a CUDA tensor (this optimizer runs only on the GPU)")
                dtype_code(t, what)
                if t.dtype != p.dtype:
                    raise TypeError(f"{what} must have the parameter's dtype {p.dtype}, got {t.dtype}")
                if not t.is_contiguous():
                    raise ValueError(f"{what} must be contiguous")
            if p.numel() == 0:
                continue
            if self.masters is not None:
                triples.append((self.masters[p], p.grad, self.momentum[p], p.data))
            else:
                triples.append((p.data, p.grad, self.momentum[p]))
        return triples

    @torch.no_grad()
    def step(self):
        """One Muon update of every matrix that has a gradient (triton_muon.py:414-448)."""
        if self.steps < 1:
            raise ValueError("ns_steps must be >= 1")
        triples = self._active()
        if not triples:
            return
        self._plan.ensure(triples, self.adjust_lr_fn, triples[0][0].device)
        run_muon_plan(self._plan, beta=self.beta, nesterov=self.is_nesterov, a=self.a, b=self.b, c=self.c,
                      ns_steps=self.steps, eps=self.eps, lr=self.lr, weight_decay=self.weight_decay,
                      timer=getattr(self, "_timer", None))

    def device_status(self, clear: bool = True) -> int:
        """Error bits the Muon kernels recorded since the last read (0 = healthy); synchronises."""
        return self._plan.read_status(clear)

    def zero_grad(self):
        """Reset gradients to zero in place (triton_muon.py:450-456)."""
        for param in self.model_params:
            if param.grad is not None:
                param.grad.zero_()
