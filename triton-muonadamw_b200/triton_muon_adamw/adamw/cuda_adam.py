"""AdamW branch of MuonAdamW on the B200: one multi-tensor CUDA launch per step.

Replaces the reference's ``TritonAdamW`` (triton_adam.py:106-161), keeping
its name, constructor, attributes (``model_params``, ``m``, ``v``,
``step_num``, ``lr``, ``beta1``, ``beta2``, ``weight_decay``, ``eps``) and
behaviour: float32 or bf16 parameters (the gradient of the parameter's dtype),
float32 ``exp_avg``/``exp_avg_sq`` allocated at construction, one
branch-global step count for the bias corrections, parameters whose ``grad``
is ``None`` skipped, ``zero_grad`` zeroing gradients in place.

Where the reference launches one Triton kernel per tensor, ``step()`` launches
one kernel for all tensors (``mad_adamw_step_multi``), driven by a tile table
that is rebuilt only when a tensor's storage changes.
"""

from __future__ import annotations

import ctypes
import weakref
from collections.abc import Iterable

import torch
import torch.nn as nn

from .. import _lib


DTYPE_CODES = {torch.float32: _lib.DTYPE_F32, torch.bfloat16: _lib.DTYPE_BF16}


def dtype_code(t: torch.Tensor, what: str) -> int:
    """C-ABI element-type code of a parameter/gradient/momentum tensor."""
    code = DTYPE_CODES.get(t.dtype)
    if code is None:
        raise TypeError(f"{what} must be float32 or bfloat16, got {t.dtype}")
    return code


def _check_tensor(p: torch.Tensor, what: str, dtype: torch.dtype | None = None) -> None:
    if not p.is_cuda:
        raise ValueError(f"{what} must be a CUDA tensor (this optimizer runs only on the GPU)")
    dtype_code(p, what)
    if dtype is not None and p.dtype != dtype:
        raise TypeError(f"{what} must have dtype {dtype}, got {p.dtype}")
    if not p.is_contiguous():
        raise ValueError(f"{what} must be contiguous")


def entry_dtype(p: torch.Tensor, g: torch.Tensor, shadow, what: str) -> int:
    """C-ABI dtype of one (param, grad[, shadow]) entry: F32, BF16, or a float32 master with bf16 grad/shadow."""
    if shadow is not None:
        if p.dtype != torch.float32 or g.dtype != torch.bfloat16 or shadow.dtype != torch.bfloat16:
            raise TypeError(f"{what}: a master entry needs a float32 master and bf16 gradient and shadow")
        return _lib.DTYPE_F32_MASTER
    return dtype_code(p, what)


class AdamWTable:
    """Device tile table over a list of (param, grad, exp_avg, exp_avg_sq[, shadow]) views.

    param and grad share one dtype (float32 or bf16), or param is a float32
    master with a bf16 grad and a bf16 shadow (the model's parameter, written
    with the update); the moments are float32.
    """

    def __init__(self):
        self.key = None
        self.grads = None
        self.table = None
        self.n_tiles = 0
        self.numel = 0
        self.replans = 0

    def ensure(self, quads, device) -> None:
        """Plan (or keep) the table for these tensors.

        The key leaves the gradient addresses out: when only they changed (new
        ``.grad`` tensors after ``zero_grad(set_to_none=True)``), they are
        rewritten in place on the stream (``mad_adamw_set_grads``) instead of
        re-planning, as long as the old and the new addresses are all 16-byte
        aligned (the planned vector width stays legal and optimal).
        """
        quads = [tuple(q) + (None,) * (5 - len(q)) for q in quads]
        key = tuple((p.data_ptr(), m.data_ptr(), v.data_ptr(), p.numel(), p.dtype, g.dtype,
                     sh.data_ptr() if sh is not None else 0) for p, g, m, v, sh in quads)
        grads = tuple(q[1].data_ptr() for q in quads)
        if key == self.key:
            if grads != self.grads:
                if all(a % 16 == 0 for a in grads) and all(a % 16 == 0 for a in self.grads):
                    lib = _lib.load()
                    arr = (ctypes.c_void_p * max(1, len(grads)))(*grads)
                    _lib.check(lib.mad_adamw_set_grads(self.table.data_ptr(), self.n_tiles, arr, len(grads),
                                                       _lib.stream_handle()), "mad_adamw_set_grads")
                    self.grads = grads
                    return
            else:
                return
        lib = _lib.load()
        arr = (_lib.AdamWTensor * max(1, len(quads)))()
        for i, (p, g, m, v, sh) in enumerate(quads):
            arr[i] = _lib.AdamWTensor(p.data_ptr(), g.data_ptr(), m.data_ptr(), v.data_ptr(), p.numel(),
                                      entry_dtype(p, g, sh, "AdamW parameter"), 0,
                                      sh.data_ptr() if sh is not None else None)
        nbytes = ctypes.c_int64()
        _lib.check(lib.mad_adamw_table_bytes(arr, len(quads), ctypes.byref(nbytes)), "mad_adamw_table_bytes")
        self.table = torch.empty(max(1, nbytes.value), dtype=torch.uint8, device=device)
        n_tiles = ctypes.c_int64()
        _lib.check(lib.mad_adamw_plan(arr, len(quads), self.table.data_ptr(), nbytes.value, ctypes.byref(n_tiles),
                                      _lib.stream_handle()), "mad_adamw_plan")
        self.n_tiles = n_tiles.value
        self.numel = sum(q[0].numel() for q in quads)
        self.key = key
        self.grads = grads
        self.replans += 1

    def launch(self, *, lr, beta1, beta2, eps, weight_decay, bias1, bias2, reduce=None) -> None:
        """One launch over the table; ``reduce`` (a ``GradReduce``) sums each gradient over ranks."""
        if self.n_tiles == 0:
            return
        lib = _lib.load()
        if reduce is None:
            _lib.check(lib.mad_adamw_step_multi(self.table.data_ptr(), self.n_tiles, lr, beta1, beta2, eps,
                                                weight_decay, bias1, bias2, _lib.stream_handle()),
                       "mad_adamw_step_multi")
        else:
            _lib.check(lib.mad_adamw_step_multi_reduce(self.table.data_ptr(), self.n_tiles, lr, beta1, beta2, eps,
                                                       weight_decay, bias1, bias2, ctypes.byref(reduce),
                                                       _lib.stream_handle()), "mad_adamw_step_multi_reduce")


class TritonAdamW:
    """AdamW over float32 or bf16 CUDA parameters, one CUDA launch per step.

    The name is the reference's (``triton_muon_adamw.adamw.TritonAdamW``) so
    imports keep working; there is no Triton code behind it.
    """

    def __init__(
        self,
        params: Iterable[nn.Parameter] | list[nn.Parameter],
        lr=1e-3,
        betas: tuple[float, float] = (0.9, 0.999),
        weight_decay=1e-2,
        eps=1e-7,
    ):
        self.model_params = list(params)
        self.beta1 = betas[0]
        self.beta2 = betas[1]
        self.lr = lr
        self.weight_decay = weight_decay
        self.eps = eps
        self.step_num = 0
        self.m = {}
        self.v = {}
        for param in self.model_params:
            self.m[param] = torch.zeros_like(param, dtype=torch.float32)
            self.v[param] = torch.zeros_like(param, dtype=torch.float32)
        self.masters = None  # {param: float32 master} in mixed-precision mode (MuonAdamW(master_weights=True))
        self._table = AdamWTable()
        self._signature = None   # (gradients, by weak reference; parameter and gradient addresses) last planned

    def _active(self):
        quads = []
        masters = self.masters
        for p in self.model_params:
            g = p.grad
            if g is None:
                continue
            if not (p.is_cuda and g.is_cuda and p.dtype in DTYPE_CODES and g.dtype == p.dtype
                    and p.is_contiguous() and g.is_contiguous()):
                _check_tensor(p, "AdamW parameter")          # raises the specific error
                _check_tensor(g, "AdamW gradient", p.dtype)
            if masters is not None:
                quads.append((masters[p], g, self.m[p], self.v[p], p.detach()))
            else:
                quads.append((p.detach(), g, self.m[p], self.v[p]))
        return quads

    @torch.no_grad()
    def step(self):
        """One AdamW update of every parameter that has a gradient (triton_adam.py:132-153).

        The host side is one pass over the parameters: when every parameter
        and gradient is the tensor (and storage) of the previous step, the
        planned table is launched as is; otherwise the tensors are validated
        and the table re-planned or patched.
        """
        self.step_num += 1
        grads = [p.grad for p in self.model_params]
        addrs = tuple(g.data_ptr() if g is not None else 0 for g in grads) + \
            tuple(p.data_ptr() for p in self.model_params)
        sig = self._signature
        if sig is None or addrs != sig[1] or any((r() if r is not None else None) is not g
                                                 for r, g in zip(sig[0], grads)):
            quads = self._active()
            if not quads:
                self._signature = None
                return
            self._table.ensure(quads, quads[0][0].device)
            # Weak references: a gradient dropped by zero_grad(set_to_none=True) is freed, not kept alive here.
            self._signature = ([weakref.ref(g) if g is not None else None for g in grads], addrs)
        elif self._table.n_tiles == 0:
            return
        if getattr(self, "_timer", None) is not None:
            self._timer.mark("adamw")
        self._table.launch(lr=self.lr, beta1=self.beta1, beta2=self.beta2, eps=self.eps,
                           weight_decay=self.weight_decay, bias1=1 - self.beta1 ** self.step_num,
                           bias2=1 - self.beta2 ** self.step_num)

    def zero_grad(self):
        """Reset gradients to zero in place (triton_adam.py:155-161)."""
        for param in self.model_params:
            if param.grad is not None:
                param.grad.zero_()
