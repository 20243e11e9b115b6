"""CPU oracle for the MuonAdamW optimizer step.  TEST INFRASTRUCTURE ONLY.

This module restates, with plain torch CPU arithmetic, the algorithm of the
reference project Mithun-033/Triton-MuonAdamW for its one hot path,
``MuonAdamW.step()``.  It is the *checker*: only ``tests/``, the repository's
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg import it.  The
shipped optimizer (``triton_muon_adamw``) never imports it and has no CPU path.

Reference paths below are relative to the reference project root; ``PKG`` is
its ``MuonAdamW package/`` directory.

Two restatements live here:

* ``OracleMuonAdamW`` follows the reference's *Triton* path
  (``PKG/triton_muon_adamw/optimizer.py:70-175`` routing,
  ``PKG/triton_muon_adamw/adamw/triton_adam.py`` AdamW,
  ``PKG/triton_muon_adamw/muon/triton_muon.py`` Muon) with every bf16 rounding
  point of that path made explicit and every matrix product accumulated in
  float64, so its result does not depend on the host's BLAS blocking.
* ``ReferenceWrapperCPU`` follows the reference's comparison wrapper
  ``PyTorchMuonAdamW`` (``optimizer.py:178-260``), i.e. ``torch.optim.AdamW``
  (fused) and ``torch.optim.Muon`` running on the host cores.  It is the CPU
  baseline that ``bench.py`` times.

AdamW scalars follow the reference Triton kernel on the GPU (float32
arguments, ``1-beta`` formed in float32); the Triton interpreter used for the
AdamW golden forms ``1-beta`` in double instead, a difference of ~1e-8 on the
parameters that the golden test tolerates explicitly.

Parity pin: ``tests/golden/make_golden.py`` imports the reference package in
the development container and records its outputs (``PyTorchMuonAdamW`` on CPU,
``TritonAdamW`` under the Triton interpreter) into ``tests/golden/``;
``tests/test_oracle_golden.py`` checks both restatements against them.  The
reference's Newton-Schulz Triton kernels do not run in the Triton 3.6
interpreter (bf16 is unsupported there), so the Triton-path Muon restatement is
pinned through the wrapper goldens (same rounding points, same coefficients)
rather than through the Triton kernels themselves.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

# Newton-Schulz coefficients torch.optim.Muon uses by default; the reference
# wrapper does not forward its own coefficients (optimizer.py:228-236), so these
# are what PyTorchMuonAdamW computes with.
TORCH_MUON_COEFFS = (3.4445, -4.7750, 2.0315)


def bf16_round(x: torch.Tensor) -> torch.Tensor:
    """Round to bfloat16 (round-to-nearest-even) and return as float32."""
    return x.to(torch.bfloat16).to(torch.float32)


# --------------------------------------------------------------------------
# AdamW branch  (triton_adam.py)
# --------------------------------------------------------------------------

def adamw_update_(p, g, m, v, *, lr, beta1, beta2, eps, weight_decay, bias1, bias2):
    """One elementwise AdamW update in float32, in place on ``p``, ``m``, ``v``.

    Follows ``triton_adam.py:53-63``: moments first, then bias-corrected
    moments, then decoupled decay applied multiplicatively to the old value.
    The kernel there receives its scalars as float32 and forms ``1-beta1``,
    ``1-beta2`` and ``1-lr*wd`` in float32; every operation below is one
    IEEE float32 rounding (division and square root correctly rounded), in
    the kernel's order.

    A bf16 parameter (and gradient) is read as float32, the arithmetic is the
    same, and the new value is rounded to bf16 on the store; the moments stay
    float32 (triton_adam.py:128-130 allocates them as float32).
    """
    f = torch.float32
    one = torch.tensor(1.0, dtype=f)
    b1, b2 = torch.tensor(beta1, dtype=f), torch.tensor(beta2, dtype=f)
    lr_f, wd_f = torch.tensor(lr, dtype=f), torch.tensor(weight_decay, dtype=f)
    g = g.to(f)
    m_t = (b1 * m) + ((one - b1) * g)
    v_t = (b2 * v) + ((one - b2) * (g * g))
    # IEEE float32 division and square root, as the formula is written (and as
    # the Triton interpreter, whose goldens pin this restatement, evaluates it):
    # torch's CPU `tensor / 0-dim tensor` multiplies by the reciprocal instead,
    # and its vectorised float32 sqrt is not correctly rounded -- each one ulp
    # off on a fraction of a percent of elements.  A float64 result rounded once
    # to float32 is the correctly rounded float32 result (double rounding is
    # innocuous for division and square root when 53 >= 2*24 + 2).
    m_c = (m_t.double() / float(torch.tensor(bias1, dtype=f))).to(f)
    v_c = (v_t.double() / float(torch.tensor(bias2, dtype=f))).to(f)
    denom = torch.sqrt(v_c.double()).to(f) + torch.tensor(eps, dtype=f)
    decayed = (one - lr_f * wd_f) * p.to(f)
    p.copy_(decayed - lr_f * (m_c / denom))
    m.copy_(m_t)
    v.copy_(v_t)


def adamw_bias_corrections(beta1: float, beta2: float, step: int) -> tuple[float, float]:
    """Host bias corrections with the branch-global step count (triton_adam.py:137-148)."""
    return 1.0 - beta1 ** step, 1.0 - beta2 ** step


# --------------------------------------------------------------------------
# Muon branch  (triton_muon.py)
# --------------------------------------------------------------------------

def muon_momentum_(grad: torch.Tensor, mom: torch.Tensor, beta: float, nesterov: bool,
                   cpu_torch_alpha: bool = False) -> torch.Tensor:
    """Momentum EMA in place on ``mom`` and the (optionally Nesterov) update.

    ``triton_muon.py:346``: ``momentum.mul_(beta).add_(grad, alpha=1-beta)``
    (buffer updated): one float32 product with ``beta``, then torch's fused
    ``self + alpha*other`` -- a single rounding, emulated here in float64 --
    with ``alpha = 1-beta`` formed in double by Python.
    ``triton_muon.py:348-349``: Nesterov returns ``grad + beta*(mom - grad)``
    as a new tensor (three float32 roundings) and leaves the buffer alone.
    With bf16 buffers every one of these eager ops rounds its result to bf16
    (torch computes in float32 and rounds on the store), which is what happens
    below through the tensors' dtype; the fused add rounds float32 first.

    ``alpha`` is a float32 scalar, as in torch's CUDA ``add`` kernel (it
    computes in float32 for bf16 tensors), which is where the reference runs.
    torch's CPU kernel instead rounds ``alpha`` to the tensor dtype first;
    ``cpu_torch_alpha=True`` reproduces that, to pin the other rounding points
    bit for bit against goldens recorded on CPU.
    """
    f = torch.float32
    fbeta = torch.tensor(beta, dtype=f)
    scaled = (mom.to(f) * fbeta).to(mom.dtype)
    alpha = float(torch.tensor(1.0 - beta, dtype=f))
    if cpu_torch_alpha:
        alpha = float(torch.tensor(alpha, dtype=mom.dtype))
    mom.copy_((scaled.double() + alpha * grad.double()).to(f))
    return muon_nesterov(grad, mom, beta) if nesterov else mom.clone()


def muon_nesterov(grad: torch.Tensor, mom: torch.Tensor, beta: float) -> torch.Tensor:
    """``grad + beta * (momentum - grad)`` (triton_muon.py:348-349), each op rounded to the tensors' dtype.

    ``beta * t`` with a Python float multiplies in float32 by float32(beta)
    (the scalar is never rounded to t's dtype), then rounds to t's dtype.
    """
    f = torch.float32
    return grad + ((mom - grad).to(f) * torch.tensor(beta, dtype=f)).to(mom.dtype)


def to_wide_bf16(u: torch.Tensor) -> tuple[torch.Tensor, bool]:
    """bf16 cast, then transpose tall matrices so rows <= cols (triton_muon.py:351-354)."""
    x = bf16_round(u)
    transposed = x.shape[0] > x.shape[1]
    if transposed:
        x = x.t().contiguous()
    return x, transposed


def frobenius_normalize(x: torch.Tensor, eps: float) -> tuple[torch.Tensor, float]:
    """``X / max(||X||_F, eps)`` with the reference's bf16 rounding points.

    ``triton_muon.py:356`` divides a bf16 tensor by its bf16 norm: the norm is
    accumulated in float32 and rounded to bf16, clamped, and each quotient is
    rounded to bf16.  Returns the normalised matrix and the bf16 norm used.
    """
    sumsq = float((x.double() * x.double()).sum())
    norm = float(bf16_round(torch.tensor(math.sqrt(sumsq), dtype=torch.float32)))
    norm = max(norm, float(bf16_round(torch.tensor(eps, dtype=torch.float32))))
    return bf16_round(x / torch.tensor(norm, dtype=torch.float32)), norm


def ns_iteration(x: torch.Tensor, a: float, b: float, c: float, triton_scalars: bool = False) -> torch.Tensor:
    """One Newton-Schulz iteration (triton_muon.py:313-325).

    Each product is bf16 x bf16 accumulated wide and rounded once to bf16, as
    ``torch.optim.Muon`` (the wrapper's path) does it:

    * ``A  = bf16(X Xᵀ)``                 -- ns_kernel_1, triton_muon.py:35-93
    * ``B  = bf16(b A + c (A Aᵀ))``       -- ns_kernel_2, triton_muon.py:119-188
    * ``X' = bf16(a X + B X)``            -- ns_kernel_3, triton_muon.py:215-278

    ``triton_scalars=True`` models the reference's Triton kernels exactly:
    there ``b_coeff * A`` (:182) and ``a_coeff * X`` (:275) multiply a float
    ``tl.constexpr`` by a bf16 block, and Triton's scalar promotion keeps such
    a product in the tensor's type -- the coefficient is rounded to bf16
    (a = 3.4445 -> 3.4375, b = -4.775 -> -4.78125) and the product is rounded
    to bf16 before the float32 accumulator is added.  ``c_coeff * acc`` meets a
    float32 block and stays float32.  (Pinned against the reference kernels on
    the GPU by tests/test_gpu_reference.py.)
    """
    xd = x.double()
    A = bf16_round((xd @ xd.t()).float())
    Ad = A.double()
    if triton_scalars:
        ah, bh = float(bf16_round(torch.tensor(a))), float(bf16_round(torch.tensor(b)))
        c32 = float(torch.tensor(c, dtype=torch.float32))
        bA = bf16_round((bh * Ad).float()).double()
        B = bf16_round((bA + c32 * (Ad @ Ad.t())).float())
        aX = bf16_round((ah * xd).float()).double()
        return bf16_round((aX + B.double() @ xd).float())
    B = bf16_round((b * Ad + c * (Ad @ Ad.t())).float())
    return bf16_round((a * xd + B.double() @ xd).float())


def orthogonalize(u: torch.Tensor, coeffs, ns_steps: int, eps: float, normalize: str = "reference",
                  triton_scalars: bool = False) -> torch.Tensor:
    """bf16 orthogonalised update in the parameter's orientation (triton_muon.py:351-366).

    ``normalize="reference"`` rounds ``X/||X||`` to bf16 before the first
    iteration, as the reference does.  ``normalize="fold"`` is the
    algebraically identical ordering of the CUDA path: X stays unnormalised
    and s = 1/||X|| scales the first Gram product (by s²) and the first update
    (by s) before their bf16 roundings.  The two orderings differ only by bf16
    rounding placement (about 1-2% relative on small matrices, more on tiny
    ones), which is why tests hold the CUDA path tightly to "fold" and to the
    reference tolerance against "reference".  ``triton_scalars`` (with
    ``normalize="reference"``) applies the reference Triton kernels' bf16
    rounding of ``a``, ``b`` and of their products (see ``ns_iteration``).
    """
    a, b, c = coeffs
    x, transposed = to_wide_bf16(u)
    if normalize == "reference":
        x, _ = frobenius_normalize(x, eps)
        for _ in range(ns_steps):
            x = ns_iteration(x, a, b, c, triton_scalars)
    elif normalize == "fold":
        if triton_scalars:
            raise ValueError("triton_scalars models the reference Triton path, which normalises first")
        sumsq = float((x.double() * x.double()).sum())
        norm = float(bf16_round(torch.tensor(math.sqrt(sumsq), dtype=torch.float32)))
        norm = max(norm, float(bf16_round(torch.tensor(eps, dtype=torch.float32))))
        s = float(torch.tensor(1.0, dtype=torch.float32) / torch.tensor(norm, dtype=torch.float32))
        xd = x.double()
        for it in range(ns_steps):
            s1 = s if it == 0 else 1.0
            A = bf16_round(((s1 * s1) * (xd @ xd.t())).float()).double()
            B = bf16_round((b * A + c * (A @ A)).float()).double()
            xd = bf16_round((s1 * (a * xd + B @ xd)).float()).double()
        x = xd.float()
    else:
        raise ValueError(normalize)
    return x.t() if transposed else x


def scaled_lr(lr: float, shape, adjust_lr_fn: str) -> float:
    """Shape-dependent Muon learning rate (triton_muon.py:424-431).

    ``match_rms_adamw`` raises in the reference (``max`` of an int); it is
    restated as torch's definition ``0.2*lr*sqrt(max(rows, cols))``.
    """
    rows, cols = shape[0], shape[1]
    if adjust_lr_fn == "original":
        return lr * math.sqrt(max(1.0, rows / cols))
    if adjust_lr_fn == "match_rms_adamw":
        return 0.2 * lr * math.sqrt(max(rows, cols))
    if adjust_lr_fn == "spectral_unclamped":
        return lr * math.sqrt(rows / cols)
    raise AssertionError(f"Invalid adjust_lr_fn: {adjust_lr_fn}")


def muon_apply_(p: torch.Tensor, o: torch.Tensor, lr: float, weight_decay: float, slr: float) -> None:
    """Decoupled decay then the scaled update, as two float32 subtractions (triton_muon.py:368-372).

    Each product of a Python float and a tensor is formed in float32 with the
    float32 scalar and rounded to the tensor's dtype, then subtracted; with
    bf16 parameters the update ``out`` is bf16 as well.
    """
    f = torch.float32
    p.sub_((p.to(f) * torch.tensor(lr * weight_decay, dtype=f)).to(p.dtype))
    p.sub_((o.to(p.dtype).to(f) * torch.tensor(slr, dtype=f)).to(p.dtype))


def muon_matrix_step_(p, g, mom, *, lr, beta, nesterov, coeffs, ns_steps, eps, weight_decay,
                      adjust_lr_fn="original", normalize="reference") -> torch.Tensor:
    """Full Muon update of one matrix (triton_muon.py:327-372, lr from :424-431).

    Returns the bf16-valued orthogonalised update so tests can compare it
    directly, not only through ``lr``-scaled parameters.
    """
    u = muon_momentum_(g, mom, beta, nesterov)
    o = orthogonalize(u, coeffs, ns_steps, eps, normalize)
    muon_apply_(p, o, lr, weight_decay, scaled_lr(lr, p.shape, adjust_lr_fn))
    return o


# --------------------------------------------------------------------------
# Routing  (optimizer.py)
# --------------------------------------------------------------------------

def split_params(model=None, explicit=None):
    """Parameter routing of ``MuonAdamW.__init__`` (optimizer.py:107-130).

    Auto mode: 2-D trainable parameters that are neither the input embedding
    nor the output head go to Muon, everything else to AdamW; parameters that
    share storage are taken once.
    """
    if explicit is not None:
        return list(explicit.get("adam", [])), list(explicit.get("muon", []))
    embed = model.get_input_embeddings().weight
    out = model.get_output_embeddings()
    head = out.weight if out is not None else None
    adam, muon, seen = [], [], set()
    for p in model.parameters():
        if not p.requires_grad or p.data_ptr() in seen:
            continue
        seen.add(p.data_ptr())
        if p.ndim == 2 and p is not embed and p is not head:
            muon.append(p)
        else:
            adam.append(p)
    return adam, muon


@dataclass
class OracleMuonAdamW:
    """CPU restatement of ``MuonAdamW`` (optimizer.py:70-175) over float32 or bf16 tensors.

    Holds its own copies of the parameters (``params_adam``/``params_muon``)
    and their gradients; ``step()`` is AdamW then Muon (optimizer.py:156-159).
    """

    params_adam: list
    params_muon: list
    adam: dict = field(default_factory=dict)   # lr, betas, eps, weight_decay
    muon: dict = field(default_factory=dict)   # lr, beta, eps, weight_decay, coeffs, nesterov, ns_steps,
    #                                            adjust_lr_fn, normalize ("reference" | "fold")
    step_num: int = 0

    def __post_init__(self):
        self.exp_avg = [torch.zeros_like(p, dtype=torch.float32) for p in self.params_adam]
        self.exp_avg_sq = [torch.zeros_like(p, dtype=torch.float32) for p in self.params_adam]
        self.momentum = [torch.zeros_like(p) for p in self.params_muon]
        self.last_updates = [None] * len(self.params_muon)

    def step(self, grads_adam, grads_muon):
        self.step_num += 1
        b1, b2 = self.adam["betas"]
        bias1, bias2 = adamw_bias_corrections(b1, b2, self.step_num)
        for p, g, m, v in zip(self.params_adam, grads_adam, self.exp_avg, self.exp_avg_sq):
            if g is None:
                continue
            adamw_update_(p, g, m, v, lr=self.adam["lr"], beta1=b1, beta2=b2, eps=self.adam["eps"],
                          weight_decay=self.adam["weight_decay"], bias1=bias1, bias2=bias2)
        mc = self.muon
        for i, (p, g, mom) in enumerate(zip(self.params_muon, grads_muon, self.momentum)):
            if g is None:
                continue
            self.last_updates[i] = muon_matrix_step_(
                p, g, mom, lr=mc["lr"], beta=mc["beta"], nesterov=mc["nesterov"], coeffs=mc["coeffs"],
                ns_steps=mc["ns_steps"], eps=mc["eps"], weight_decay=mc["weight_decay"],
                adjust_lr_fn=mc.get("adjust_lr_fn", "original"), normalize=mc.get("normalize", "reference"))


class ReferenceWrapperCPU:
    """Host-core restatement of ``PyTorchMuonAdamW`` (optimizer.py:178-260).

    Builds ``torch.optim.AdamW(fused=True)`` and ``torch.optim.Muon`` over the
    given CPU parameters exactly as the wrapper does -- including not
    forwarding the Muon coefficients or eps (optimizer.py:228-236) -- so its
    results are the wrapper's results.
    """

    def __init__(self, adam_params, muon_params, *, adam: dict, muon: dict):
        self.adamw = torch.optim.AdamW(adam_params, lr=adam["lr"], betas=adam["betas"],
                                       weight_decay=adam["weight_decay"], eps=adam["eps"],
                                       fused=True) if adam_params else None
        self.muon = torch.optim.Muon(muon_params, lr=muon["lr"], momentum=muon["beta"],
                                     weight_decay=muon["weight_decay"], nesterov=muon["nesterov"],
                                     ns_steps=muon["ns_steps"],
                                     adjust_lr_fn=muon.get("adjust_lr_fn", "original")) if muon_params else None

    def step(self):
        if self.adamw is not None:
            self.adamw.step()
        if self.muon is not None:
            self.muon.step()


# --------------------------------------------------------------------------
# Synthetic parameter sets  (BASELINE.json configs)
# --------------------------------------------------------------------------

def gpt_c1_shapes(d=512, layers=4, ffn=2048, vocab=8192):
    """Parameter shapes of the CPU-runnable config: a GPT decoder with tied embeddings.

    Returns ``(adam_shapes, muon_shapes)``: the tied embedding, LayerNorm
    weights/biases and linear biases go to AdamW, the block weights to Muon.
    At the defaults this is 16.8M parameters.
    """
    adam = [(vocab, d)]                     # token embedding, tied with the head
    muon = []
    for _ in range(layers):
        adam += [(d,), (d,)]                # ln1
        for _ in range(4):                  # q, k, v, o projections
            muon.append((d, d))
            adam.append((d,))
        adam += [(d,), (d,)]                # ln2
        muon.append((ffn, d))               # fc
        adam.append((ffn,))
        muon.append((d, ffn))               # proj
        adam.append((d,))
    adam += [(d,), (d,)]                    # final ln
    return adam, muon


def llama_shapes(d, layers, n_heads, n_kv_heads, ffn, vocab):
    """Parameter shapes of a Llama-style decoder with an untied head (RMSNorm, SwiGLU).

    Position embedding is rotary (no parameters); embeddings, head and norms go
    to AdamW, the seven block matrices per layer to Muon.
    """
    hd = d // n_heads
    adam = [(vocab, d), (vocab, d)]
    muon = []
    for _ in range(layers):
        adam += [(d,), (d,)]
        muon += [(n_heads * hd, d), (n_kv_heads * hd, d), (n_kv_heads * hd, d), (d, n_heads * hd),
                 (ffn, d), (ffn, d), (d, ffn)]
    adam.append((d,))
    return adam, muon


def llama_8b_shapes():
    return llama_shapes(4096, 32, 32, 8, 14336, 128256)


def llama_1b3_shapes():
    return llama_shapes(2048, 24, 16, 16, 5504, 32000)


def ns_flops(shape, ns_steps: int, symmetric: bool = True) -> float:
    """Newton-Schulz flops for one matrix: per iteration 3m²n+m³ (triangles) or 4m²n+2m³ (dense)."""
    m, n = min(shape), max(shape)
    per = 3 * m * m * n + m ** 3 if symmetric else 4 * m * m * n + 2 * m ** 3
    return float(per) * ns_steps
