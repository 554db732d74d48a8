"""High-level API: the drop-in for ``sinkhorn.sinkhorn`` (src/sinkhorn/sinkhorn.py).

``sinkhorn(...)`` and ``SinkhornOutput`` keep the reference's signatures and
results; the work runs in libsinkhorn_b200 on CUDA tensors. Differences from
the reference, all deliberate:

* ``backend`` accepts "cuda" (default) and "triton" (alias); CPU tensors raise
  instead of falling back to PyTorch (sinkhorn.py:182-187).
* ``check_every`` (default 10, the Triton cadence) sets the convergence-check
  period; 1 reproduces the PyTorch path's iteration counts.
* On the gradient path the reference forwards ``cg_max_iters`` into the
  ``grad_iters`` slot of ``sinkhorn_differentiable`` (a positional shift,
  sinkhorn.py:193-207 vs autograd.py:181-196); that mapping is kept so
  gradients match, but the returned ``n_iters`` / ``converged`` are the
  forward's real values instead of ``max_iters`` / True.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import Tensor

from . import _tensors as T
from .autograd import TransportPlanFunction, _check_backend, sinkhorn_differentiable
from .cuda import plan as _plan
from .cuda.forward import sinkhorn_forward_cuda


def _needs_grad(*xs) -> bool:
    return torch.is_grad_enabled() and any(
        isinstance(x, Tensor) and x.requires_grad for x in xs)


@dataclass
class SinkhornOutput:
    """Output container for Sinkhorn computation (sinkhorn.py:11-102)."""

    f: Tensor
    """Row dual potential (B, N)"""

    g: Tensor
    """Column dual potential (B, M)"""

    n_iters: int
    """Number of iterations performed"""

    converged: bool
    """Whether the algorithm converged"""

    def transport_plan(self, C: Tensor, epsilon: float, mask_a: Tensor | None = None,
                       mask_b: Tensor | None = None) -> Tensor:
        """P_ij = exp((f_i + g_j - C_ij) / eps), 0 at masked rows / columns."""
        if _needs_grad(C, self.f, self.g):
            return TransportPlanFunction.apply(C, self.f, self.g, epsilon, mask_a, mask_b)
        return _plan.transport_plan(C, self.f, self.g, epsilon, mask_a, mask_b)

    def cost(self, C: Tensor, epsilon: float) -> Tensor:
        """<P, C> per batch item (B,), masks ignored as in the reference."""
        if _needs_grad(C, self.f, self.g):
            P = self.transport_plan(C, epsilon)
            return (P * C).sum(dim=(-2, -1))
        return _plan.cost(C, self.f, self.g, epsilon).to(C.dtype)

    def sinkhorn_divergence(self, C: Tensor, epsilon: float, a: Tensor | None = None,
                            b: Tensor | None = None) -> Tensor:
        """The reference's dual estimate <f, a> + <g, b> (sinkhorn.py:69-102)."""
        del C, epsilon
        if a is None:
            a = torch.ones(self.f.shape, device=self.f.device, dtype=self.f.dtype)
            a = a / a.sum(dim=-1, keepdim=True)
        if b is None:
            b = torch.ones(self.g.shape, device=self.g.device, dtype=self.g.dtype)
            b = b / b.sum(dim=-1, keepdim=True)
        return (self.f * a).sum(dim=-1) + (self.g * b).sum(dim=-1)


def sinkhorn(
    C: Tensor,
    a: Tensor | None = None,
    b: Tensor | None = None,
    epsilon: float = 0.1,
    tau_a: float | None = None,
    tau_b: float | None = None,
    mask_a: Tensor | None = None,
    mask_b: Tensor | None = None,
    backend: str = "cuda",
    max_iters: int = 100,
    threshold: float = 1e-6,
    implicit_diff: bool = True,
    cg_max_iters: int = 50,
    cg_tol: float = 1e-6,
    check_every: int = 10,
    f_init: Tensor | None = None,
    g_init: Tensor | None = None,
) -> SinkhornOutput:
    """Unified entry point for Sinkhorn optimal transport (sinkhorn.py:105-226).

    Computes dual potentials (f, g) of entropic OT, balanced (tau None) or
    KL-unbalanced (rho = eps/(eps+tau)), with optional row / column masks.
    ``f_init`` / ``g_init`` warm-start the forward solve (not the
    differentiable path, whose backward recomputes from zero potentials).
    """
    if C.dim() != 3:
        raise ValueError(f"C must be 3D (B, N, M), got {C.dim()}D")
    _check_backend(backend)
    T.check_cost(C, allow_bf16=True)
    if torch.is_grad_enabled() and implicit_diff and C.requires_grad:
        if C.dtype == torch.bfloat16:
            raise TypeError("a bfloat16 C is supported by the forward solve only "
                            "(the differentiable path computes in float32)")
        if f_init is not None or g_init is not None:
            raise ValueError("f_init / g_init warm-start the forward only; call sinkhorn "
                             "under torch.no_grad() or without requires_grad on C")
        info: dict = {}
        f, g = sinkhorn_differentiable(C, a, b, epsilon, tau_a, tau_b, mask_a, mask_b,
                                       max_iters, threshold, grad_iters=cg_max_iters,
                                       backend=backend, check_every=check_every,
                                       info=info)
        return SinkhornOutput(f=f, g=g, n_iters=info["n_iters"],
                              converged=info["converged"])
    f, g, n_iters, converged = sinkhorn_forward_cuda(
        C, a, b, epsilon, tau_a, tau_b, mask_a, mask_b, max_iters, threshold,
        check_every=check_every, f_init=f_init, g_init=g_init)
    return SinkhornOutput(f=f, g=g, n_iters=n_iters, converged=converged)
