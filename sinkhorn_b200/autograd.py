"""Autograd integration: the drop-in for ``sinkhorn.autograd``.

``SinkhornFunction`` / ``sinkhorn_differentiable`` keep the reference's
signatures and gradient semantics (src/sinkhorn/autograd.py:18-253):

* forward: the CUDA solve, without a tape;
* backward: ``0 < grad_iters < max_iters`` -> truncated backprop through
  ``grad_iters`` iterations restarted from the converged (f, g) on raw C,
  masks applied to the final potentials only (autograd.py:83-97,134-178);
  otherwise a full recompute from zeros with masks and a per-iteration
  convergence check (autograd.py:98-113). Both run in libsinkhorn_b200
  (``sk_backward``): O(K(N+M)) saved vectors instead of an O(K N M) tape,
  dC written once.

Known deviation: with masks, the reference's full-recompute backward returns
NaN gradients at every unmasked entry (torch.logsumexp's backward over an
all -inf row gives exp(nan)); this implementation returns the finite
gradient of the same masked iteration (0 at masked entries).

``TransportPlanFunction`` makes ``SinkhornOutput.transport_plan``
differentiable in C, f and g with a fused adjoint kernel.
"""

from __future__ import annotations

import ctypes
from typing import Any

import torch
from torch import Tensor

from . import _tensors as T
from .cuda.forward import sinkhorn_forward_cuda
from .cuda.plan import plan_backward, transport_plan

_TINY = float(torch.tensor(1e-38, dtype=torch.float32))  # fp32 value of the clamp


def sinkhorn_backward_cuda(C: Tensor, a: Tensor | None, b: Tensor | None, epsilon: float,
                           tau_a, tau_b, mask_a, mask_b, max_iters: int, threshold: float,
                           grad_iters: int, f_star: Tensor, g_star: Tensor,
                           grad_f: Tensor | None, grad_g: Tensor | None,
                           need_dlog: bool = False):
    """Gradient of <f, grad_f> + <g, grad_g> w.r.t. C (and log a, log b).

    Returns (dC, dlog_a, dlog_b, K) with K the number of iterations
    differentiated."""
    T.check_cost(C)
    B, N, M = C.shape
    dev = C.device
    a_ = T.vec(a, (B, N), dev, "a")
    b_ = T.vec(b, (B, M), dev, "b")
    ma = T.mask(mask_a, (B, N), dev, "mask_a")
    mb = T.mask(mask_b, (B, M), dev, "mask_b")
    fs = T.vec(f_star, (B, N), dev, "f_star")
    gs = T.vec(g_star, (B, M), dev, "g_star")
    gf = T.vec(grad_f, (B, N), dev, "grad_f")
    gg = T.vec(grad_g, (B, M), dev, "grad_g")
    full = not (0 < grad_iters < max_iters)
    kmax = max_iters if full else grad_iters
    lib = T.lib()
    dC = torch.empty(B, N, M, device=dev, dtype=torch.float32)
    dla = torch.empty(B, N, device=dev, dtype=torch.float32) if need_dlog else None
    dlb = torch.empty(B, M, device=dev, dtype=torch.float32) if need_dlog else None
    K = ctypes.c_int(0)
    with torch.cuda.device(dev):
        ws = T.workspace(lib.sk_backward_workspace_bytes(B, N, M, max(kmax, 1)), dev)
        rc = lib.sk_backward(*T.cost_args(C), T.ptr(a_), T.ptr(b_), T.ptr(ma), T.ptr(mb),
                             float(epsilon), T.tau_arg(tau_a), T.tau_arg(tau_b),
                             int(max_iters), float(threshold), int(grad_iters), T.ptr(fs),
                             T.ptr(gs), T.ptr(gf), T.ptr(gg), dC.data_ptr(), T.ptr(dla),
                             T.ptr(dlb), ws.data_ptr(), ws.numel(), ctypes.byref(K),
                             T.stream_of(dev))
        T.check(rc, "sk_backward")
    return dC, dla, dlb, int(K.value)


def _dlog_to_marginal(dlog: Tensor, x: Tensor) -> Tensor:
    """d/dx log(x.clamp(min=1e-38)) = 1/x where x >= 1e-38 (clamp_min passes
    the gradient there), else 0."""
    xd = x.detach().to(torch.float32)
    keep = xd >= _TINY
    g = torch.where(keep, dlog / torch.where(keep, xd, torch.ones_like(xd)),
                    torch.zeros_like(dlog))
    return g.to(x.dtype)


class SinkhornFunction(torch.autograd.Function):
    """Autograd function for Sinkhorn with the recompute backward on the GPU."""

    @staticmethod
    def forward(ctx: Any, C: Tensor, a: Tensor | None, b: Tensor | None, epsilon: float,
                tau_a: float | None, tau_b: float | None, mask_a: Tensor | None,
                mask_b: Tensor | None, max_iters: int, threshold: float, grad_iters: int,
                backend: str, check_every: int = 10, info: dict | None = None
                ) -> tuple[Tensor, Tensor]:
        with torch.no_grad():
            f, g, n_iters, converged = sinkhorn_forward_cuda(
                C, a, b, epsilon, tau_a, tau_b, mask_a, mask_b, max_iters, threshold,
                check_every=check_every)
        if info is not None:
            info["n_iters"] = n_iters
            info["converged"] = converged
        ctx.save_for_backward(C, a, b, mask_a, mask_b, f, g)
        ctx.epsilon = epsilon
        ctx.tau_a = tau_a
        ctx.tau_b = tau_b
        ctx.max_iters = max_iters
        ctx.threshold = threshold
        ctx.grad_iters = grad_iters
        return f, g

    @staticmethod
    def backward(ctx: Any, grad_f: Tensor, grad_g: Tensor):
        C, a, b, mask_a, mask_b, f_conv, g_conv = ctx.saved_tensors
        need_a = a is not None and ctx.needs_input_grad[1]
        need_b = b is not None and ctx.needs_input_grad[2]
        dC, dla, dlb, _ = sinkhorn_backward_cuda(
            C.detach(), a, b, ctx.epsilon, ctx.tau_a, ctx.tau_b, mask_a, mask_b,
            ctx.max_iters, ctx.threshold, ctx.grad_iters, f_conv, g_conv, grad_f, grad_g,
            need_dlog=need_a or need_b)
        da = _dlog_to_marginal(dla, a) if need_a else None
        db = _dlog_to_marginal(dlb, b) if need_b else None
        dC = dC if ctx.needs_input_grad[0] else None
        return (dC, da, db) + (None,) * 11


def sinkhorn_differentiable(
    C: Tensor,
    a: Tensor | None = None,
    b: Tensor | None = None,
    epsilon: float = 0.1,
    tau_a: float | None = None,
    tau_b: float | None = None,
    mask_a: Tensor | None = None,
    mask_b: Tensor | None = None,
    max_iters: int = 100,
    threshold: float = 1e-6,
    grad_iters: int = 0,
    cg_max_iters: int = 50,
    cg_tol: float = 1e-6,
    backend: str = "cuda",
    check_every: int = 10,
    info: dict | None = None,
) -> tuple[Tensor, Tensor]:
    """Differentiable Sinkhorn (autograd.py:181-253).

    grad_iters: 0 = full recompute, 0 < grad_iters < max_iters = truncated.
    cg_max_iters / cg_tol are accepted and unused, as in the reference.
    ``info`` (optional dict) receives the forward's n_iters / converged.
    """
    del cg_max_iters, cg_tol
    _check_backend(backend)
    T.check_cost(C)
    B, N, M = C.shape
    # Defaults of autograd.py:223-233 are built on the device by the kernels
    # when a / b are None (uniform, or mask / count); they carry no gradient.
    return SinkhornFunction.apply(C, a, b, epsilon, tau_a, tau_b, mask_a, mask_b,
                                  max_iters, threshold, grad_iters, backend, check_every,
                                  info)


class TransportPlanFunction(torch.autograd.Function):
    """P = exp((f + g - C)/eps) with masked entries 0, differentiable in C, f, g.

    The backward recomputes P tile by tile (sk_plan_backward): P is not saved."""

    @staticmethod
    def forward(ctx: Any, C: Tensor, f: Tensor, g: Tensor, epsilon: float,
                mask_a: Tensor | None, mask_b: Tensor | None) -> Tensor:
        P = transport_plan(C.detach(), f.detach(), g.detach(), epsilon, mask_a, mask_b)
        ctx.save_for_backward(C, f, g, mask_a, mask_b)
        ctx.epsilon = epsilon
        return P

    @staticmethod
    def backward(ctx: Any, grad_P: Tensor):
        C, f, g, mask_a, mask_b = ctx.saved_tensors
        dC, df, dg = plan_backward(C.detach(), f.detach(), g.detach(), ctx.epsilon, grad_P,
                                   mask_a, mask_b, need_dC=ctx.needs_input_grad[0],
                                   need_df=ctx.needs_input_grad[1],
                                   need_dg=ctx.needs_input_grad[2])
        return dC, df, dg, None, None, None


_BACKENDS = ("cuda", "triton")


def _check_backend(backend: str) -> None:
    """This package has exactly one backend. "triton" is accepted as an alias
    so code written for the reference's default keeps working."""
    if backend not in _BACKENDS:
        raise ValueError(
            f"backend {backend!r} is not provided by sinkhorn_b200 (only 'cuda'; "
            "'triton' is an alias of it)")
