"""Implicit differentiation of the Sinkhorn fixed point on the GPU.

Mirrors the reference module ``sinkhorn.pytorch.implicit_diff``
(src/sinkhorn/pytorch/implicit_diff.py) name for name, with the same
arguments, defaults and results. The work runs in libsinkhorn_b200.so
(sk_implicit.cu):

* ``implicit_gradient`` never materialises the plan: the CG matvec is one band
  pass over C per iteration giving P (p_g / c) and P^T (p_f / r) together, the
  CG update and the batch-wide stopping test run on the device (no host
  synchronisation inside the loop), and dC = -(1/eps) P (lambda_f + lambda_g)
  is one more pass over C.
* ``schur_complement_matvec``, ``cg_solve``, ``jvp_sinkhorn``,
  ``vjp_sinkhorn`` and ``conjugate_gradient_solve`` take a dense plan P, as in
  the reference, and run the same kernels reading P instead of recomputing it.

All tensors are float32 on a CUDA device; there is no CPU path.
"""

from __future__ import annotations

import ctypes

import torch
from torch import Tensor

from . import _tensors as T
from .cuda.plan import transport_plan

MODE_SCHUR, MODE_VJP, MODE_JVP = 0, 1, 2


def _rho(epsilon: float, tau: float | None) -> float:
    """implicit_diff.py:228-233: 0 when balanced (tau None or inf)."""
    if tau is None or tau == float("inf"):
        return 0.0
    return epsilon / (epsilon + tau)


def _dense_plan(P: Tensor) -> Tensor:
    T.check_cost(P, "P")
    return P.detach().to(torch.float32).contiguous()


def compute_transport_plan(C: Tensor, f: Tensor, g: Tensor, epsilon: float,
                           mask_a: Tensor | None = None,
                           mask_b: Tensor | None = None) -> Tensor:
    """P_ij = exp((f_i + g_j - C_ij)/eps), 0 at masked rows / columns
    (implicit_diff.py:12-42)."""
    return transport_plan(C, f, g, epsilon, mask_a, mask_b)


def _matvec(v_f: Tensor, v_g: Tensor, P: Tensor, rho_a: float, rho_b: float, reg: float,
            mode: int, mask_a: Tensor | None = None,
            mask_b: Tensor | None = None) -> tuple[Tensor, Tensor]:
    P_ = _dense_plan(P)
    B, N, M = P_.shape
    dev = P_.device
    vf = T.vec(v_f, (B, N), dev, "v_f")
    vg = T.vec(v_g, (B, M), dev, "v_g")
    ma = T.mask(mask_a, (B, N), dev, "mask_a")
    mb = T.mask(mask_b, (B, M), dev, "mask_b")
    of = torch.empty(B, N, device=dev, dtype=torch.float32)
    og = torch.empty(B, M, device=dev, dtype=torch.float32)
    lib = T.lib()
    with torch.cuda.device(dev):
        ws = T.workspace(lib.sk_implicit_workspace_bytes(B, N, M), dev)
        rc = lib.sk_implicit_matvec(None, B, N, M, 0, 0, 0, None, None, 1.0, T.ptr(ma),
                                    T.ptr(mb), P_.data_ptr(), vf.data_ptr(), vg.data_ptr(),
                                    float(rho_a), float(rho_b), float(reg), mode,
                                    of.data_ptr(), og.data_ptr(), ws.data_ptr(), ws.numel(),
                                    T.stream_of(dev))
        T.check(rc, "sk_implicit_matvec")
    return of, og


def schur_complement_matvec(v_f: Tensor, v_g: Tensor, P: Tensor, rho_a: float, rho_b: float,
                            reg: float = 1e-5) -> tuple[Tensor, Tensor]:
    """(I - J_T^T + reg I) v on a dense plan (implicit_diff.py:45-104)."""
    return _matvec(v_f, v_g, P, rho_a, rho_b, reg, MODE_SCHUR)


def jvp_sinkhorn(v_f: Tensor, v_g: Tensor, P: Tensor, epsilon: float, rho_a: float = 0.0,
                 rho_b: float = 0.0, mask_a: Tensor | None = None,
                 mask_b: Tensor | None = None) -> tuple[Tensor, Tensor]:
    """J_T v, 0 at masked entries (implicit_diff.py:253-278)."""
    del epsilon
    return _matvec(v_f, v_g, P, rho_a, rho_b, 0.0, MODE_JVP, mask_a, mask_b)


def vjp_sinkhorn(v_f: Tensor, v_g: Tensor, P: Tensor, epsilon: float, rho_a: float = 0.0,
                 rho_b: float = 0.0, mask_a: Tensor | None = None,
                 mask_b: Tensor | None = None) -> tuple[Tensor, Tensor]:
    """J_T^T v, 0 at masked entries (implicit_diff.py:281-309)."""
    del epsilon
    return _matvec(v_f, v_g, P, rho_a, rho_b, 0.0, MODE_VJP, mask_a, mask_b)


def _cg(C: Tensor | None, f: Tensor | None, g: Tensor | None, epsilon: float,
        mask_a: Tensor | None, mask_b: Tensor | None, P: Tensor | None, rhs_f: Tensor,
        rhs_g: Tensor, rho_a: float, rho_b: float, max_iters: int, tol: float, reg: float,
        want_grads: bool):
    if P is not None:
        P_ = _dense_plan(P)
        B, N, M = P_.shape
        dev = P_.device
        cargs = (None, B, N, M, 0, 0, 0)
        fp = gp = None
        ma = mb = None
    else:
        T.check_cost(C)
        B, N, M = C.shape
        dev = C.device
        P_ = None
        cargs = T.cost_args(C)
        f_ = T.vec(f, (B, N), dev, "f")
        g_ = T.vec(g, (B, M), dev, "g")
        fp, gp = f_.data_ptr(), g_.data_ptr()
        ma = T.mask(mask_a, (B, N), dev, "mask_a")
        mb = T.mask(mask_b, (B, M), dev, "mask_b")
    rf = T.vec(rhs_f, (B, N), dev, "rhs_f")
    rg = T.vec(rhs_g, (B, M), dev, "rhs_g")
    lf = torch.empty(B, N, device=dev, dtype=torch.float32)
    lg = torch.empty(B, M, device=dev, dtype=torch.float32)
    ga = torch.empty(B, N, device=dev, dtype=torch.float32) if want_grads else None
    gb = torch.empty(B, M, device=dev, dtype=torch.float32) if want_grads else None
    n = ctypes.c_int(0)
    lib = T.lib()
    with torch.cuda.device(dev):
        ws = T.workspace(lib.sk_implicit_workspace_bytes(B, N, M), dev)
        rc = lib.sk_implicit_cg(*cargs, fp, gp, float(epsilon), T.ptr(ma), T.ptr(mb),
                                T.ptr(P_), rf.data_ptr(), rg.data_ptr(), float(rho_a),
                                float(rho_b), int(max_iters), float(tol), float(reg),
                                lf.data_ptr(), lg.data_ptr(), T.ptr(ga), T.ptr(gb),
                                ws.data_ptr(), ws.numel(), ctypes.byref(n), T.stream_of(dev))
        T.check(rc, "sk_implicit_cg")
    return lf, lg, ga, gb, n.value


def cg_solve(rhs_f: Tensor, rhs_g: Tensor, P: Tensor, rho_a: float = 0.0, rho_b: float = 0.0,
             max_iters: int = 50, tol: float = 1e-5,
             reg: float = 1e-5) -> tuple[Tensor, Tensor, int]:
    """Solve (I - J_T^T + reg I) lambda = rhs by batched CG on a dense plan
    (implicit_diff.py:107-193). Returns (lambda_f, lambda_g, n_iters)."""
    lf, lg, _, _, n = _cg(None, None, None, 1.0, None, None, P, rhs_f, rhs_g, rho_a, rho_b,
                          max_iters, tol, reg, False)
    return lf, lg, n


def conjugate_gradient_solve(rhs_f: Tensor, rhs_g: Tensor, P: Tensor, epsilon: float,
                             rho_a: float = 0.0, rho_b: float = 0.0,
                             mask_a: Tensor | None = None, mask_b: Tensor | None = None,
                             max_iters: int = 50, tol: float = 1e-5,
                             regularization: float = 1e-5) -> tuple[Tensor, Tensor, int]:
    """Legacy wrapper of cg_solve (implicit_diff.py:312-326); the masks are
    unused there too."""
    del epsilon, mask_a, mask_b
    return cg_solve(rhs_f, rhs_g, P, rho_a, rho_b, max_iters, tol, regularization)


def implicit_gradient(C: Tensor, f: Tensor, g: Tensor, grad_f: Tensor, grad_g: Tensor,
                      epsilon: float, tau_a: float | None = None, tau_b: float | None = None,
                      mask_a: Tensor | None = None, mask_b: Tensor | None = None,
                      cg_max_iters: int = 50,
                      cg_tol: float = 1e-5) -> tuple[Tensor, Tensor, Tensor]:
    """(dL/dC, dL/da, dL/db) by the implicit function theorem
    (implicit_diff.py:196-249), the plan never stored: CG with reg = 1e-5 on
    (I - J_T^T + reg I) lambda = (grad_f, grad_g), then
    dC = -(1/eps) P (lambda_f[:, None] + lambda_g[None, :]), da = eps lambda_f,
    db = eps lambda_g."""
    rho_a, rho_b = _rho(epsilon, tau_a), _rho(epsilon, tau_b)
    lf, lg, ga, gb, _ = _cg(C, f, g, epsilon, mask_a, mask_b, None, grad_f, grad_g, rho_a,
                            rho_b, cg_max_iters, cg_tol, 1e-5, True)
    B, N, M = C.shape
    dev = C.device
    f_ = T.vec(f, (B, N), dev, "f")
    g_ = T.vec(g, (B, M), dev, "g")
    ma = T.mask(mask_a, (B, N), dev, "mask_a")
    mb = T.mask(mask_b, (B, M), dev, "mask_b")
    dC = torch.empty(B, N, M, device=dev, dtype=torch.float32)
    with torch.cuda.device(dev):
        rc = T.lib().sk_implicit_dC(*T.cost_args(C), f_.data_ptr(), g_.data_ptr(),
                                    float(epsilon), T.ptr(ma), T.ptr(mb), lf.data_ptr(),
                                    lg.data_ptr(), dC.data_ptr(), T.stream_of(dev))
        T.check(rc, "sk_implicit_dC")
    return dC, ga, gb


__all__ = ["compute_transport_plan", "schur_complement_matvec", "cg_solve",
           "implicit_gradient", "jvp_sinkhorn", "vjp_sinkhorn", "conjugate_gradient_solve"]
