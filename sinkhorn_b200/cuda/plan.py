"""Transport plan, cost, JVP and the plan adjoint on the GPU (C ABI wrappers).

``transport_plan`` / ``cost`` implement SinkhornOutput.transport_plan / .cost
(src/sinkhorn/sinkhorn.py:27-67); ``jvp_cuda`` keeps the signature of
``jvp_triton`` (src/sinkhorn/triton/jvp_kernel.py:113-182); ``jvp_cuda_free``
is its P-free form (the plan is recomputed from C, f, g tile by tile).
"""

from __future__ import annotations

import torch
from torch import Tensor

from .. import _tensors as T


def transport_plan(C: Tensor, f: Tensor, g: Tensor, epsilon: float,
                   mask_a: Tensor | None = None, mask_b: Tensor | None = None) -> Tensor:
    """P = exp((f + g - C)/eps), 0 at masked rows/columns; dense (B,N,M)."""
    T.check_cost(C)
    B, N, M = C.shape
    dev = C.device
    f_ = T.vec(f, (B, N), dev, "f")
    g_ = T.vec(g, (B, M), dev, "g")
    ma = T.mask(mask_a, (B, N), dev, "mask_a")
    mb = T.mask(mask_b, (B, M), dev, "mask_b")
    P = torch.empty(B, N, M, device=dev, dtype=torch.float32)
    with torch.cuda.device(dev):
        rc = T.lib().sk_transport_plan(*T.cost_args(C), f_.data_ptr(), g_.data_ptr(),
                                       float(epsilon), T.ptr(ma), T.ptr(mb), P.data_ptr(),
                                       T.stream_of(dev))
        T.check(rc, "sk_transport_plan")
    return P


def cost(C: Tensor, f: Tensor, g: Tensor, epsilon: float) -> Tensor:
    """sum_ij P_ij C_ij per batch item with the unmasked plan, P never stored."""
    T.check_cost(C)
    B, N, M = C.shape
    dev = C.device
    f_ = T.vec(f, (B, N), dev, "f")
    g_ = T.vec(g, (B, M), dev, "g")
    out = torch.empty(B, device=dev, dtype=torch.float32)
    lib = T.lib()
    with torch.cuda.device(dev):
        ws = T.workspace(lib.sk_cost_workspace_bytes(B, N, M), dev)
        rc = lib.sk_cost(*T.cost_args(C), f_.data_ptr(), g_.data_ptr(), float(epsilon),
                         out.data_ptr(), ws.data_ptr(), ws.numel(), T.stream_of(dev))
        T.check(rc, "sk_cost")
    return out


def marginal_error(C: Tensor, f: Tensor, g: Tensor, a: Tensor, b: Tensor, epsilon: float,
                   mask_a: Tensor | None = None, mask_b: Tensor | None = None) -> Tensor:
    """Max over the batch of the marginal violations of the masked plan
    (compute_marginal_error, pytorch/balanced.py:183-213): a 0-d tensor on
    C's device, from one pass over C (P never stored)."""
    T.check_cost(C)
    B, N, M = C.shape
    dev = C.device
    f_ = T.vec(f, (B, N), dev, "f")
    g_ = T.vec(g, (B, M), dev, "g")
    a_ = T.vec(a, (B, N), dev, "a")
    b_ = T.vec(b, (B, M), dev, "b")
    ma = T.mask(mask_a, (B, N), dev, "mask_a")
    mb = T.mask(mask_b, (B, M), dev, "mask_b")
    out = torch.empty((), device=dev, dtype=torch.float32)
    lib = T.lib()
    with torch.cuda.device(dev):
        ws = T.workspace(lib.sk_marginal_error_workspace_bytes(B, N, M), dev)
        rc = lib.sk_marginal_error(*T.cost_args(C), f_.data_ptr(), g_.data_ptr(),
                                   a_.data_ptr(), b_.data_ptr(), float(epsilon), T.ptr(ma),
                                   T.ptr(mb), out.data_ptr(), ws.data_ptr(), ws.numel(),
                                   T.stream_of(dev))
        T.check(rc, "sk_marginal_error")
    return out


def plan_backward(C: Tensor, f: Tensor, g: Tensor, epsilon: float, grad_P: Tensor,
                  mask_a: Tensor | None = None, mask_b: Tensor | None = None,
                  need_dC: bool = True, need_df: bool = True, need_dg: bool = True):
    """Adjoint of the plan: W = grad_P * P / eps; returns (-W, sum_j W, sum_i W)
    (masked entries pass nothing); unneeded outputs are None."""
    T.check_cost(C)
    B, N, M = C.shape
    dev = C.device
    f_ = T.vec(f, (B, N), dev, "f")
    g_ = T.vec(g, (B, M), dev, "g")
    gP = grad_P.detach().to(torch.float32).contiguous()
    if tuple(gP.shape) != (B, N, M):
        raise ValueError("grad_P must have the shape of C")
    ma = T.mask(mask_a, (B, N), dev, "mask_a")
    mb = T.mask(mask_b, (B, M), dev, "mask_b")
    dC = torch.empty(B, N, M, device=dev, dtype=torch.float32) if need_dC else None
    df = torch.empty(B, N, device=dev, dtype=torch.float32) if need_df else None
    dg = torch.empty(B, M, device=dev, dtype=torch.float32) if need_dg else None
    lib = T.lib()
    with torch.cuda.device(dev):
        ws = T.workspace(lib.sk_jvp_workspace_bytes(B, N, M), dev)
        rc = lib.sk_plan_backward(*T.cost_args(C), f_.data_ptr(), g_.data_ptr(),
                                  float(epsilon), T.ptr(ma), T.ptr(mb), gP.data_ptr(),
                                  T.ptr(dC), T.ptr(df), T.ptr(dg), ws.data_ptr(), ws.numel(),
                                  T.stream_of(dev))
        T.check(rc, "sk_plan_backward")
    return dC, df, dg


def jvp_cuda(v_f: Tensor, v_g: Tensor, P: Tensor, rho_a: float = 0.0, rho_b: float = 0.0,
             block_size: int = 128) -> tuple[Tensor, Tensor]:
    """jvp_triton on a materialised plan P (B,N,M):
    out_f = rho_a v_f + (1-rho_a) (P v_g)/(P 1), out_g likewise with P^T."""
    del block_size
    T.check_cost(P, "P")
    B, N, M = P.shape
    dev = P.device
    P_ = P.contiguous()
    vf = T.vec(v_f, (B, N), dev, "v_f")
    vg = T.vec(v_g, (B, M), dev, "v_g")
    of = torch.empty(B, N, device=dev, dtype=torch.float32)
    og = torch.empty(B, M, device=dev, dtype=torch.float32)
    lib = T.lib()
    with torch.cuda.device(dev):
        ws = T.workspace(lib.sk_jvp_workspace_bytes(B, N, M), dev)
        rc = lib.sk_jvp_plan(P_.data_ptr(), B, N, M, vf.data_ptr(), vg.data_ptr(),
                             float(rho_a), float(rho_b), of.data_ptr(), og.data_ptr(),
                             ws.data_ptr(), ws.numel(), T.stream_of(dev))
        T.check(rc, "sk_jvp_plan")
    return of, og


def jvp_cuda_free(v_f: Tensor, v_g: Tensor, C: Tensor, f: Tensor, g: Tensor,
                  epsilon: float, rho_a: float = 0.0, rho_b: float = 0.0
                  ) -> tuple[Tensor, Tensor]:
    """jvp_cuda with P = exp((f+g-C)/eps) recomputed on the fly (never stored)."""
    T.check_cost(C)
    B, N, M = C.shape
    dev = C.device
    f_ = T.vec(f, (B, N), dev, "f")
    g_ = T.vec(g, (B, M), dev, "g")
    vf = T.vec(v_f, (B, N), dev, "v_f")
    vg = T.vec(v_g, (B, M), dev, "v_g")
    of = torch.empty(B, N, device=dev, dtype=torch.float32)
    og = torch.empty(B, M, device=dev, dtype=torch.float32)
    lib = T.lib()
    with torch.cuda.device(dev):
        ws = T.workspace(lib.sk_jvp_workspace_bytes(B, N, M), dev)
        rc = lib.sk_jvp(*T.cost_args(C), f_.data_ptr(), g_.data_ptr(), float(epsilon),
                        vf.data_ptr(), vg.data_ptr(), float(rho_a), float(rho_b),
                        of.data_ptr(), og.data_ptr(), ws.data_ptr(), ws.numel(),
                        T.stream_of(dev))
        T.check(rc, "sk_jvp")
    return of, og
