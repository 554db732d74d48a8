"""CUDA kernels behind the reference's backend API (replaces ``sinkhorn.triton``)."""

from .forward import sinkhorn_forward_cuda
from .lse_kernel import lse_col, lse_row
from .plan import cost, jvp_cuda, jvp_cuda_free, plan_backward, transport_plan

__all__ = ["sinkhorn_forward_cuda", "lse_row", "lse_col", "transport_plan", "cost",
           "jvp_cuda", "jvp_cuda_free", "plan_backward"]
