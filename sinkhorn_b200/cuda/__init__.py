"""CUDA kernels behind the reference's backend API (replaces ``sinkhorn.triton``)."""

from .forward import sinkhorn_forward_cuda

__all__ = ["sinkhorn_forward_cuda"]
