"""Argument checks and pointer plumbing between torch tensors and the C ABI."""

from __future__ import annotations

import math

import torch
from torch import Tensor

from . import _lib


def ptr(t: Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def tau_arg(tau: float | None) -> float:
    """The C ABI encodes the reference's tau=None (balanced) as +inf."""
    return math.inf if tau is None else float(tau)


def check_cost(C: Tensor, name: str = "C", allow_bf16: bool = False) -> None:
    """allow_bf16: the forward solve also takes a bfloat16 cost (sk_forward_bf16)."""
    if not isinstance(C, Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if C.dim() != 3:
        raise ValueError(f"{name} must be 3D (B, N, M), got {C.dim()}D")
    if not C.is_cuda:
        raise RuntimeError(
            f"{name} is on {C.device}: the cuda backend runs on CUDA tensors only "
            "(there is no CPU fallback)")
    if C.dtype != torch.float32 and not (allow_bf16 and C.dtype == torch.bfloat16):
        raise TypeError(f"{name} must be float32 (the cuda backend computes in fp32"
                        f"{'; the forward solve also takes bfloat16' if allow_bf16 else ''}), "
                        f"got {C.dtype}")
    if any(s < 0 for s in C.stride()):
        raise ValueError(f"{name} has a negative stride")


def vec(x: Tensor | None, shape: tuple, device, name: str) -> Tensor | None:
    """A dense float32 (B,n) vector on `device` (None passes through)."""
    if x is None:
        return None
    if not isinstance(x, Tensor):
        raise TypeError(f"{name} must be a torch.Tensor or None")
    if tuple(x.shape) != tuple(shape):
        raise ValueError(f"{name} must have shape {tuple(shape)}, got {tuple(x.shape)}")
    if x.device != device:
        raise ValueError(f"{name} is on {x.device}, C is on {device}")
    return x.detach().to(torch.float32).contiguous()


def mask(x: Tensor | None, shape: tuple, device, name: str) -> Tensor | None:
    """A dense uint8 (B,n) mask (nonzero = valid)."""
    if x is None:
        return None
    if not isinstance(x, Tensor):
        raise TypeError(f"{name} must be a torch.Tensor or None")
    if tuple(x.shape) != tuple(shape):
        raise ValueError(f"{name} must have shape {tuple(shape)}, got {tuple(x.shape)}")
    if x.device != device:
        raise ValueError(f"{name} is on {x.device}, C is on {device}")
    if x.dtype == torch.bool:
        return x.contiguous().view(torch.uint8)
    return (x != 0).contiguous().view(torch.uint8)


def workspace(nbytes: int, device) -> Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


def cost_args(C: Tensor) -> tuple:
    B, N, M = C.shape
    sb, sn, sm = C.stride()
    return (C.data_ptr(), B, N, M, sb, sn, sm)


lib = _lib.load
check = _lib.check
