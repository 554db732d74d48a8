"""CUDA forward Sinkhorn: the drop-in for ``sinkhorn.triton.forward``.

``sinkhorn_forward_cuda`` has the signature, argument meaning and return tuple
of ``sinkhorn_forward_triton`` (src/sinkhorn/triton/forward.py:85-186) and runs
the whole solve in libsinkhorn_b200 (``sk_forward``): fused row/column sweeps,
masks applied inside the kernels (no masked copy of C), the convergence check
decided on the device every ``check_every`` iterations (10, as in the Triton
path; 1 reproduces the PyTorch path).
"""

from __future__ import annotations

import ctypes

import torch
from torch import Tensor

from .. import _tensors as T


def sinkhorn_forward_cuda(
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
    block_size: int = 128,
    check_every: int = 10,
    f_init: Tensor | None = None,
    g_init: Tensor | None = None,
) -> tuple[Tensor, Tensor, int, bool]:
    """Sinkhorn forward pass on the GPU.

    Args follow sinkhorn_forward_triton; ``block_size`` is accepted for
    signature compatibility and ignored (tiling is chosen per shape).
    ``check_every`` is the convergence-check period. A bfloat16 ``C`` is
    solved by the fp32 arithmetic on its exactly widened values, reading half
    the bytes (sk_forward_bf16); f and g are float32. ``f_init`` / ``g_init``
    (optional, either may be given; the other starts at 0) warm-start the
    solve (sk_forward_warm); n_iters then counts this call's iterations.

    Returns:
        f (B,N), g (B,M), n_iters, converged
    """
    del block_size
    T.check_cost(C, allow_bf16=True)
    bf16 = C.dtype == torch.bfloat16
    B, N, M = C.shape
    dev = C.device
    a_ = T.vec(a, (B, N), dev, "a")
    b_ = T.vec(b, (B, M), dev, "b")
    ma = T.mask(mask_a, (B, N), dev, "mask_a")
    mb = T.mask(mask_b, (B, M), dev, "mask_b")
    if not float(epsilon) > 0:
        raise ValueError(f"epsilon must be positive, got {epsilon}")
    if int(max_iters) < 0:
        raise ValueError("max_iters must be >= 0")
    if int(check_every) < 1:
        raise ValueError("check_every must be >= 1")
    lib = T.lib()
    with torch.cuda.device(dev):
        warm = f_init is not None or g_init is not None
        if warm and bf16:
            raise ValueError("f_init / g_init are not supported with a bfloat16 C")
        if warm:
            f = torch.zeros(B, N, device=dev, dtype=torch.float32)
            g = torch.zeros(B, M, device=dev, dtype=torch.float32)
            if f_init is not None:
                f.copy_(T.vec(f_init, (B, N), dev, "f_init"))
            if g_init is not None:
                g.copy_(T.vec(g_init, (B, M), dev, "g_init"))
        else:
            f = torch.empty(B, N, device=dev, dtype=torch.float32)
            g = torch.empty(B, M, device=dev, dtype=torch.float32)
        ws = T.workspace(lib.sk_forward_workspace_bytes(B, N, M), dev)
        n_iters = ctypes.c_int(0)
        conv = ctypes.c_int(0)
        entry = lib.sk_forward_bf16 if bf16 else (lib.sk_forward_warm if warm else
                                                   lib.sk_forward)
        rc = entry(*T.cost_args(C), T.ptr(a_), T.ptr(b_), T.ptr(ma), T.ptr(mb),
                   float(epsilon), T.tau_arg(tau_a), T.tau_arg(tau_b),
                   int(max_iters), float(threshold), int(check_every),
                   f.data_ptr(), g.data_ptr(), ws.data_ptr(), ws.numel(),
                   ctypes.byref(n_iters), ctypes.byref(conv),
                   T.stream_of(dev))
        T.check(rc, "sk_forward_bf16" if bf16 else ("sk_forward_warm" if warm else "sk_forward"))
    return f, g, int(n_iters.value), bool(conv.value)
