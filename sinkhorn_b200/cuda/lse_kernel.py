"""Streaming softmins: the drop-in for ``sinkhorn.triton.lse_kernel``.

``lse_row`` / ``lse_col`` keep the signatures and results of the reference
wrappers (src/sinkhorn/triton/lse_kernel.py:210-293):
``-eps * logsumexp`` along a row / column, 0 where no term is finite.
"""

from __future__ import annotations

import torch
from torch import Tensor

from .. import _tensors as T


def lse_row(C: Tensor, g: Tensor, epsilon: float, block_size: int = 128) -> Tensor:
    """out[b,n] = -eps * logsumexp_m((g[b,m] - C[b,n,m]) / eps)."""
    del block_size
    T.check_cost(C)
    B, N, M = C.shape
    g_ = T.vec(g, (B, M), C.device, "g")
    out = torch.empty(B, N, device=C.device, dtype=torch.float32)
    with torch.cuda.device(C.device):
        rc = T.lib().sk_lse_row(*T.cost_args(C), g_.data_ptr(), float(epsilon),
                                out.data_ptr(), T.stream_of(C.device))
        T.check(rc, "sk_lse_row")
    return out


def lse_col(C: Tensor, f: Tensor, epsilon: float, block_size: int = 128) -> Tensor:
    """out[b,m] = -eps * logsumexp_n((f[b,n] - C[b,n,m]) / eps)."""
    del block_size
    T.check_cost(C)
    B, N, M = C.shape
    f_ = T.vec(f, (B, N), C.device, "f")
    out = torch.empty(B, M, device=C.device, dtype=torch.float32)
    lib = T.lib()
    with torch.cuda.device(C.device):
        ws = T.workspace(lib.sk_lse_col_workspace_bytes(B, N, M), C.device)
        rc = lib.sk_lse_col(*T.cost_args(C), f_.data_ptr(), float(epsilon), out.data_ptr(),
                            ws.data_ptr(), ws.numel(), T.stream_of(C.device))
        T.check(rc, "sk_lse_col")
    return out
