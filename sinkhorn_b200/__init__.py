"""sinkhorn_b200: log-domain Sinkhorn optimal transport on B200 (sm_100a).

A drop-in ``backend="cuda"`` for the vv137/sinkhorn API: ``sinkhorn``,
``SinkhornOutput`` and ``sinkhorn_differentiable`` keep the reference's
signatures and semantics; the work runs in hand-written CUDA kernels
(libsinkhorn_b200.so, C ABI in include/sinkhorn_b200.h).
"""

__version__ = "0.1.0"

from .autograd import SinkhornFunction, sinkhorn_differentiable
from .cuda.plan import marginal_error as compute_marginal_error
from .sinkhorn import SinkhornOutput, sinkhorn

__all__ = ["sinkhorn", "SinkhornOutput", "sinkhorn_differentiable", "SinkhornFunction",
           "compute_marginal_error", "__version__"]
