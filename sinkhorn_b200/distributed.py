"""Multi-GPU Sinkhorn: batch sharding and row sharding over torch.distributed.

One process per GPU; the collectives run on the default (or given) process
group -- NCCL over NVLink on B200 boxes. The reference has no distributed
code; both modes keep its single-process results:

* ``sinkhorn_batch_sharded``: each rank solves its own batch items. The
  reference's convergence test is a max over the whole batch
  (src/sinkhorn/triton/forward.py:176-182), so every check period the ranks
  all-reduce(MAX) one float -- the residual -- and stop together; the
  iteration counts are those of the unsharded batch.
* ``sinkhorn_row_sharded``: one problem whose C is split by rows. Rank r holds
  rows [r0, r1) of every item, its slice of f and a full copy of g. The
  f-update is local; the g-update merges the P per-rank column LSE vectors,
  exchanged with one all-gather of B*M+1 floats per iteration (the extra float
  carries the rank's f residual, so the convergence decision needs no other
  collective and is taken identically on every rank).

The per-rank work goes through an *engine* (default: the CUDA kernels of
this package via the sk_solver_* ABI); the drivers only schedule it and run
the collectives, which lets the same driver code run on CPU ``gloo`` ranks in
tests.
"""

from __future__ import annotations

import torch
import torch.distributed as dist
from torch import Tensor

from .cuda.solver import SinkhornSolver


# ---------------------------------------------------------------------------
# engines

class CudaBatchEngine:
    """Per-rank engine of the batch-sharded driver (sk_solver_* on one GPU)."""

    def __init__(self, C, a, b, epsilon, tau_a, tau_b, mask_a, mask_b, max_iters,
                 threshold, check_every):
        self.s = SinkhornSolver(C, a, b, epsilon, tau_a, tau_b, mask_a, mask_b,
                                max_iters=max_iters, threshold=threshold,
                                check_every=check_every, decide=False)

    def iterate(self, n: int) -> None:
        self.s.iterate(n)

    def residual(self) -> Tensor:
        """(1,) float tensor on the collective's device (a view: all-reduce in place)."""
        return self.s.residual_view()

    def clear_residual(self) -> None:
        self.s.clear_residual()

    def mark_done(self, converged: bool, n_iters: int) -> None:
        self.s.mark_done(converged, n_iters)

    def result(self):
        return self.s.f, self.s.g


class CudaRowEngine:
    """Per-rank engine of the row-sharded driver: this rank's rows of C."""

    def __init__(self, C_rows, a_rows, b, epsilon, tau_a, tau_b, mask_a_rows, mask_b,
                 max_iters, threshold, check_every):
        self.s = SinkhornSolver(C_rows, a_rows, b, epsilon, tau_a, tau_b, mask_a_rows,
                                mask_b, max_iters=max_iters, threshold=threshold,
                                check_every=check_every, decide=True)
        B, N, M = C_rows.shape
        self.shape = (B, N, M)
        self.partial = torch.empty(B * M + 1, device=C_rows.device, dtype=torch.float32)

    def row_sweep(self) -> None:
        self.s.row_sweep()

    def col_partial(self) -> Tensor:
        s = self.s
        rc = s.lib.sk_solver_col_partial(*s._cargs, s.epsilon, self.partial.data_ptr(),
                                         s.ws.data_ptr(), s.ws.numel(), s.stream)
        from . import _lib
        _lib.check(rc, "sk_solver_col_partial")
        return self.partial

    def col_finish(self, parts: Tensor) -> None:
        s = self.s
        B, N, M = self.shape
        from . import _tensors as T
        from . import _lib
        rc = s.lib.sk_solver_col_finish(parts.data_ptr(), parts.shape[0], B, N, M,
                                        T.ptr(s.mask_b), s.epsilon, s.tau_b,
                                        s.g.data_ptr(), s.ws.data_ptr(), s.ws.numel(),
                                        s.stream)
        _lib.check(rc, "sk_solver_col_finish")

    def done(self) -> tuple[bool, int, bool]:
        st = self.s.status()
        return st["done"], st["n_iters"], st["converged"]

    def result(self):
        return self.s.f, self.s.g


# ---------------------------------------------------------------------------
# drivers

def _world(group):
    return dist.get_world_size(group), dist.get_rank(group)


def all_reduce_max_keep_nan(r: Tensor, group=None) -> Tensor:
    """In-place all-reduce MAX of a non-negative residual that keeps NaN.

    A float MAX may drop a NaN (fmax semantics), which would let the other
    ranks' small residuals stop a batch whose one item diverged; the
    reference's max over the whole batch stays NaN and never passes the
    threshold test (src/sinkhorn/triton/forward.py:176-182). So the reduction
    runs on the bit patterns: for non-negative IEEE floats the integer order is
    the numeric order, and a (positive) NaN sorts above +inf."""
    r.abs_()  # a NaN with its sign bit set would sort below every number
    bits = r.view(torch.int32 if r.element_size() == 4 else torch.int64)
    dist.all_reduce(bits, op=dist.ReduceOp.MAX, group=group)
    return r


def sinkhorn_batch_sharded(C: Tensor, a: Tensor | None = None, b: Tensor | None = None,
                           epsilon: float = 0.1, tau_a: float | None = None,
                           tau_b: float | None = None, mask_a: Tensor | None = None,
                           mask_b: Tensor | None = None, max_iters: int = 100,
                           threshold: float = 1e-6, check_every: int = 10, group=None,
                           engine=None):
    """Solve this rank's batch items (C: (B_local, N, M)) with the global
    convergence test of the whole batch. Returns (f, g, n_iters, converged)
    for the local items; n_iters / converged are identical on every rank."""
    if engine is None:
        engine = CudaBatchEngine(C, a, b, epsilon, tau_a, tau_b, mask_a, mask_b,
                                 max_iters, threshold, check_every)
    checks = threshold > 0
    n_iters, converged = max_iters, False
    done = 0
    while done < max_iters:
        step = min(check_every if checks else max_iters, max_iters - done)
        engine.iterate(step)
        done += step
        if checks and done % check_every == 0:
            r = all_reduce_max_keep_nan(engine.residual(), group)
            if float(r.item()) < threshold:
                n_iters, converged = done, True
                engine.mark_done(True, done)
                break
            engine.clear_residual()
    f, g = engine.result()
    return f, g, n_iters, converged


def global_row_marginal(mask_rows: Tensor | None, n_global: int, B: int, n_local: int,
                        device, group=None) -> Tensor:
    """Default marginal of forward.py:132-142 for a row shard: uniform 1/N over
    the global rows, or mask / (global count of valid rows, clamped at 1)."""
    if mask_rows is None:
        return torch.full((B, n_local), 1.0, device=device, dtype=torch.float32) / n_global
    m = mask_rows.to(torch.float32)
    cnt = m.sum(dim=-1, keepdim=True)
    dist.all_reduce(cnt, op=dist.ReduceOp.SUM, group=group)
    return m / cnt.clamp(min=1)


def sinkhorn_row_sharded(C_rows: Tensor, a_rows: Tensor | None = None,
                         b: Tensor | None = None, epsilon: float = 0.1,
                         tau_a: float | None = None, tau_b: float | None = None,
                         mask_a_rows: Tensor | None = None, mask_b: Tensor | None = None,
                         max_iters: int = 100, threshold: float = 1e-6,
                         check_every: int = 10, n_global: int | None = None, group=None,
                         engine=None):
    """Solve one problem whose cost rows are split over the ranks.

    C_rows: this rank's rows (B, N_local, M); a_rows / mask_a_rows: its slice
    of a / mask_a; b / mask_b: full. Returns (f_rows, g, n_iters, converged) with
    g and the counts identical on every rank."""
    P, _ = _world(group)
    B, n_local, M = C_rows.shape
    if a_rows is None:
        if n_global is None:
            t = torch.tensor([n_local], device=C_rows.device, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
            n_global = int(t.item())
        a_rows = global_row_marginal(mask_a_rows, n_global, B, n_local, C_rows.device,
                                     group)
    if engine is None:
        engine = CudaRowEngine(C_rows, a_rows, b, epsilon, tau_a, tau_b, mask_a_rows,
                               mask_b, max_iters, threshold, check_every)
    parts = None
    poll = check_every if threshold > 0 else max_iters
    for it in range(max_iters):
        engine.row_sweep()
        part = engine.col_partial()
        if parts is None:
            parts = part.new_empty((P * part.numel(),))
        dist.all_gather_into_tensor(parts, part, group=group)
        engine.col_finish(parts.view(P, -1))
        if (it + 1) % poll == 0 or it + 1 == max_iters:
            done, n, conv = engine.done()
            if done:
                f, g = engine.result()
                return f, g, n, conv
    f, g = engine.result()
    return f, g, max_iters, False
