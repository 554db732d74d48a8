"""Multi-GPU Sinkhorn: batch sharding and row sharding over torch.distributed.

One process per GPU; the collectives run on the default (or given) process
group -- NCCL over NVLink on B200 boxes. The reference has no distributed
code; both modes keep its single-process results:

* ``sinkhorn_batch_sharded``: each rank solves its own batch items. The
  reference's convergence test is a max over the whole batch
  (src/sinkhorn/triton/forward.py:176-182), so every check period the ranks
  all-reduce(MAX) the residual -- on the device, with no host round trip --
  and a queued kernel takes the decision; the host learns of it one check
  period behind, like the single-GPU solve, and all ranks stop at the same
  iteration count: that of the unsharded batch.
* ``sinkhorn_row_sharded``: one problem whose C is split by rows. Rank r holds
  rows [r0, r1) of every item, its slice of f and a full copy of g. The
  f-update is local (one read of the rank's rows per iteration where the
  single-read iteration applies); the g-update merges the P per-rank column
  LSE vectors, either with two all-reduces of B*M floats -- MAX of the ranks'
  LSEs, then SUM of each rank's exp(LSE - max) (``merge="allreduce"``) --,
  with one all-gather of the P vectors (``merge="gather"``), or over NVLink
  peer memory (``merge="peer"``: each rank's merge kernel stores its vector
  into every rank's receive buffer and raises a flag there; the finish
  kernel waits for the P flags on the device -- no collective call and no
  host synchronisation per iteration). The ranks' f residual rides in the
  vectors' last slot, so every rank takes the same convergence decision
  without another collective.

The per-rank work goes through an *engine* (default: the CUDA kernels of
this package via the sk_solver_* ABI); the drivers only schedule it and run
the collectives, which lets the same driver code run on CPU ``gloo`` ranks in
tests.
"""

from __future__ import annotations

import torch
import torch.distributed as dist
from torch import Tensor

import ctypes

from .cuda.solver import ST_DONE, SinkhornSolver


# ---------------------------------------------------------------------------
# engines

class CudaBatchEngine:
    """Per-rank engine of the batch-sharded driver (sk_solver_* on one GPU).

    The kernels run with decide = 0: a check iteration leaves its residual in
    the status record, the driver reduces it across ranks in place, and
    ``decide`` queues the decision kernel (sk_solver_decide) -- nothing waits
    for the host. ``poll`` reads the decision of the check before the last
    one (a pinned copy queued after it), so the host waits one check period
    behind the GPU, never the GPU for the host."""

    def __init__(self, C, a, b, epsilon, tau_a, tau_b, mask_a, mask_b, max_iters,
                 threshold, check_every):
        self.s = SinkhornSolver(C, a, b, epsilon, tau_a, tau_b, mask_a, mask_b,
                                max_iters=max_iters, threshold=threshold,
                                check_every=check_every, decide=False)
        self.max_iters = max_iters
        self._host = torch.zeros((2, 16), dtype=torch.int32).pin_memory()
        self._ev = [torch.cuda.Event(), torch.cuda.Event()]
        self._k = 0

    def iterate(self, n: int) -> None:
        self.s.iterate(n)

    def residual(self) -> Tensor:
        """(1,) float tensor on the collective's device (a view: all-reduce in place)."""
        return self.s.residual_view()

    def decide(self) -> None:
        from . import _lib
        with torch.cuda.device(self.s.device):
            rc = self.s.lib.sk_solver_decide(self.s.ws.data_ptr(), self.s.stream)
            _lib.check(rc, "sk_solver_decide")
            slot = self._k % 2
            self._host[slot].copy_(self.s.status_view()[:16], non_blocking=True)
            self._ev[slot].record(torch.cuda.current_stream(self.s.device))
        self._k += 1

    def poll(self) -> bool:
        """Whether the check before the last one decided to stop."""
        if self._k < 2:
            return False
        prev = (self._k - 2) % 2
        self._ev[prev].synchronize()
        return bool(self._host[prev][ST_DONE].item())

    def outcome(self) -> tuple[int, bool]:
        st = self.s.status()
        if st["done"]:
            return st["n_iters"], st["converged"]
        return self.max_iters, False

    def result(self):
        return self.s.f, self.s.g


class CudaRowEngine:
    """Per-rank engine of the row-sharded driver: this rank's rows of C.

    ``partial`` is the rank's column LSE over its rows (B*M floats) plus its f
    residual in slot B*M: one single-read step (f-update and chunk partials)
    and the chunk merge where the shape has a fused plan, else the row sweep
    and a column sweep."""

    def __init__(self, C_rows, a_rows, b, epsilon, tau_a, tau_b, mask_a_rows, mask_b,
                 max_iters, threshold, check_every):
        self.s = SinkhornSolver(C_rows, a_rows, b, epsilon, tau_a, tau_b, mask_a_rows,
                                mask_b, max_iters=max_iters, threshold=threshold,
                                check_every=check_every, decide=True)
        B, N, M = C_rows.shape
        self.shape = (B, N, M)
        self.single_read = self.s.fused
        dev = C_rows.device
        self._partial = torch.empty(B * M + 1, device=dev, dtype=torch.float32)
        # the rescaled sums; slot B*M (unused) stays 0 through the SUM all-reduce
        self._s = torch.zeros(B * M + 1, device=dev, dtype=torch.float32)
        self._peer = None  # the peer-memory exchange, set up on first use

    def reset(self) -> None:
        """Start the solve again (prologue: marginals, potentials, status)."""
        self.s.init()

    def partial(self) -> Tensor:
        from . import _lib
        s = self.s
        with torch.cuda.device(s.device):
            if self.single_read:
                s.fused_step()
                rc = s.lib.sk_solver_chunk_merge(*s._cargs, self._partial.data_ptr(),
                                                 s.ws.data_ptr(), s.ws.numel(), s.stream)
                _lib.check(rc, "sk_solver_chunk_merge")
            else:
                s.row_sweep()
                rc = s.lib.sk_solver_col_partial(*s._cargs, s.epsilon,
                                                 self._partial.data_ptr(), s.ws.data_ptr(),
                                                 s.ws.numel(), s.stream)
                _lib.check(rc, "sk_solver_col_partial")
        return self._partial

    def col_finish(self, parts: Tensor) -> None:
        """g-update from the all-gathered (P, B*M+1) partials."""
        from . import _lib
        from . import _tensors as T
        s = self.s
        B, N, M = self.shape
        with torch.cuda.device(s.device):
            rc = s.lib.sk_solver_col_finish(parts.data_ptr(), parts.shape[0], B, N, M,
                                            T.ptr(s.mask_b), s.epsilon, s.tau_b,
                                            s.g.data_ptr(), s.ws.data_ptr(), s.ws.numel(),
                                            s.stream)
            _lib.check(rc, "sk_solver_col_finish")

    def rescale(self, part: Tensor, gmax: Tensor) -> Tensor:
        """exp(part - gmax) over the B*M columns: this rank's share of the sums."""
        from . import _lib
        s = self.s
        B, N, M = self.shape
        with torch.cuda.device(s.device):
            rc = s.lib.sk_solver_rank_rescale(part.data_ptr(), gmax.data_ptr(),
                                              self._s.data_ptr(), B * M, s.stream)
            _lib.check(rc, "sk_solver_rank_rescale")
        return self._s

    def col_finish_pairs(self, gmax: Tensor, ssum: Tensor) -> None:
        """g-update from the all-reduced (max, sum) pairs."""
        from . import _lib
        from . import _tensors as T
        s = self.s
        B, N, M = self.shape
        with torch.cuda.device(s.device):
            rc = s.lib.sk_solver_col_finish_pairs(gmax.data_ptr(), ssum.data_ptr(), B, N, M,
                                                  T.ptr(s.mask_b), s.epsilon, s.tau_b,
                                                  s.g.data_ptr(), s.ws.data_ptr(),
                                                  s.ws.numel(), s.stream)
            _lib.check(rc, "sk_solver_col_finish_pairs")

    def done(self) -> tuple[bool, int, bool]:
        st = self.s.status()
        return st["done"], st["n_iters"], st["converged"]

    def result(self):
        return self.s.f, self.s.g

    # -- the exchange over peer memory (merge="peer", fused shapes) --------
    def peer_begin(self, group=None) -> None:
        """Before a solve's first iteration: the ranks' receive buffers (set
        up once per engine), this rank's flags cleared, a host barrier."""
        if self._peer is None:
            B, N, M = self.shape
            self._peer = PeerExchange(B, M, self.s.device, group)
        self._peer.reset(self.s.stream)

    def peer_step(self) -> None:
        """The step on this rank's rows, then its column LSE vector stored
        into every rank's buffer (and the flags raised)."""
        from . import _lib
        s, ex = self.s, self._peer
        with torch.cuda.device(s.device):
            s.fused_step()
            rc = s.lib.sk_solver_chunk_merge_peer(*s._cargs, ex.bases, ex.P, ex.rank,
                                                  s.ws.data_ptr(), s.ws.numel(), s.stream)
            _lib.check(rc, "sk_solver_chunk_merge_peer")

    def peer_finish(self) -> None:
        """Wait for the P vectors of this iteration (on the device) and apply
        the g-update from their merge."""
        from . import _lib
        from . import _tensors as T
        s, ex = self.s, self._peer
        B, N, M = self.shape
        with torch.cuda.device(s.device):
            rc = s.lib.sk_solver_col_finish_peer(ex.own, ex.P, B, N, M, T.ptr(s.mask_b),
                                                 s.epsilon, s.tau_b, s.g.data_ptr(),
                                                 s.ws.data_ptr(), s.ws.numel(), s.stream)
            _lib.check(rc, "sk_solver_col_finish_peer")

    def close(self) -> None:
        """Release the peer exchange (a host barrier of every rank first)."""
        if self._peer is not None:
            self._peer.close()
            self._peer = None


class PeerExchange:
    """The ranks' receive buffers of the peer-memory exchange (one node, one
    GPU per rank, P <= 8): this rank's own buffer (sk_peer_buffer_alloc) and
    the others' opened from their CUDA IPC handles, gathered once with
    all_gather_object. ``bases[q]`` is rank q's buffer in this process."""

    def __init__(self, B: int, M: int, device, group=None):
        from . import _lib
        from . import _tensors as T
        self.P, self.rank = _world(group)
        self.group = group
        self.device = device
        self.B, self.M = B, M
        lib = T.lib()
        self.lib = lib
        nbytes = lib.sk_peer_buffer_bytes(self.P, B, M)
        if nbytes == 0:
            raise ValueError(f"the peer exchange takes 1..8 ranks, got {self.P}")
        own = ctypes.c_void_p()
        with torch.cuda.device(device):
            _lib.check(lib.sk_peer_buffer_alloc(nbytes, ctypes.byref(own)),
                       "sk_peer_buffer_alloc")
            handle = (ctypes.c_char * 64)()
            _lib.check(lib.sk_peer_handle(own, handle), "sk_peer_handle")
        self.own = own
        handles = [None] * self.P
        dist.all_gather_object(handles, bytes(handle), group=group)
        self._opened = []
        ptrs = []
        with torch.cuda.device(device):
            for q in range(self.P):
                if q == self.rank:
                    ptrs.append(own.value)
                    continue
                h = (ctypes.c_char * 64).from_buffer_copy(handles[q])
                p = ctypes.c_void_p()
                _lib.check(lib.sk_peer_open(h, ctypes.byref(p)), "sk_peer_open")
                self._opened.append(p)
                ptrs.append(p.value)
        self.bases = (ctypes.c_void_p * self.P)(*ptrs)

    def reset(self, stream) -> None:
        """Clear this rank's flags, then wait for every rank to have done so."""
        from . import _lib
        with torch.cuda.device(self.device):
            _lib.check(self.lib.sk_peer_reset(self.own, self.P, self.B, self.M, stream),
                       "sk_peer_reset")
            torch.cuda.synchronize(self.device)
        _barrier(self.group, self.device)

    def close(self) -> None:
        """Every rank is done with every buffer before any is released."""
        torch.cuda.synchronize(self.device)
        _barrier(self.group, self.device)
        with torch.cuda.device(self.device):
            for p in self._opened:
                self.lib.sk_peer_close(p)
            self.lib.sk_peer_buffer_free(self.own)
        self._opened = []


def _barrier(group, device):
    if dist.get_backend(group) == "nccl":
        dist.barrier(group=group, device_ids=[torch.device(device).index])
    else:
        dist.barrier(group=group)


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
    for the local items; n_iters / converged are identical on every rank.

    Each check period: the period's iterations, the residual all-reduced
    (MAX, NaN kept) in the device's status record, and the decision kernel,
    all queued; the host then waits for the previous period's decision, so
    every rank takes the same number of periods (and collectives)."""
    if engine is None:
        engine = CudaBatchEngine(C, a, b, epsilon, tau_a, tau_b, mask_a, mask_b,
                                 max_iters, threshold, check_every)
    checks = threshold > 0
    done = 0
    while done < max_iters:
        step = min(check_every if checks else max_iters, max_iters - done)
        engine.iterate(step)
        done += step
        if checks and done % check_every == 0:
            all_reduce_max_keep_nan(engine.residual(), group)
            engine.decide()
            if engine.poll():
                break
    n_iters, converged = engine.outcome()
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


MERGES = ("allreduce", "gather", "peer")


def sinkhorn_row_sharded(C_rows: Tensor, a_rows: Tensor | None = None,
                         b: Tensor | None = None, epsilon: float = 0.1,
                         tau_a: float | None = None, tau_b: float | None = None,
                         mask_a_rows: Tensor | None = None, mask_b: Tensor | None = None,
                         max_iters: int = 100, threshold: float = 1e-6,
                         check_every: int = 10, n_global: int | None = None, group=None,
                         engine=None, merge: str = "allreduce"):
    """Solve one problem whose cost rows are split over the ranks.

    C_rows: this rank's rows (B, N_local, M); a_rows / mask_a_rows: its slice
    of a / mask_a; b / mask_b: full. Returns (f_rows, g, n_iters, converged) with
    g and the counts identical on every rank. ``merge``: "allreduce" (MAX of
    the ranks' column LSEs, then SUM of their rescaled sums: 2 x (B*M+1)
    floats per iteration), "gather" (one all-gather of the P LSE vectors) or
    "peer" (stores into the other ranks' buffers over NVLink and device-side
    flags; shapes with a single-read iteration, else "gather")."""
    if merge not in MERGES:
        raise ValueError(f"merge must be one of {MERGES}, got {merge!r}")
    P, _ = _world(group)
    B, n_local, M = C_rows.shape
    if a_rows is None:
        if n_global is None:
            t = torch.tensor([n_local], device=C_rows.device, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
            n_global = int(t.item())
        a_rows = global_row_marginal(mask_a_rows, n_global, B, n_local, C_rows.device,
                                     group)
    own_engine = engine is None
    if own_engine:
        engine = CudaRowEngine(C_rows, a_rows, b, epsilon, tau_a, tau_b, mask_a_rows,
                               mask_b, max_iters, threshold, check_every)
    try:
        return _row_sharded_loop(engine, merge, P, max_iters, threshold, check_every, group)
    finally:
        if own_engine and hasattr(engine, "close"):
            engine.close()  # the peer buffers of an engine made here


def _row_sharded_loop(engine, merge, P, max_iters, threshold, check_every, group):
    parts = gmax = None
    poll = check_every if threshold > 0 else max_iters
    if merge == "peer":
        if getattr(engine, "single_read", False):
            engine.peer_begin(group)
        else:
            merge = "gather"
    for it in range(max_iters):
        if merge == "peer":
            engine.peer_step()
            engine.peer_finish()
            if (it + 1) % poll == 0 or it + 1 == max_iters:
                done, n, conv = engine.done()
                if done:
                    f, g = engine.result()
                    return f, g, n, conv
            continue
        part = engine.partial()
        if merge == "gather":
            if parts is None:
                parts = part.new_empty((P * part.numel(),))
            dist.all_gather_into_tensor(parts, part, group=group)
            engine.col_finish(parts.view(P, -1))
        else:
            if gmax is None:
                gmax = part.new_empty(part.shape)
            gmax.copy_(part)
            dist.all_reduce(gmax, op=dist.ReduceOp.MAX, group=group)
            ssum = engine.rescale(part, gmax)
            dist.all_reduce(ssum, op=dist.ReduceOp.SUM, group=group)
            engine.col_finish_pairs(gmax, ssum)
        if (it + 1) % poll == 0 or it + 1 == max_iters:
            done, n, conv = engine.done()
            if done:
                f, g = engine.result()
                return f, g, n, conv
    f, g = engine.result()
    return f, g, max_iters, False
