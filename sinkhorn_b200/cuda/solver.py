"""Step-level access to the CUDA solve (sk_solver_* in the C ABI).

``SinkhornSolver`` owns the potentials and the workspace of one problem and
exposes the pieces of sinkhorn_forward_triton's loop
(src/sinkhorn/triton/forward.py:161-184): ``row_sweep`` (f-update),
``col_sweep`` (g-update, residual, iteration counter), ``iterate`` (both,
n times, no host sync) and the status record. Drivers that interleave their
own work between sweeps -- a collective across ranks, per-kernel timing --
use it; ``sinkhorn_forward_cuda`` is the one-call path.
"""

from __future__ import annotations

import ctypes

import torch
from torch import Tensor

from .. import _tensors as T

# status record at offset 0 of the workspace (int32 fields)
ST_ITER, ST_DONE, ST_NITERS, ST_CONVERGED, ST_RESIDUAL = 0, 1, 2, 3, 4
ST_ERR = 10  # int index of Status.err (byte offset 40)


def plan_query(C: Tensor) -> dict:
    """Which kernels a cost of this shape / layout runs on."""
    lib = T.lib()
    vec, fused = ctypes.c_int(0), ctypes.c_int(0)
    chunks = ctypes.c_int64(0)
    rc = lib.sk_plan_query(*T.cost_args(C), ctypes.byref(vec), ctypes.byref(fused),
                           ctypes.byref(chunks))
    T.check(rc, "sk_plan_query")
    return {"vec": vec.value, "fused": fused.value >= 1, "forward_fused": fused.value >= 2,
            "persist": fused.value == 3, "chunks": chunks.value}


def ex2_rate(device=None) -> float:
    """Measured ex2.approx results per second of the current (or given) GPU:
    the exponential floor of a sweep (one exp per element of C)."""
    import torch
    lib = T.lib()
    with torch.cuda.device(device if device is not None else torch.cuda.current_device()):
        nbytes = int(lib.sk_probe_ex2_scratch_bytes())
        scratch = torch.empty(max(nbytes, 4), dtype=torch.uint8, device="cuda")
        rate = ctypes.c_double(0.0)
        rc = lib.sk_probe_ex2_rate(scratch.data_ptr(), nbytes, ctypes.byref(rate),
                                   torch.cuda.current_stream().cuda_stream)
        T.check(rc, "sk_probe_ex2_rate")
    return rate.value


class SinkhornSolver:
    def __init__(self, C: Tensor, a: Tensor | None = None, b: Tensor | None = None,
                 epsilon: float = 0.1, tau_a: float | None = None,
                 tau_b: float | None = None, mask_a: Tensor | None = None,
                 mask_b: Tensor | None = None, max_iters: int = 100,
                 threshold: float = 1e-6, check_every: int = 10, decide: bool = True):
        T.check_cost(C)
        self.C = C
        B, N, M = C.shape
        self.shape = (B, N, M)
        self.device = C.device
        self.a = T.vec(a, (B, N), C.device, "a")
        self.b = T.vec(b, (B, M), C.device, "b")
        self.mask_a = T.mask(mask_a, (B, N), C.device, "mask_a")
        self.mask_b = T.mask(mask_b, (B, M), C.device, "mask_b")
        self.epsilon = float(epsilon)
        self.tau_a = T.tau_arg(tau_a)
        self.tau_b = T.tau_arg(tau_b)
        self.max_iters = int(max_iters)
        self.threshold = float(threshold)
        self.check_every = int(check_every)
        self.decide = bool(decide)
        self.lib = T.lib()
        self.f = torch.empty(B, N, device=C.device, dtype=torch.float32)
        self.g = torch.empty(B, M, device=C.device, dtype=torch.float32)
        self.ws = T.workspace(self.lib.sk_forward_workspace_bytes(B, N, M), C.device)
        self._cargs = T.cost_args(C)
        self.plan = plan_query(C)
        self.fused = bool(self.plan["fused"])            # single-read steps available
        self.persist = bool(self.plan["persist"])        # one-launch solve available
        self.forward_fused = bool(self.plan["forward_fused"])  # what sk_forward runs
        self.init()

    @property
    def stream(self) -> int:
        return T.stream_of(self.device)

    def init(self) -> None:
        with torch.cuda.device(self.device):
            rc = self.lib.sk_solver_init(
                *self._cargs, T.ptr(self.a), T.ptr(self.b), T.ptr(self.mask_a),
                T.ptr(self.mask_b), self.max_iters, self.threshold, self.check_every,
                int(self.decide), self.f.data_ptr(), self.g.data_ptr(), self.ws.data_ptr(),
                self.ws.numel(), self.stream)
            T.check(rc, "sk_solver_init")

    def row_sweep(self) -> None:
        rc = self.lib.sk_solver_row_sweep(*self._cargs, T.ptr(self.mask_a), self.epsilon,
                                          self.tau_a, self.f.data_ptr(), self.ws.data_ptr(),
                                          self.ws.numel(), self.stream)
        T.check(rc, "sk_solver_row_sweep")

    def col_sweep(self) -> None:
        rc = self.lib.sk_solver_col_sweep(*self._cargs, T.ptr(self.mask_b), self.epsilon,
                                          self.tau_b, self.g.data_ptr(), self.ws.data_ptr(),
                                          self.ws.numel(), self.stream)
        T.check(rc, "sk_solver_col_sweep")

    def fused_step(self) -> None:
        """f-update + per-chunk column partials in one read of C (fused shapes)."""
        rc = self.lib.sk_solver_fused_step(*self._cargs, T.ptr(self.mask_a), self.epsilon,
                                           self.tau_a, self.f.data_ptr(), self.ws.data_ptr(),
                                           self.ws.numel(), self.stream)
        T.check(rc, "sk_solver_fused_step")

    def fused_finish(self) -> None:
        """Merge the chunk partials: g-update, residual, check (fused shapes)."""
        rc = self.lib.sk_solver_fused_finish(*self._cargs, T.ptr(self.mask_b), self.epsilon,
                                             self.tau_b, self.g.data_ptr(), self.ws.data_ptr(),
                                             self.ws.numel(), self.stream)
        T.check(rc, "sk_solver_fused_finish")

    def solve(self) -> None:
        """The remaining iterations as one persistent launch (sk_solver_solve;
        shapes whose plan has ``persist``)."""
        with torch.cuda.device(self.device):
            rc = self.lib.sk_solver_solve(*self._cargs, T.ptr(self.mask_a), T.ptr(self.mask_b),
                                          self.epsilon, self.tau_a, self.tau_b,
                                          self.f.data_ptr(), self.g.data_ptr(),
                                          self.ws.data_ptr(), self.ws.numel(), self.stream)
            T.check(rc, "sk_solver_solve")

    def iterate(self, n: int, fused: bool | None = None) -> None:
        """n iterations on the kernels sk_forward uses (``fused=True`` opts in to
        the single-read iteration where the shape has one)."""
        use_fused = self.forward_fused if fused is None else (bool(fused) and self.fused)
        with torch.cuda.device(self.device):
            for _ in range(int(n)):
                if use_fused:
                    self.fused_step()
                    self.fused_finish()
                else:
                    self.row_sweep()
                    self.col_sweep()

    def status_view(self) -> Tensor:
        """int32 view of the status record (device, no sync)."""
        return self.ws[:64].view(torch.int32)

    def residual_view(self) -> Tensor:
        """float32 view (shape (1,)) of the last check iteration's residual."""
        return self.ws[16:20].view(torch.float32)

    def status(self) -> dict:
        it, done, n, conv = (ctypes.c_int(0) for _ in range(4))
        res = ctypes.c_float(0)
        with torch.cuda.device(self.device):
            rc = self.lib.sk_solver_status(self.ws.data_ptr(), ctypes.byref(it),
                                           ctypes.byref(done), ctypes.byref(n),
                                           ctypes.byref(conv), ctypes.byref(res),
                                           self.stream)
            T.check(rc, "sk_solver_status")
        err = int(self.status_view()[ST_ERR].item())  # 2: a bounded wait gave up
        return dict(iter=it.value, done=bool(done.value), n_iters=n.value,
                    converged=bool(conv.value), residual=res.value, err=err)

    def mark_done(self, converged: bool, n_iters: int) -> None:
        """Record an externally taken decision (e.g. a cross-rank check): every
        later sweep returns immediately."""
        st = self.status_view()
        st[ST_DONE] = 1
        st[ST_NITERS] = int(n_iters)
        st[ST_CONVERGED] = int(bool(converged))

    def clear_residual(self) -> None:
        self.status_view()[ST_RESIDUAL] = 0
