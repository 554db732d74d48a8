"""Multi-rank driver logic on CPU ``gloo`` ranks (world sizes 2, 4 and 8).

The drivers in sinkhorn_b200.distributed run unchanged; the per-rank GPU work
is replaced by a float64 numpy engine with the same semantics, so the test
checks the collective plumbing -- the global residual all-reduce of batch
sharding, the all-gather / merge / decision of row sharding, the global
default marginal -- against the oracle's single-process solve. A failure
test kills one rank mid-solve and checks that the survivor raises instead of
hanging.
"""

from __future__ import annotations

import datetime
import os
import socket
import traceback

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle as O


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _lse(x, axis):
    mx = np.max(x, axis=axis, keepdims=True)
    shift = np.where(np.isfinite(mx), mx, 0.0)
    with np.errstate(divide="ignore", invalid="ignore"):
        out = np.log(np.sum(np.exp(x - shift), axis=axis, keepdims=True)) + shift
    return np.squeeze(out, axis=axis)


def _guard(sm):
    return np.where(np.isinf(sm), 0.0, sm)


class NumpyBatchEngine:
    """One rank's items, masked forward semantics, float64."""

    def __init__(self, C, a, b, eps, tau_a, tau_b, ma, mb, max_iters, thr, ce):
        self.C = C.astype(np.float64)
        B, N, M = C.shape
        a = O.default_marginal(ma, B, N) if a is None else a
        b = O.default_marginal(mb, B, M) if b is None else b
        self.la, self.lb = O.log_marginal(a), O.log_marginal(b)
        self.ma = np.ones((B, N), bool) if ma is None else ma.astype(bool)
        self.mb = np.ones((B, M), bool) if mb is None else mb.astype(bool)
        self.eps, self.ce = eps, ce
        self.ra, self.rb = O.compute_rho(eps, tau_a), O.compute_rho(eps, tau_b)
        self.f, self.g = np.zeros((B, N)), np.zeros((B, M))
        self.it, self.res, self.done, self.n = 0, 0.0, False, None
        self.thr, self.max_iters = thr, max_iters
        self._r = torch.zeros(1, dtype=torch.float64)

    def _once(self):
        e, valid = self.eps, self.ma[:, :, None] & self.mb[:, None, :]
        xr = np.where(valid, (self.g[:, None, :] - self.C) / e, -np.inf)
        fn = self.ra * self.f + (1 - self.ra) * (e * self.la + _guard(-e * _lse(xr, 2)))
        xc = np.where(valid, (fn[:, :, None] - self.C) / e, -np.inf)
        gn = self.rb * self.g + (1 - self.rb) * (e * self.lb + _guard(-e * _lse(xc, 1)))
        fn, gn = np.where(self.ma, fn, 0.0), np.where(self.mb, gn, 0.0)
        r = max(np.abs(fn - self.f).max(), np.abs(gn - self.g).max())
        self.f, self.g = fn, gn
        self.it += 1
        if self.ce and self.it % self.ce == 0:
            self.res = max(self.res, r)

    def iterate(self, n):
        for _ in range(n):
            if not self.done:
                self._once()

    def residual(self):
        """The check's residual, in a tensor the driver reduces in place."""
        self._r.fill_(self.res)
        return self._r

    def decide(self):
        # the same decision as the device kernel: the reduced residual of the
        # check just run against the threshold (NaN never passes)
        if not self.done and float(self._r.item()) < self.thr:
            self.done, self.n = True, self.it
        self.res = 0.0

    def poll(self):
        return self.done

    def outcome(self):
        return (self.n, True) if self.done else (self.max_iters, False)

    def result(self):
        return self.f, self.g


class NumpyRowEngine:
    """One rank's rows of a row-sharded problem, float64."""

    def __init__(self, C_rows, a_rows, b, eps, tau_a, tau_b, ma_rows, mb, max_iters, thr, ce):
        self.C = C_rows.astype(np.float64)
        B, n, M = C_rows.shape
        self.la = O.log_marginal(a_rows)
        b = O.default_marginal(mb, B, M) if b is None else b
        self.lb = O.log_marginal(b)
        self.ma = np.ones((B, n), bool) if ma_rows is None else ma_rows.astype(bool)
        self.mb = np.ones((B, M), bool) if mb is None else mb.astype(bool)
        self.eps, self.ce, self.max_iters, self.thr = eps, ce, max_iters, thr
        self.ra, self.rb = O.compute_rho(eps, tau_a), O.compute_rho(eps, tau_b)
        self.f, self.g = np.zeros((B, n)), np.zeros((B, M))
        self.it, self.rf, self.state = 0, 0.0, (False, 0, False)

    def _check(self):
        return self.ce and (self.it + 1) % self.ce == 0 and self.thr > 0

    def row_sweep(self):
        if self.state[0]:
            return
        e, valid = self.eps, self.ma[:, :, None] & self.mb[:, None, :]
        xr = np.where(valid, (self.g[:, None, :] - self.C) / e, -np.inf)
        fn = self.ra * self.f + (1 - self.ra) * (e * self.la + _guard(-e * _lse(xr, 2)))
        fn = np.where(self.ma, fn, 0.0)
        self.rf = np.abs(fn - self.f).max() if self._check() else 0.0
        self.f = fn

    def partial(self):
        self.row_sweep()
        return self.col_partial()

    def rescale(self, part, gmax):
        p, m = part.numpy()[:-1], gmax.numpy()[:-1]
        with np.errstate(invalid="ignore"):
            s = np.where(np.isneginf(m), 0.0, np.exp(p - m))
        return torch.from_numpy(np.concatenate([s, [0.0]]))

    def col_finish_pairs(self, gmax, ssum):
        m, s = gmax.numpy(), ssum.numpy()
        with np.errstate(divide="ignore"):
            lse = np.where(np.isneginf(m[:-1]), -np.inf, m[:-1] + np.log(s[:-1]))
        parts = torch.from_numpy(np.concatenate([lse, [m[-1]]])[None, :])
        self.col_finish(parts)

    def col_partial(self):
        e, valid = self.eps, self.ma[:, :, None] & self.mb[:, None, :]
        xc = np.where(valid, (self.f[:, :, None] - self.C) / e, -np.inf)
        part = _lse(xc, 1).reshape(-1)
        return torch.from_numpy(np.concatenate([part, [self.rf]]))

    def col_finish(self, parts):
        if self.state[0]:
            return
        p = parts.numpy()
        B, M = self.g.shape
        lse = _lse(p[:, :-1], 0).reshape(B, M)
        e = self.eps
        gn = self.rb * self.g + (1 - self.rb) * (e * self.lb + _guard(-e * lse))
        gn = np.where(self.mb, gn, 0.0)
        r = max(np.abs(gn - self.g).max(), p[:, -1].max())
        check = self._check()
        self.g = gn
        self.it += 1
        if check and r < self.thr:
            self.state = (True, self.it, True)
        elif self.it >= self.max_iters:
            self.state = (True, self.it, False)

    def done(self):
        return self.state

    def result(self):
        return self.f, self.g

    # the peer-memory exchange's driver protocol, its data moved by a gloo
    # all-gather (the CUDA engine stores into the other ranks' buffers)
    single_read = True

    def peer_begin(self, group=None):
        dist.barrier(group=group)

    def peer_step(self):
        self._part = self.partial()

    def peer_finish(self):
        parts = [torch.empty_like(self._part) for _ in range(dist.get_world_size())]
        dist.all_gather(parts, self._part)
        self.col_finish(torch.stack(parts))


def _problem():
    rng = np.random.default_rng(3)
    B, N, M = 2, 41, 30
    C = rng.standard_normal((B, N, M)).astype(np.float32)
    ma = rng.random((B, N)) > 0.2
    mb = rng.random((B, M)) > 0.2
    return C, ma, mb


def _worker(rank, world, port, mode, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=20))
        from sinkhorn_b200.distributed import (sinkhorn_batch_sharded,
                                               sinkhorn_row_sharded)
        C, ma, mb = _problem()
        eps, tau, iters, thr, ce = 0.3, 1.0, 200, 1e-7, 10
        if mode in ("batch", "batch_nan"):
            sl = slice(rank, rank + 1)  # one item per rank
            cls = NumpyBatchEngine
            if mode == "batch_nan" and rank == 1:
                class Diverging(NumpyBatchEngine):
                    # this rank's item diverges: its residual is NaN at every
                    # check, while rank 0's converges below the threshold
                    def residual(self):
                        self._r.fill_(float("nan"))
                        return self._r
                cls = Diverging
            eng = cls(C[sl], None, None, eps, tau, None, ma[sl], mb[sl], iters, thr, ce)
            f, g, n, conv = sinkhorn_batch_sharded(C[sl], epsilon=eps, tau_a=tau,
                                                   max_iters=iters, threshold=thr,
                                                   check_every=ce, engine=eng)
        else:
            N = C.shape[1]
            # uneven shards (one of a single row at 4 and 8 ranks)
            cuts = {2: [0, 17, N], 4: [0, 9, 10, 26, N],
                    8: [0, 3, 4, 11, 12, 20, 26, 35, N]}[world]
            rows = slice(cuts[rank], cuts[rank + 1])
            ma_t = torch.from_numpy(ma[:, rows])
            from sinkhorn_b200.distributed import global_row_marginal
            a_rows = global_row_marginal(ma_t, N, C.shape[0], ma_t.shape[1], "cpu").numpy()
            if mode == "row_fail" and rank == 1:
                class Dying(NumpyRowEngine):
                    def partial(self):
                        if self.it == 3:
                            os._exit(3)  # the rank disappears between steps
                        return super().partial()
                cls = Dying
            else:
                cls = NumpyRowEngine
            eng = cls(C[:, rows], a_rows, None, eps, tau, None, ma[:, rows], mb, iters,
                      thr, ce)
            f, g, n, conv = sinkhorn_row_sharded(C[:, rows], a_rows, None, eps, tau, None,
                                                 torch.from_numpy(ma[:, rows]),
                                                 torch.from_numpy(mb), iters, thr, ce,
                                                 n_global=N, engine=eng,
                                                 merge={"row_gather": "gather",
                                                        "row_peer": "peer"}.get(mode,
                                                                                "allreduce"))
        q.put((rank, "ok", np.asarray(f), np.asarray(g), n, conv))
        dist.destroy_process_group()
    except Exception:  # noqa: BLE001 - report to the parent
        q.put((rank, "error", traceback.format_exc(), None, None, None))


def _run(mode, timeout=90, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for p in procs:
        p.join(timeout)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    while not q.empty():
        r = q.get()
        out[r[0]] = r[1:]
    return out, [p.exitcode for p in procs]


def _reference():
    C, ma, mb = _problem()
    return O.forward(C, None, None, 0.3, 1.0, None, ma, mb, 200, 1e-7, 10), C, ma, mb


def test_batch_sharded_matches_single_process():
    (fo, go, no, co), C, ma, mb = _reference()
    out, codes = _run("batch")
    assert codes == [0, 0], (codes, out)
    for r in (0, 1):
        st, f, g, n, conv = out[r]
        assert st == "ok", f
        assert (n, conv) == (no, co)
        np.testing.assert_allclose(f, fo[r:r + 1], atol=1e-9)
        np.testing.assert_allclose(g, go[r:r + 1], atol=1e-9)


def test_batch_sharded_nan_residual_on_one_rank_never_converges():
    """The reference's max over the whole batch stays NaN when one item
    diverges, so the threshold test never passes and the solve runs to
    max_iters unconverged (src/sinkhorn/triton/forward.py:176-182); the
    ranks' residual all-reduce must keep that NaN."""
    out, codes = _run("batch_nan")
    assert codes == [0, 0], (codes, out)
    for r in (0, 1):
        st, f, g, n, conv = out[r]
        assert st == "ok", f
        assert (n, conv) == (200, False)


@pytest.mark.parametrize("mode", ["row", "row_gather", "row_peer"])
def test_row_sharded_matches_single_process(mode):
    """The merges of the ranks' column LSEs: two all-reduces (MAX, then SUM of
    the rescaled sums), one all-gather, and the peer exchange's driver
    protocol (step + push, then the finish that waits for every rank)."""
    (fo, go, no, co), C, ma, mb = _reference()
    out, codes = _run(mode)
    assert codes == [0, 0], (codes, out)
    f = np.concatenate([out[0][1], out[1][1]], axis=1)
    for r in (0, 1):
        st, fr, g, n, conv = out[r]
        assert st == "ok", fr
        assert (n, conv) == (no, co)
        np.testing.assert_allclose(g, go, atol=1e-9)
    np.testing.assert_allclose(f, fo, atol=1e-9)


@pytest.mark.parametrize("world", [4, 8])
@pytest.mark.parametrize("mode", ["row", "row_peer"])
def test_row_sharded_four_and_eight_ranks_match_single_process(mode, world):
    """The same merges over 4 and 8 ranks (uneven shards, single-row ones
    among them): every rank's g and the concatenated f equal the
    single-process solve."""
    (fo, go, no, co), C, ma, mb = _reference()
    out, codes = _run(mode, timeout=120, world=world)
    assert codes == [0] * world, (codes, out)
    f = np.concatenate([out[r][1] for r in range(world)], axis=1)
    for r in range(world):
        st, fr, g, n, conv = out[r]
        assert st == "ok", fr
        assert (n, conv) == (no, co)
        np.testing.assert_allclose(g, go, atol=1e-9)
    np.testing.assert_allclose(f, fo, atol=1e-9)


def test_a_rank_that_dies_mid_solve_makes_the_other_raise():
    out, codes = _run("row_fail", timeout=120)
    assert codes[1] == 3
    assert codes[0] == 0  # the survivor returned after reporting
    assert out[0][0] == "error", out
