"""GPU tests of the persistent solve (k_fused_iter with PERSIST: the whole
forward solve in one cooperative launch, the opt-in sk_solver_solve on
single-read shapes whose units fit one wave of clusters) and of the
single-read step on clusters of 4 and 8 CTAs, for rows of 16384 < M <= 65536
columns.

The persistent solve merges the chunk partials in k_col_finish's order, so it
must be bit-identical to the step path (single-read steps + k_col_finish) on
the same problem, convergence decision included; both are compared with the
fp64 oracle as well."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import check_forward_parity

pytestmark = pytest.mark.gpu


def _t(x):
    return None if x is None else torch.from_numpy(np.asarray(x)).cuda()


def _problem(B, N, M, seed, masked=False):
    rng = np.random.default_rng(seed)
    x = rng.random((B, N, 3), dtype=np.float32)
    y = rng.random((B, M, 3), dtype=np.float32)
    C = ((x[:, :, None, :] - y[:, None, :, :]) ** 2).sum(-1).astype(np.float32)
    C = (C / C.max()).astype(np.float32)
    ma = rng.random((B, N)) > 0.15 if masked else None
    mb = rng.random((B, M)) > 0.15 if masked else None
    return C, ma, mb


def test_plan_marks_persistent_shapes():
    from sinkhorn_b200.cuda.solver import plan_query
    for shape, fwd, persist in (((1, 16384, 16384), True, True), ((2, 64, 16384), True, True),
                                ((1, 64, 32768), True, True), ((1, 300, 65536), True, True),
                                ((1, 256, 8192), True, True), ((300, 64, 8192), True, False),
                                ((1, 64, 4096), True, False), ((1, 64, 65540), False, False)):
        q = plan_query(torch.empty(shape, device="cuda"))
        assert q["forward_fused"] == fwd and q["persist"] == persist, (shape, q)


@pytest.mark.parametrize("B,N,M,eps,tau,masked,iters,thr,ce", [
    (1, 2000, 16384, 0.05, None, False, 30, 0.0, 10),
    (2, 700, 8192, 0.1, 1.0, True, 200, 1e-6, 1),
    (3, 300, 12288, 0.05, 0.5, True, 300, 1e-6, 10),   # row parts of 6144: guarded lanes
    (1, 900, 32768, 0.05, None, False, 20, 0.0, 10),   # 4-CTA clusters
    (1, 400, 65536, 0.02, 0.3, True, 60, 1e-6, 10),    # 8-CTA clusters
])
def test_persistent_solve_equals_step_path(B, N, M, eps, tau, masked, iters, thr, ce):
    from sinkhorn_b200.cuda.solver import SinkhornSolver
    C, ma, mb = _problem(B, N, M, seed=B * N + M, masked=masked)
    Ct = _t(C)
    kw = dict(epsilon=eps, tau_a=tau, tau_b=tau, mask_a=_t(ma), mask_b=_t(mb),
              max_iters=iters, threshold=thr, check_every=ce)
    s1 = SinkhornSolver(Ct, **kw)
    assert s1.fused and s1.persist
    s1.solve()
    s2 = SinkhornSolver(Ct, **kw)
    s2.iterate(iters, fused=True)
    st1, st2 = s1.status(), s2.status()
    assert st1["err"] == 0 and st2["err"] == 0
    assert (st1["n_iters"], st1["converged"]) == (st2["n_iters"], st2["converged"])
    assert torch.equal(s1.f, s2.f) and torch.equal(s1.g, s2.g)
    check_forward_parity(s1.f, s1.g, st1["n_iters"], st1["converged"], dict(
        C=C, eps=eps, tau_a=tau, tau_b=tau, mask_a=ma, mask_b=mb, max_iters=iters,
        threshold=thr, check_every=ce))


@pytest.mark.parametrize("B,N,M,eps,tau,masked,iters,thr,ce", [
    (1, 300, 32768, 0.05, None, False, 300, 1e-6, 10),
    (2, 150, 20000, 0.1, 1.0, True, 300, 1e-6, 1),     # 4-CTA clusters, parts of 5000
    (1, 128, 65536, 0.05, None, False, 40, 0.0, 10),   # 8-CTA clusters
    (1, 1200, 65536, 0.05, None, False, 20, 0.0, 10),  # ~70 rows per unit
    (40, 32, 32768, 0.1, None, False, 30, 0.0, 10),    # more units than one wave: steps
])
def test_public_forward_on_large_rows(B, N, M, eps, tau, masked, iters, thr, ce):
    """sinkhorn() where a row is split over 4 or 8 CTAs: against the oracle."""
    from sinkhorn_b200 import sinkhorn
    from sinkhorn_b200.cuda.solver import plan_query
    C, ma, mb = _problem(B, N, M, seed=N + M, masked=masked)
    Ct = _t(C)
    assert plan_query(Ct)["forward_fused"]
    out = sinkhorn(Ct, epsilon=eps, tau_a=tau, tau_b=tau, mask_a=_t(ma), mask_b=_t(mb),
                   max_iters=iters, threshold=thr, backend="cuda", check_every=ce)
    check_forward_parity(out.f, out.g, out.n_iters, out.converged, dict(
        C=C, eps=eps, tau_a=tau, tau_b=tau, mask_a=ma, mask_b=mb, max_iters=iters,
        threshold=thr, check_every=ce))


def test_persistent_solve_handles_zero_and_one_iteration():
    from sinkhorn_b200.cuda.solver import SinkhornSolver
    from oracle import oracle as O
    C, _, _ = _problem(1, 256, 16384, seed=3)
    Ct = _t(C)
    s0 = SinkhornSolver(Ct, epsilon=0.05, max_iters=0, threshold=1e-6)
    s0.solve()
    assert s0.status()["err"] == 0
    assert not s0.f.abs().max().item() and not s0.g.abs().max().item()
    s1 = SinkhornSolver(Ct, epsilon=0.05, max_iters=1, threshold=1e-6, check_every=1)
    assert s1.persist
    s1.solve()
    st = s1.status()
    n = st["n_iters"] if st["done"] else 1
    fo, go, no, co = O.forward(C, None, None, 0.05, None, None, None, None, 1, 1e-6, 1)
    assert st["err"] == 0 and (n, st["converged"]) == (no, co) == (1, False)
    np.testing.assert_allclose(s1.f.cpu().numpy(), fo, atol=1e-4, rtol=2e-6)
    np.testing.assert_allclose(s1.g.cpu().numpy(), go, atol=1e-4, rtol=2e-6)
