"""GPU parity of the single-read fused iterations against the fp64 oracle and
against the two-sweep kernels: k_fused_iter + k_col_finish (contiguous rows;
one-CTA units for 2048 < M < 8192, M % 4 == 0, 2-CTA clusters up to
M = 16384, M % 8 == 0; sk_forward's default on both) and k_rows_fused +
k_col_finish (contiguous rows, 512 <= M <= 2048, M % 4 == 0; sk_forward's
default there)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import ORACLE_RTOL, check_forward_parity, pot_tolerance
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _t(x):
    return None if x is None else torch.from_numpy(np.asarray(x)).cuda()


def _problem(B, N, M, seed, masked=False, scale=1.0):
    rng = np.random.default_rng(seed)
    x = rng.random((B, N, 3), dtype=np.float32)
    y = rng.random((B, M, 3), dtype=np.float32)
    C = ((x[:, :, None, :] - y[:, None, :, :]) ** 2).sum(-1).astype(np.float32)
    C = (C / C.max() * scale).astype(np.float32)
    ma = rng.random((B, N)) > 0.15 if masked else None
    mb = rng.random((B, M)) > 0.15 if masked else None
    return C, ma, mb


def test_plan_selects_the_fused_path():
    from sinkhorn_b200.cuda.solver import plan_query
    for shape, fused, fwd in (((1, 300, 2048), True, False), ((2, 64, 16384), True, True),
                              ((1, 64, 4104), True, True), ((1, 64, 8192), True, True),
                              ((1, 64, 1024), True, False), ((16, 2048, 2048), True, True),
                              ((64, 1024, 1024), True, True), ((10, 512, 512), True, True),
                              ((1, 64, 256), False, False), ((1, 64, 32768), True, True),
                              ((1, 64, 2052), True, True), ((1, 64, 2050), False, False)):
        C = torch.zeros(shape, device="cuda")
        q = plan_query(C)
        assert q["fused"] == fused and q["forward_fused"] == fwd, shape
    # chunks hold at most 2048 rows (their previous f is kept on chip)
    C = torch.zeros(1, 5000, 8192, device="cuda")
    assert plan_query(C)["chunks"] >= 3
    Ct = torch.zeros(1, 4096, 64, device="cuda").transpose(1, 2)  # strided: no fused path
    assert not plan_query(Ct)["fused"]


@pytest.mark.parametrize("B,N,M,eps,tau,masked,iters,thr,ce,scale", [
    (1, 300, 2048, 0.05, None, False, 40, 0.0, 10, 1.0),
    (2, 150, 4104, 0.1, 1.0, True, 60, 1e-6, 10, 1.0),
    (1, 96, 16384, 0.05, None, False, 25, 0.0, 10, 1.0),
    (3, 40, 8192, 0.2, 0.5, True, 80, 1e-6, 1, 1.0),
    (1, 3, 2048, 0.1, None, False, 30, 0.0, 10, 1.0),
    # small eps: column terms span far more than the unchecked fold allows, so
    # later rows take the checked path that moves column references
    (1, 256, 4096, 0.004, None, False, 30, 0.0, 10, 1.0),
    (2, 128, 2048, 0.01, 0.3, True, 30, 0.0, 10, 1.0),
    # large cost range (C up to 100)
    (1, 200, 4096, 0.5, None, False, 30, 0.0, 10, 100.0),
    # one-CTA units: rows that do not fill the lanes' float4 groups (2052,
    # 3000, 6000), masks, rho != 0, every-iteration checks, a small eps
    (2, 130, 2052, 0.1, 1.0, True, 60, 1e-6, 10, 1.0),
    (3, 77, 3000, 0.05, None, True, 40, 0.0, 10, 1.0),
    (1, 150, 6000, 0.2, 0.5, True, 80, 1e-6, 1, 1.0),
    (2, 64, 7168, 0.004, None, False, 30, 0.0, 10, 1.0),
])
def test_fused_iteration_matches_oracle(B, N, M, eps, tau, masked, iters, thr, ce, scale):
    """The single-read iteration runs the same solve as
    sinkhorn_forward_triton: compare with the fp64 oracle."""
    from sinkhorn_b200.cuda.solver import SinkhornSolver
    C, ma, mb = _problem(B, N, M, seed=B * N + M, masked=masked, scale=scale)
    s = SinkhornSolver(_t(C), None, None, eps, tau, tau, _t(ma), _t(mb), max_iters=iters,
                       threshold=thr, check_every=ce)
    assert s.fused
    s.iterate(iters, fused=True)
    st = s.status()
    assert st["err"] == 0
    n, conv = (st["n_iters"] if st["done"] else iters), st["converged"]
    check_forward_parity(s.f, s.g, n, conv, dict(
        C=C, eps=eps, tau_a=tau, tau_b=tau, mask_a=ma, mask_b=mb, max_iters=iters,
        threshold=thr, check_every=ce))


def test_fused_and_two_sweep_paths_agree():
    from sinkhorn_b200.cuda.solver import SinkhornSolver
    C, _, _ = _problem(1, 512, 4096, seed=3)
    Ct = _t(C)
    s1 = SinkhornSolver(Ct, epsilon=0.05, max_iters=10 ** 6, threshold=0.0)
    s2 = SinkhornSolver(Ct, epsilon=0.05, max_iters=10 ** 6, threshold=0.0)
    assert s1.fused and s1.forward_fused
    s1.iterate(50, fused=True)
    s2.iterate(50, fused=False)
    torch.cuda.synchronize()
    assert (s1.f - s2.f).abs().max().item() < 1e-4
    assert (s1.g - s2.g).abs().max().item() < 1e-4
    assert s1.status()["iter"] == s2.status()["iter"] == 50
    assert s1.status()["err"] == 0


@pytest.mark.parametrize("B,N,M", [(1, 512, 4096), (2, 300, 2048)])
def test_fused_unbalanced_far_from_convergence(B, N, M):
    """rho != 0 mixes each row's previous f into the new one; both CTAs of a
    row must use the same previous value although f is updated in place.
    Compared with the two-sweep kernels after a few iterations, while f
    still moves a lot from one iteration to the next."""
    from sinkhorn_b200.cuda.solver import SinkhornSolver
    C, _, _ = _problem(B, N, M, seed=11)
    Ct = _t(C)
    kw = dict(epsilon=0.05, tau_a=0.1, tau_b=0.1, max_iters=10 ** 6, threshold=0.0)
    s1 = SinkhornSolver(Ct, **kw)
    s2 = SinkhornSolver(Ct, **kw)
    s1.iterate(8, fused=True)
    s2.iterate(8, fused=False)
    torch.cuda.synchronize()
    assert s1.status()["err"] == 0
    assert (s1.f - s2.f).abs().max().item() < 1e-4
    assert (s1.g - s2.g).abs().max().item() < 1e-4


@pytest.mark.parametrize("B,N,M,eps,tau,masked,thr,ce", [
    (1, 300, 8192, 0.05, None, False, 1e-6, 10),
    (2, 200, 8192, 0.1, 1.0, True, 1e-6, 1),
    (1, 64, 16384, 0.2, None, False, 1e-5, 10),
])
def test_public_forward_on_fused_shapes(B, N, M, eps, tau, masked, thr, ce):
    """sinkhorn() on shapes where sk_forward runs the fused iteration:
    convergence decided on the device through k_col_finish, potentials and
    iteration count against the oracle."""
    from sinkhorn_b200 import sinkhorn
    from sinkhorn_b200.cuda.solver import plan_query
    C, ma, mb = _problem(B, N, M, seed=N + M, masked=masked)
    Ct = _t(C)
    assert plan_query(Ct)["forward_fused"]
    out = sinkhorn(Ct, epsilon=eps, tau_a=tau, tau_b=tau, mask_a=_t(ma), mask_b=_t(mb),
                   max_iters=300, threshold=thr, backend="cuda", check_every=ce)
    check_forward_parity(out.f, out.g, out.n_iters, out.converged, dict(
        C=C, eps=eps, tau_a=tau, tau_b=tau, mask_a=ma, mask_b=mb, max_iters=300,
        threshold=thr, check_every=ce))


def _prefix_problem(B, N, M, seed):
    """cfg3-like: C ~ N(0,1), prefix masks of random lengths, softmax marginals."""
    gen = torch.Generator().manual_seed(seed)
    C = torch.randn(B, N, M, generator=gen)
    la = torch.randint(N // 4, N + 1, (B,), generator=gen)
    lb = torch.randint(M // 4, M + 1, (B,), generator=gen)
    ma = torch.arange(N)[None, :] < la[:, None]
    mb = torch.arange(M)[None, :] < lb[:, None]
    a = torch.softmax(torch.randn(B, N, generator=gen).masked_fill(~ma, float("-inf")), -1)
    b = torch.softmax(torch.randn(B, M, generator=gen).masked_fill(~mb, float("-inf")), -1)
    return C, a, b, ma, mb


@pytest.mark.parametrize("B,N,M,eps,tau,masked,iters,thr,ce", [
    (1, 300, 1024, 0.05, None, False, 40, 0.0, 10),
    (3, 100, 512, 0.1, 1.0, True, 60, 1e-6, 10),
    (2, 257, 2048, 0.05, 0.5, True, 50, 1e-6, 1),
    (1, 5, 1024, 0.1, None, False, 30, 0.0, 10),     # fewer rows than one stage
    (2, 64, 1028, 0.02, None, False, 30, 0.0, 10),   # M % 8 != 0, small eps
    (1, 1500, 600, 0.1, 0.3, True, 40, 1e-6, 10),    # many chunks, M not a power of two
])
def test_rows_fused_iteration_matches_oracle(B, N, M, eps, tau, masked, iters, thr, ce):
    """k_rows_fused (one CTA per row chunk, whole rows staged) runs the solve
    of sinkhorn_forward_triton: compare with the fp64 oracle."""
    from sinkhorn_b200.cuda.solver import SinkhornSolver, plan_query
    C, ma, mb = _problem(B, N, M, seed=7 * B + N + M, masked=masked)
    Ct = _t(C)
    assert plan_query(Ct)["fused"]
    s = SinkhornSolver(Ct, None, None, eps, tau, tau, _t(ma), _t(mb), max_iters=iters,
                       threshold=thr, check_every=ce)
    s.iterate(iters, fused=True)
    st = s.status()
    assert st["err"] == 0
    n, conv = (st["n_iters"] if st["done"] else iters), st["converged"]
    check_forward_parity(s.f, s.g, n, conv, dict(
        C=C, eps=eps, tau_a=tau, tau_b=tau, mask_a=ma, mask_b=mb, max_iters=iters,
        threshold=thr, check_every=ce))


def test_rows_fused_prefix_masks_match_oracle():
    """Prefix masks (the masked, unbalanced batch workload in miniature): the
    kernel stages only each item's valid rows and column span."""
    from sinkhorn_b200.cuda.forward import sinkhorn_forward_cuda
    from sinkhorn_b200.cuda.solver import plan_query
    C, a, b, ma, mb = _prefix_problem(10, 512, 1024, seed=0)
    assert plan_query(C.cuda())["forward_fused"]
    f, g, n, conv = sinkhorn_forward_cuda(C.cuda(), a.cuda(), b.cuda(), 0.1, 1.0, 1.0,
                                          ma.cuda(), mb.cuda(), 60, 1e-6)
    fo, go, no, co = O.forward(C, a, b, 0.1, 1.0, 1.0, ma, mb, 60, 1e-6, 10)
    assert n == no and conv == co
    tol = pot_tolerance(0.1)
    np.testing.assert_allclose(f.cpu().numpy(), fo, atol=tol, rtol=ORACLE_RTOL)
    np.testing.assert_allclose(g.cpu().numpy(), go, atol=tol, rtol=ORACLE_RTOL)
    assert not f.cpu()[~ma].any() and not g.cpu()[~mb].any()


@pytest.mark.parametrize("M,tau", [(2048, None), (1024, 0.5), (512, None)])
def test_rows_fused_far_start_matches_oracle(M, tau):
    """k_rows_fused sums each row against its previous LSE. Rows whose costs
    sit 400 eps above the rest leave that sum's range in the first iterations
    (their stages are summed again from each lane's max) while the other
    stages keep the one-pass sums: parity with the fp64 oracle throughout."""
    from sinkhorn_b200.cuda.solver import SinkhornSolver, plan_query
    B, N, eps, iters = 2, 300, 0.05, 40
    rng = np.random.default_rng(M)
    C = rng.random((B, N, M), dtype=np.float32)
    C += (rng.random((B, N, 1)) < 0.3).astype(np.float32) * np.float32(400 * eps)
    Ct = _t(C)
    assert plan_query(Ct)["fused"]
    s = SinkhornSolver(Ct, None, None, eps, tau, tau, max_iters=iters, threshold=0.0)
    s.iterate(iters, fused=True)
    assert s.status()["err"] == 0
    fo, go, _, _ = O.forward(C, None, None, eps, tau, tau, None, None, iters, 0.0, 10)
    tol = pot_tolerance(eps)
    np.testing.assert_allclose(s.f.cpu().numpy(), fo, atol=tol, rtol=ORACLE_RTOL)
    np.testing.assert_allclose(s.g.cpu().numpy(), go, atol=tol, rtol=ORACLE_RTOL)


def test_rows_fused_and_two_sweep_paths_agree():
    from sinkhorn_b200.cuda.solver import SinkhornSolver
    C, _, _ = _problem(2, 700, 2048, seed=5)
    Ct = _t(C)
    kw = dict(epsilon=0.05, tau_a=0.2, tau_b=0.2, max_iters=10 ** 6, threshold=0.0)
    s1 = SinkhornSolver(Ct, **kw)
    s2 = SinkhornSolver(Ct, **kw)
    s1.iterate(30, fused=True)
    s2.iterate(30, fused=False)
    torch.cuda.synchronize()
    assert s1.status()["err"] == 0
    assert (s1.f - s2.f).abs().max().item() < 1e-4
    assert (s1.g - s2.g).abs().max().item() < 1e-4


@pytest.mark.parametrize("M", [8192, 32768])
def test_fused_iteration_starved_columns_are_summed_directly(M):
    """k_fused_iter's column lanes fold the row lanes' exponentials against a
    per-lane pivot; columns 5 and M - 3 cost 60 more than the rest at
    eps = 0.05, so in the first iterations their pivoted sums fall below
    2^-72 and they are summed again straight from C: parity with the fp64
    oracle (2- and 4-CTA clusters)."""
    from sinkhorn_b200.cuda.solver import SinkhornSolver, plan_query
    C, _, _ = _problem(1, 300, M, seed=M + 1)
    C[:, :, 5] += 60.0
    C[:, :, M - 3] += 60.0
    Ct = _t(C)
    assert plan_query(Ct)["fused"]
    s = SinkhornSolver(Ct, None, None, 0.05, max_iters=25, threshold=0.0)
    s.iterate(25, fused=True)
    assert s.status()["err"] == 0
    fo, go, _, _ = O.forward(C, None, None, 0.05, None, None, None, None, 25, 0.0, 10)
    tol = pot_tolerance(0.05)
    np.testing.assert_allclose(s.f.cpu().numpy(), fo, atol=tol, rtol=ORACLE_RTOL)
    np.testing.assert_allclose(s.g.cpu().numpy(), go, atol=tol, rtol=ORACLE_RTOL)
    assert np.isfinite(s.g.cpu().numpy()).all()
