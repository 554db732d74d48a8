"""GPU parity of the forward solve and the softmins against the oracle and the
reference's golden vectors (called through the C ABI via the Python mirror)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import (ORACLE_RTOL, check_forward_parity, forward_golden_names,
                      iterations_agree, load_golden, pot_tolerance)
from oracle import oracle as O

pytestmark = pytest.mark.gpu

FWD = forward_golden_names()


def _t(x, dtype=None):
    if x is None:
        return None
    t = torch.from_numpy(np.asarray(x))
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()


def _residual_oracle(d):
    def at(k):
        args = (d["C"], d.get("a"), d.get("b"), d["eps"], d["tau_a"], d["tau_b"],
                d.get("mask_a"), d.get("mask_b"))
        f1, g1, _, _ = O.forward(*args, k, 0.0, 1)
        f0, g0, _, _ = O.forward(*args, k - 1, 0.0, 1)
        return max(np.abs(f1 - f0).max(), np.abs(g1 - g0).max())
    return at


@pytest.mark.parametrize("name", FWD)
def test_forward_matches_golden(name):
    from sinkhorn_b200.cuda.forward import sinkhorn_forward_cuda
    d = load_golden(name)
    f, g, n, conv = sinkhorn_forward_cuda(
        _t(d["C"]), _t(d.get("a")), _t(d.get("b")), d["eps"], d["tau_a"], d["tau_b"],
        _t(d.get("mask_a")), _t(d.get("mask_b")), d["max_iters"], d["threshold"],
        check_every=d["check_every"])
    tol = pot_tolerance(d["eps"])
    assert iterations_agree(n, conv, d, _residual_oracle(d)), (n, conv, d["n_iters"])
    np.testing.assert_allclose(f.cpu().numpy(), d["f"], rtol=0, atol=tol)
    np.testing.assert_allclose(g.cpu().numpy(), d["g"], rtol=0, atol=tol)


@pytest.mark.parametrize("name", FWD)
def test_forward_matches_oracle_both_cadences(name):
    """Same inputs through the fp64 oracle, check every 10 and every 1."""
    from sinkhorn_b200.cuda.forward import sinkhorn_forward_cuda
    d = load_golden(name)
    for ce in (10, 1):
        f, g, n, conv = sinkhorn_forward_cuda(
            _t(d["C"]), _t(d.get("a")), _t(d.get("b")), d["eps"], d["tau_a"],
            d["tau_b"], _t(d.get("mask_a")), _t(d.get("mask_b")), d["max_iters"],
            d["threshold"], check_every=ce)
        check_forward_parity(f, g, n, conv, dict(d, check_every=ce))


def test_lse_row_col_match_triton_golden():
    from sinkhorn_b200.cuda.lse_kernel import lse_col, lse_row
    d = load_golden("tri_lse")
    r = lse_row(_t(d["C"]), _t(d["g"]), d["eps"]).cpu().numpy()
    c = lse_col(_t(d["C"]), _t(d["f"]), d["eps"]).cpu().numpy()
    np.testing.assert_allclose(r, d["row"], atol=1e-5)
    np.testing.assert_allclose(c, d["col"], atol=1e-5)
    assert r[1, 2] == 0.0 and c[0, 4] == 0.0


@pytest.mark.parametrize("shape", [(1, 1, 1), (2, 3, 5), (1, 129, 127), (3, 64, 520),
                                   (1, 1000, 8), (2, 17, 4100)])
@pytest.mark.parametrize("eps", [0.05, 1.0])
def test_lse_odd_shapes(shape, eps):
    from sinkhorn_b200.cuda.lse_kernel import lse_col, lse_row
    rng = np.random.default_rng(sum(shape))
    C = rng.standard_normal(shape).astype(np.float32)
    g = rng.standard_normal((shape[0], shape[2])).astype(np.float32)
    f = rng.standard_normal((shape[0], shape[1])).astype(np.float32)
    np.testing.assert_allclose(lse_row(_t(C), _t(g), eps).cpu().numpy(),
                               O.lse_row(C, g, eps), atol=2e-5 * max(1, eps), rtol=1e-5)
    np.testing.assert_allclose(lse_col(_t(C), _t(f), eps).cpu().numpy(),
                               O.lse_col(C, f, eps), atol=2e-5 * max(1, eps), rtol=1e-5)


def test_noncontiguous_cost_uses_strided_path():
    from sinkhorn_b200.cuda.forward import sinkhorn_forward_cuda
    rng = np.random.default_rng(5)
    Ct = rng.standard_normal((2, 40, 36)).astype(np.float32)
    C = _t(Ct).transpose(1, 2)  # (2, 36, 40) view with sCm != 1
    f, g, n, conv = sinkhorn_forward_cuda(C, epsilon=0.2, max_iters=50, threshold=0.0)
    fo, go, no, _ = O.forward(np.ascontiguousarray(Ct.transpose(0, 2, 1)), epsilon=0.2,
                              max_iters=50, threshold=0.0, check_every=10)
    assert n == no == 50
    np.testing.assert_allclose(f.cpu().numpy(), fo, atol=1e-4, rtol=ORACLE_RTOL)
    np.testing.assert_allclose(g.cpu().numpy(), go, atol=1e-4, rtol=ORACLE_RTOL)


@pytest.mark.parametrize("B,N,M,tau,masked", [
    (3, 200, 1024, 1.0, True),     # two sweeps per iteration
    (1, 256, 8192, None, False),   # the fused single-read iteration
])
def test_warm_start_resumes_bit_exactly(B, N, M, tau, masked):
    """A threshold-0 solve of 100 iterations equals 30 iterations followed by
    70 more started from the saved potentials (sk_forward_warm): each
    iteration depends only on (f, g), so a checkpoint loses nothing."""
    from sinkhorn_b200.cuda.forward import sinkhorn_forward_cuda
    rng = np.random.default_rng(B * N + M)
    C = torch.from_numpy(rng.random((B, N, M), dtype=np.float32)).cuda()
    ma = torch.from_numpy(rng.random((B, N)) > 0.2).cuda() if masked else None
    mb = torch.from_numpy(rng.random((B, M)) > 0.2).cuda() if masked else None
    f1, g1, n1, _ = sinkhorn_forward_cuda(C, None, None, 0.05, tau, tau, ma, mb, 100, 0.0)
    f0, g0, n0, _ = sinkhorn_forward_cuda(C, None, None, 0.05, tau, tau, ma, mb, 30, 0.0)
    f2, g2, n2, _ = sinkhorn_forward_cuda(C, None, None, 0.05, tau, tau, ma, mb, 70, 0.0,
                                          f_init=f0, g_init=g0)
    assert (n1, n0, n2) == (100, 30, 70)
    assert torch.equal(f1, f2) and torch.equal(g1, g2)


def test_warm_start_matches_the_reference_warm_iterations():
    """sk_forward_warm from the reference's (f_init, g_init) against
    _sinkhorn_iters_from_init (autograd.py:134-178) itself: without masks the
    forward iteration and the reference's warm iteration are the same map."""
    from sinkhorn_b200.cuda.forward import sinkhorn_forward_cuda
    d = load_golden("warm_init_balanced")
    f, g, n, conv = sinkhorn_forward_cuda(
        _t(d["C"]), _t(d["a"]), _t(d["b"]), d["eps"], d["tau_a"], d["tau_b"], None, None,
        d["n_iters"], 0.0, f_init=_t(d["f_init"]), g_init=_t(d["g_init"]))
    assert (n, conv) == (d["n_iters"], False)
    tol = pot_tolerance(d["eps"])
    np.testing.assert_allclose(f.cpu().numpy(), d["f"], rtol=0, atol=tol)
    np.testing.assert_allclose(g.cpu().numpy(), d["g"], rtol=0, atol=tol)


@pytest.mark.parametrize("B,N,M,tau,ce,thr,kernel", [
    (3, 200, 1024, 1.0, 1, 1e-6, "two sweeps"),
    (1, 256, 8192, 0.5, 10, 1e-6, "fused"),         # k_fused_iter + k_col_finish
    (2, 300, 4096, 1.0, 10, 1e-6, "fused"),         # its one-CTA units
    (12, 512, 1024, 1.0, 1, 1e-6, "rows fused"),    # k_rows_fused + k_col_finish
    (10, 512, 1024, None, 10, 0.0, "rows fused"),
    (2, 100, 90, 0.5, 1, 1e-6, "on chip"),          # one-launch solve
])
def test_warm_start_matches_oracle(B, N, M, tau, ce, thr, kernel):
    """sk_forward_warm and the oracle started from the same random non-zero
    potentials (masked entries included, prefix masks so rows and columns
    outside the valid ranges are exercised), masked and unbalanced: the
    iteration count and the potentials, on each kernel family."""
    from sinkhorn_b200.cuda.forward import sinkhorn_forward_cuda
    from sinkhorn_b200.cuda.solver import plan_query
    rng = np.random.default_rng(B * N + M)
    C = rng.random((B, N, M), dtype=np.float32)
    la = rng.integers(N // 2, N + 1, B)
    lb = rng.integers(M // 2, M + 1, B)
    ma = (np.arange(N)[None, :] < la[:, None]) & (rng.random((B, N)) > 0.1)
    mb = (np.arange(M)[None, :] < lb[:, None]) & (rng.random((B, M)) > 0.1)
    fi = (0.3 * rng.standard_normal((B, N))).astype(np.float32)
    gi = (0.3 * rng.standard_normal((B, M))).astype(np.float32)
    Ct = _t(C)
    q = plan_query(Ct)
    assert q["forward_fused"] == (kernel in ("fused", "rows fused")), q
    f, g, n, conv = sinkhorn_forward_cuda(Ct, None, None, 0.05, tau, tau, _t(ma), _t(mb), 300,
                                          thr, check_every=ce, f_init=_t(fi), g_init=_t(gi))
    check_forward_parity(f, g, n, conv, dict(
        C=C, eps=0.05, tau_a=tau, tau_b=tau, mask_a=ma, mask_b=mb, max_iters=300,
        threshold=thr, check_every=ce, f_init=fi, g_init=gi))
    assert not f.cpu().numpy()[~ma].any() and not g.cpu().numpy()[~mb].any()


def test_warm_start_first_residual_counts_masked_start_values():
    """The first residual of a warm start measures the step from the given
    potentials, masked entries included (they are reset to 0): a threshold
    just above that step stops after one iteration, just below it does not."""
    from sinkhorn_b200.cuda.forward import sinkhorn_forward_cuda
    d = load_golden("warm_init_masked_unbal")
    args = (d["C"], d["a"], d["b"], d["eps"], d["tau_a"], d["tau_b"], d["mask_a"], d["mask_b"])
    f1, g1, _, _ = O.forward(*args, 1, 0.0, 1, f_init=d["f_init"], g_init=d["g_init"])
    step = max(np.abs(f1 - d["f_init"]).max(), np.abs(g1 - d["g_init"]).max())
    targs = (_t(d["C"]), _t(d["a"]), _t(d["b"]), d["eps"], d["tau_a"], d["tau_b"],
             _t(d["mask_a"]), _t(d["mask_b"]))
    for thr, iters, want in ((step * 1.01, 5, (1, True)), (step * 0.99, 1, (1, False))):
        _, _, n, conv = sinkhorn_forward_cuda(*targs, iters, thr, check_every=1,
                                              f_init=_t(d["f_init"]), g_init=_t(d["g_init"]))
        assert (n, conv) == want, (thr, step)


def test_warm_start_from_a_converged_solution_stops_at_the_first_check():
    from sinkhorn_b200 import sinkhorn
    rng = np.random.default_rng(5)
    x = rng.random((2, 300, 3), dtype=np.float32)
    y = rng.random((2, 500, 3), dtype=np.float32)
    C = ((x[:, :, None, :] - y[:, None, :, :]) ** 2).sum(-1).astype(np.float32)
    C = torch.from_numpy(C / C.max()).cuda()
    kw = dict(epsilon=0.02, max_iters=5000, threshold=1e-6, backend="cuda", check_every=1)
    out = sinkhorn(C, **kw)
    assert out.converged and out.n_iters > 5
    again = sinkhorn(C, f_init=out.f, g_init=out.g, **kw)
    assert again.converged and again.n_iters == 1
    torch.testing.assert_close(again.f, out.f, atol=1e-5, rtol=0)


def test_warm_start_is_rejected_on_the_differentiable_path():
    from sinkhorn_b200 import sinkhorn
    C = torch.rand(1, 16, 16, device="cuda", requires_grad=True)
    with pytest.raises(ValueError):
        sinkhorn(C, epsilon=0.1, backend="cuda", f_init=torch.zeros(1, 16, device="cuda"))


@pytest.mark.parametrize("B,N,M,masked,tau,ce,thr,transposed", [
    (6, 100, 90, True, 1.0, 1, 1e-6, False),   # batch-wide checks at grid barriers
    (1, 200, 224, False, None, 10, 1e-6, False),
    (3, 80, 96, False, 0.5, 10, 0.0, True),    # strided C staged on chip
])
def test_onchip_solve_matches_oracle(B, N, M, masked, tau, ce, thr, transposed):
    """Shapes whose C fits in one SM's shared memory run the whole solve in
    one launch (sk_onchip.cu)."""
    from sinkhorn_b200.cuda.forward import sinkhorn_forward_cuda
    rng = np.random.default_rng(N * M + B)
    if transposed:
        base = rng.standard_normal((B, M, N)).astype(np.float32)
        C = np.ascontiguousarray(base.transpose(0, 2, 1))
        Ct = torch.from_numpy(base).cuda().transpose(1, 2)
    else:
        C = rng.standard_normal((B, N, M)).astype(np.float32)
        Ct = torch.from_numpy(C).cuda()
    ma = rng.random((B, N)) > 0.2 if masked else None
    mb = rng.random((B, M)) > 0.2 if masked else None
    tm = lambda x: None if x is None else torch.from_numpy(x).cuda()  # noqa: E731
    f, g, n, conv = sinkhorn_forward_cuda(Ct, None, None, 0.1, tau, tau, tm(ma), tm(mb), 300,
                                          thr, check_every=ce)
    check_forward_parity(f, g, n, conv, dict(
        C=C, eps=0.1, tau_a=tau, tau_b=tau, mask_a=ma, mask_b=mb, max_iters=300,
        threshold=thr, check_every=ce))


def test_batch_too_large_to_be_resident_takes_the_sweep_loop():
    """160 items of 200 x 200 (one SM each) cannot all be resident for the
    on-chip solver's barriers: the solve runs the two-sweep loop instead and
    still gives the oracle's potentials."""
    from sinkhorn_b200.cuda.forward import sinkhorn_forward_cuda
    rng = np.random.default_rng(11)
    B, N, M = 160, 200, 200
    C = rng.random((B, N, M), dtype=np.float32)
    f, g, n, conv = sinkhorn_forward_cuda(torch.from_numpy(C).cuda(), None, None, 0.2, None,
                                          None, None, None, 40, 1e-7, check_every=10)
    # the check is a max over the whole batch: the oracle solves all 160 items
    check_forward_parity(f, g, n, conv, dict(
        C=C, eps=0.2, tau_a=None, tau_b=None, max_iters=40, threshold=1e-7,
        check_every=10))
