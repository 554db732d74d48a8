"""GPU parity of transport_plan / cost / jvp / plan adjoint / backward against
the reference's golden vectors and the fp64 oracle (through the C ABI)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden_names, iterations_agree, load_golden, oracle_residual
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _t(x, requires_grad=False):
    if x is None:
        return None
    t = torch.from_numpy(np.asarray(x)).cuda()
    if requires_grad:
        t.requires_grad_(True)
    return t


PLAN_CASES = [n for n in golden_names() if not n.startswith(("bwd_", "tri_", "imp_"))
              and "P" in load_golden(n)]


@pytest.mark.parametrize("name", PLAN_CASES)
def test_plan_and_cost_from_reference_potentials(name):
    from sinkhorn_b200 import SinkhornOutput
    d = load_golden(name)
    out = SinkhornOutput(f=_t(d["f"]), g=_t(d["g"]), n_iters=d["n_iters"],
                         converged=bool(d["converged"]))
    P = out.transport_plan(_t(d["C"]), d["eps"], _t(d.get("mask_a")),
                           _t(d.get("mask_b"))).cpu().numpy()
    scale = np.abs(d["P"]).max()
    np.testing.assert_allclose(P, d["P"], rtol=2e-5, atol=1e-6 * scale)
    c = out.cost(_t(d["C"]), d["eps"]).cpu().numpy()
    np.testing.assert_allclose(c, d["cost"], rtol=2e-5, atol=1e-6)


@pytest.mark.parametrize("name", [n for n in PLAN_CASES if "marginal_err" in load_golden(n)])
def test_marginal_error_from_reference_potentials(name):
    """compute_marginal_error (pytorch/balanced.py:183-213) from the
    reference's potentials: the reference's value and the fp64 oracle's."""
    from conftest import marginal_err_tolerance
    from sinkhorn_b200 import compute_marginal_error
    d = load_golden(name)
    e = float(compute_marginal_error(_t(d["C"]), _t(d["f"]), _t(d["g"]), _t(d["me_a"]),
                                     _t(d["me_b"]), d["eps"], _t(d.get("mask_a")),
                                     _t(d.get("mask_b"))))
    tol = marginal_err_tolerance(d["me_a"], d["me_b"])
    ref = float(d["marginal_err"])
    assert abs(e - ref) <= tol + 1e-3 * ref, (e, ref, tol)
    o = O.marginal_error(d["C"], d["f"], d["g"], d["me_a"], d["me_b"], d["eps"],
                         d.get("mask_a"), d.get("mask_b"))
    assert abs(e - o) <= tol + 1e-3 * o, (e, o, tol)


@pytest.mark.parametrize("masked", [False, True])
def test_marginal_error_matches_oracle_unconverged(masked):
    """A few iterations only (large violations), rectangular, with and
    without masks; float4 layout."""
    from conftest import marginal_err_tolerance
    from sinkhorn_b200 import compute_marginal_error, sinkhorn
    rng = np.random.default_rng(7)
    B, N, M = 2, 300, 2048
    C = rng.random((B, N, M), dtype=np.float32)
    a = rng.random((B, N)).astype(np.float32)
    b = rng.random((B, M)).astype(np.float32)
    ma = rng.random((B, N)) > 0.2 if masked else None
    mb = rng.random((B, M)) > 0.2 if masked else None
    a /= a.sum(-1, keepdims=True)
    b /= b.sum(-1, keepdims=True)
    out = sinkhorn(_t(C), _t(a), _t(b), epsilon=0.05, mask_a=_t(ma), mask_b=_t(mb),
                   max_iters=1, threshold=0.0, backend="cuda")
    f, g = out.f.cpu().numpy(), out.g.cpu().numpy()
    e = float(compute_marginal_error(_t(C), out.f, out.g, _t(a), _t(b), 0.05, _t(ma), _t(mb)))
    o = O.marginal_error(C, f, g, a, b, 0.05, ma, mb)
    tol = marginal_err_tolerance(a, b)
    assert o > 100 * tol  # not converged: a real violation is measured
    assert abs(e - o) <= tol + 1e-4 * o, (e, o)


def test_jvp_plan_matches_triton_golden():
    from sinkhorn_b200.cuda import jvp_cuda
    d = load_golden("tri_jvp")
    of, og = jvp_cuda(_t(d["v_f"]), _t(d["v_g"]), _t(d["P"]), d["rho_a"], d["rho_b"])
    np.testing.assert_allclose(of.cpu().numpy(), d["out_f"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(og.cpu().numpy(), d["out_g"], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("shape", [(2, 33, 47), (1, 256, 512), (3, 64, 64)])
def test_jvp_free_matches_plan_form(shape):
    from sinkhorn_b200.cuda import jvp_cuda_free
    rng = np.random.default_rng(1)
    B, N, M = shape
    C = rng.random(shape).astype(np.float32)
    f = (0.1 * rng.standard_normal((B, N))).astype(np.float32)
    g = (0.1 * rng.standard_normal((B, M))).astype(np.float32)
    vf = rng.standard_normal((B, N)).astype(np.float32)
    vg = rng.standard_normal((B, M)).astype(np.float32)
    P = O.transport_plan(C, f, g, 0.3)
    ef, eg = O.jvp(P, vf, vg, 0.25, 0.5)
    of, og = jvp_cuda_free(_t(vf), _t(vg), _t(C), _t(f), _t(g), 0.3, 0.25, 0.5)
    np.testing.assert_allclose(of.cpu().numpy(), ef, rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(og.cpu().numpy(), eg, rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("masked", [False, True])
def test_plan_adjoint_matches_oracle(masked):
    from sinkhorn_b200.cuda import plan_backward
    rng = np.random.default_rng(2)
    B, N, M = 2, 40, 52
    C = rng.random((B, N, M)).astype(np.float32)
    f = (0.2 * rng.standard_normal((B, N))).astype(np.float32)
    g = (0.2 * rng.standard_normal((B, M))).astype(np.float32)
    gP = rng.standard_normal((B, N, M)).astype(np.float32)
    ma = rng.random((B, N)) > 0.2 if masked else None
    mb = rng.random((B, M)) > 0.2 if masked else None
    edC, edf, edg = O.plan_backward(C, f, g, 0.5, gP, ma, mb)
    dC, df, dg = plan_backward(_t(C), _t(f), _t(g), 0.5, _t(gP), _t(ma), _t(mb))
    np.testing.assert_allclose(dC.cpu().numpy(), edC, rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(df.cpu().numpy(), edf, rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(dg.cpu().numpy(), edg, rtol=1e-4, atol=1e-4)


def _rel_err(x, ref):
    return float(np.abs(x - ref).max() / max(np.abs(ref).max(), 1e-30))


@pytest.mark.parametrize("name", golden_names("bwd_"))
def test_backward_matches_reference_golden(name):
    """dC within 1e-3 relative of the reference's autograd (parity contract).

    The fixture's forward used the PyTorch path (check every iteration), so the
    cuda forward runs with check_every=1 here."""
    from sinkhorn_b200 import SinkhornOutput, sinkhorn_differentiable
    d = load_golden(name)
    C = _t(d["C"], requires_grad=True)
    grad_ab = "da" in d
    a = _t(d.get("a"), requires_grad=grad_ab)
    b = _t(d.get("b"), requires_grad=grad_ab)
    f, g = sinkhorn_differentiable(C, a, b, d["eps"], d["tau_a"], d["tau_b"],
                                   _t(d.get("mask_a")), _t(d.get("mask_b")),
                                   d["max_iters"], d["threshold"], d["grad_iters"],
                                   check_every=1)
    if d["loss_kind"] == "plan_cost":
        out = SinkhornOutput(f=f, g=g, n_iters=0, converged=True)
        loss = (out.transport_plan(C, d["eps"]) * C).sum()
    else:
        # the fixture stored the upstream gradients; use them as loss weights
        loss = (f * _t(d["grad_f"])).sum() + (g * _t(d["grad_g"])).sum()
    loss.backward()
    assert _rel_err(C.grad.cpu().numpy(), d["dC"]) <= 1e-3
    if grad_ab:
        assert _rel_err(a.grad.cpu().numpy(), d["da"]) <= 1e-3
        assert _rel_err(b.grad.cpu().numpy(), d["db"]) <= 1e-3


@pytest.mark.parametrize("grad_iters", [0, 3, 10])
@pytest.mark.parametrize("masked", [False, True])
@pytest.mark.parametrize("tau", [None, 1.0])
def test_backward_matches_oracle(grad_iters, masked, tau):
    """sk_backward vs the fp64 oracle on the same (f*, g*) and upstream grads,
    truncated and full modes, with and without masks (full mode with masks is
    the case where the reference itself returns NaN)."""
    from sinkhorn_b200.autograd import sinkhorn_backward_cuda
    rng = np.random.default_rng(grad_iters + 10 * masked)
    B, N, M = 2, 48, 36
    C = rng.random((B, N, M)).astype(np.float32)
    ma = rng.random((B, N)) > 0.15 if masked else None
    mb = rng.random((B, M)) > 0.15 if masked else None
    eps, iters, thr = 0.2, 40, 1e-6
    fs, gs, _, _ = O.forward(C, None, None, eps, tau, tau, ma, mb, iters, thr, 10)
    fs, gs = fs.astype(np.float32), gs.astype(np.float32)
    gf = rng.standard_normal((B, N)).astype(np.float32)
    gg = rng.standard_normal((B, M)).astype(np.float32)
    edC, _, _, eK = O.backward(C, None, None, eps, tau, tau, ma, mb, iters, thr,
                               grad_iters, fs, gs, gf, gg)
    dC, _, _, K = sinkhorn_backward_cuda(_t(C), None, None, eps, tau, tau, _t(ma), _t(mb),
                                         iters, thr, grad_iters, _t(fs), _t(gs), _t(gf),
                                         _t(gg))
    if K != eK:
        # only the full recompute (its own per-iteration convergence from
        # zeros) may stop elsewhere, and only inside the fp32 band of the
        # threshold; dC is then compared with the oracle's backward through
        # exactly K recomputed iterations
        p = dict(C=C, eps=eps, tau_a=tau, tau_b=tau, mask_a=ma, mask_b=mb)
        ref = dict(f=fs, g=gs, n_iters=eK, converged=eK < iters, threshold=thr,
                   check_every=1)
        assert grad_iters == 0 and iterations_agree(K, K < iters, ref, oracle_residual(p)), \
            (K, eK)
        edC, _, _, _ = O.backward(C, None, None, eps, tau, tau, ma, mb, K, 0.0, 0, fs, gs,
                                  gf, gg)
    assert _rel_err(dC.cpu().numpy(), edC) <= 1e-3
    assert np.isfinite(dC.cpu().numpy()).all()
