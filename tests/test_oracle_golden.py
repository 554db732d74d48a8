"""Pin the C oracle against golden vectors produced by the reference itself.

Runs on CPU. Every fixture in tests/golden was written by
tests/golden/make_golden.py from the reference package (PyTorch path, and the
Triton path under the Triton interpreter for the ``tri_*`` cases).
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import (forward_golden_names, golden_names, implicit_fp32_budget,
                      iterations_agree, load_golden, pot_tolerance)
from oracle import oracle as O


def residual_f64(d):
    """fp64 residual max(|f_k - f_{k-1}|, |g_k - g_{k-1}|) of iteration k."""
    def at(k):
        args = (d["C"], d.get("a"), d.get("b"), d["eps"], d["tau_a"], d["tau_b"],
                d.get("mask_a"), d.get("mask_b"))
        f1, g1, _, _ = O.forward(*args, k, 0.0, 1)
        f0, g0, _, _ = O.forward(*args, k - 1, 0.0, 1)
        return max(np.abs(f1 - f0).max(), np.abs(g1 - g0).max())
    return at

FWD_CASES = forward_golden_names()


@pytest.mark.parametrize("name", FWD_CASES)
@pytest.mark.parametrize("precision", ["f64", "f32"])
def test_forward_matches_reference(name, precision):
    d = load_golden(name)
    f, g, n, conv = O.forward(d["C"], d.get("a"), d.get("b"), d["eps"], d["tau_a"],
                              d["tau_b"], d.get("mask_a"), d.get("mask_b"),
                              d["max_iters"], d["threshold"], d["check_every"],
                              precision=precision)
    tol = pot_tolerance(d["eps"])
    assert iterations_agree(n, conv, d, residual_f64(d)), (n, conv, d["n_iters"])
    np.testing.assert_allclose(f, d["f"], rtol=0, atol=tol)
    np.testing.assert_allclose(g, d["g"], rtol=0, atol=tol)


@pytest.mark.parametrize("name", [n for n in FWD_CASES if "P" in load_golden(n)])
def test_plan_and_cost_match_reference(name):
    d = load_golden(name)
    # plan from the reference's own potentials: isolates the plan arithmetic
    P = O.transport_plan(d["C"], d["f"], d["g"], d["eps"], d.get("mask_a"),
                         d.get("mask_b"))
    np.testing.assert_allclose(P, d["P"], rtol=2e-5, atol=1e-7)
    c = O.cost(d["C"], d["f"], d["g"], d["eps"])
    np.testing.assert_allclose(c, d["cost"], rtol=2e-5, atol=1e-6)


@pytest.mark.parametrize("name", [n for n in FWD_CASES if "marginal_err" in load_golden(n)])
def test_marginal_error_matches_reference(name):
    from conftest import marginal_err_tolerance
    d = load_golden(name)
    e = O.marginal_error(d["C"], d["f"], d["g"], d["me_a"], d["me_b"], d["eps"],
                         d.get("mask_a"), d.get("mask_b"))
    tol = marginal_err_tolerance(d["me_a"], d["me_b"])
    assert abs(e - float(d["marginal_err"])) <= tol + 1e-3 * float(d["marginal_err"]), \
        (e, float(d["marginal_err"]), tol)


@pytest.mark.parametrize("name", golden_names("warm_"))
@pytest.mark.parametrize("precision", ["f64", "f32"])
def test_iters_from_init_matches_reference(name, precision):
    """The warm iteration of _sinkhorn_iters_from_init (autograd.py:134-178):
    raw C, masks on the final potentials only."""
    d = load_golden(name)
    f, g = O.iters_from_init(d["C"], d["a"], d["b"], d["eps"], d["tau_a"], d["tau_b"],
                             d.get("mask_a"), d.get("mask_b"), d["f_init"], d["g_init"],
                             d["n_iters"], precision=precision)
    tol = pot_tolerance(d["eps"])
    np.testing.assert_allclose(f, d["f"], rtol=0, atol=tol)
    np.testing.assert_allclose(g, d["g"], rtol=0, atol=tol)


def test_forward_warm_start_matches_reference_without_masks():
    """Without masks the forward iteration and the reference's warm iteration
    are the same map, so the oracle's forward started from (f_init, g_init)
    (threshold 0) must land on the reference's _sinkhorn_iters_from_init."""
    d = load_golden("warm_init_balanced")
    f, g, n, conv = O.forward(d["C"], d["a"], d["b"], d["eps"], d["tau_a"], d["tau_b"],
                              None, None, d["n_iters"], 0.0, 1, f_init=d["f_init"],
                              g_init=d["g_init"])
    assert n == d["n_iters"] and not conv
    tol = pot_tolerance(d["eps"])
    np.testing.assert_allclose(f, d["f"], rtol=0, atol=tol)
    np.testing.assert_allclose(g, d["g"], rtol=0, atol=tol)


def test_forward_warm_start_residual_counts_from_the_start_potentials():
    """A forward started from (f_init, g_init) measures its first residual
    against them: one iteration with check_every=1 and a threshold above the
    true first step converges; below it does not."""
    d = load_golden("warm_init_masked_unbal")
    args = (d["C"], d["a"], d["b"], d["eps"], d["tau_a"], d["tau_b"], d["mask_a"],
            d["mask_b"])
    f1, g1, _, _ = O.forward(*args, 1, 0.0, 1, f_init=d["f_init"], g_init=d["g_init"])
    step = max(np.abs(f1 - d["f_init"]).max(), np.abs(g1 - d["g_init"]).max())
    _, _, n, conv = O.forward(*args, 5, step * 1.001, 1, f_init=d["f_init"],
                              g_init=d["g_init"])
    assert (n, conv) == (1, True)
    _, _, n, conv = O.forward(*args, 1, step * 0.999, 1, f_init=d["f_init"],
                              g_init=d["g_init"])
    assert (n, conv) == (1, False)


def test_lse_row_col_match_triton():
    d = load_golden("tri_lse")
    np.testing.assert_allclose(O.lse_row(d["C"], d["g"], d["eps"]), d["row"], atol=2e-6)
    np.testing.assert_allclose(O.lse_col(d["C"], d["f"], d["eps"]), d["col"], atol=2e-6)
    # the empty row / column give exactly 0 (lse_kernel.py:130, :206)
    assert d["row"][1, 2] == 0.0 and d["col"][0, 4] == 0.0


def test_jvp_matches_triton():
    d = load_golden("tri_jvp")
    of, og = O.jvp(d["P"], d["v_f"], d["v_g"], d["rho_a"], d["rho_b"])
    np.testing.assert_allclose(of, d["out_f"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(og, d["out_g"], rtol=1e-5, atol=1e-6)


def _bwd(d, precision="f64"):
    """dC of the loss the fixture used, from the oracle."""
    dC, da, db, K = O.backward(d["C"], d.get("a"), d.get("b"), d["eps"], d["tau_a"],
                               d["tau_b"], d.get("mask_a"), d.get("mask_b"),
                               d["max_iters"], d["threshold"], d["grad_iters"],
                               f_star=d["f"], g_star=d["g"], grad_f=d["grad_f"],
                               grad_g=d["grad_g"], precision=precision)
    if d["loss_kind"] == "plan_cost":
        # loss = sum(P*C) with P = exp((f+g-C)/eps): direct term P - C*P/eps
        P = O.transport_plan(d["C"], d["f"], d["g"], d["eps"])
        dC = dC + P - d["C"] * P / d["eps"]
    return dC, da, db, K


@pytest.mark.parametrize("name", golden_names("bwd_"))
def test_backward_matches_reference(name):
    d = load_golden(name)
    dC, da, db, K = _bwd(d)
    ref = d["dC"]
    scale = np.abs(ref).max()
    assert np.abs(dC - ref).max() <= 1e-3 * scale, np.abs(dC - ref).max() / scale
    if "da" in d:
        np.testing.assert_allclose(da, d["da"], rtol=1e-3, atol=1e-3 * np.abs(d["da"]).max())
        np.testing.assert_allclose(db, d["db"], rtol=1e-3, atol=1e-3 * np.abs(d["db"]).max())


def test_upstream_gradients_of_plan_cost():
    """grad_f/grad_g that the reference fed into SinkhornFunction.backward for
    loss = sum(P*C) are sum_j C P / eps and sum_i C P / eps."""
    d = load_golden("bwd_cfg4_small_k10")
    P = O.transport_plan(d["C"], d["f"], d["g"], d["eps"])
    w = d["C"] * P / d["eps"]
    np.testing.assert_allclose(w.sum(2), d["grad_f"], rtol=1e-4, atol=1e-6)
    np.testing.assert_allclose(w.sum(1), d["grad_g"], rtol=1e-4, atol=1e-6)


# ---------------------------------------------------------------------------
# Implicit-differentiation adjoint (sinkhorn.pytorch.implicit_diff)

def test_implicit_matvecs_match_reference():
    d = load_golden("imp_matvec")
    for mode in ("schur", "vjp", "jvp"):
        of, og = O.implicit_matvec(d["v_f"], d["v_g"], d["P"], d["rho_a"], d["rho_b"],
                                   d["reg"], mode, d["mask_a"], d["mask_b"])
        for out, ref in ((of, d[mode + "_f"]), (og, d[mode + "_g"])):
            np.testing.assert_allclose(out, ref, rtol=0,
                                       atol=2e-6 * max(1.0, np.abs(ref).max()))


def test_cg_solve_short_matches_reference():
    d = load_golden("imp_cg_short")
    for it in (1, 2, 3):
        xf, xg, n = O.cg_solve(d["rhs_f"], d["rhs_g"], d["P"], 0.0, 0.0, it, 1e-5)
        assert n == d[f"n{it}"]
        for out, ref in ((xf, d[f"x64_f{it}"]), (xg, d[f"x64_g{it}"])):
            np.testing.assert_allclose(out, ref, rtol=1e-9, atol=1e-9 * np.abs(ref).max())
        xf, xg, _ = O.cg_solve(d["rhs_f"], d["rhs_g"], d["P"], 0.0, 0.0, it, 1e-5,
                               precision="f32")
        for out, ref in ((xf, d[f"x_f{it}"]), (xg, d[f"x_g{it}"])):
            np.testing.assert_allclose(out, ref, rtol=0, atol=1e-4 * np.abs(ref).max())


@pytest.mark.parametrize("name", golden_names("imp_grad_"))
def test_implicit_gradient_matches_reference(name):
    d = load_golden(name)
    args = (d["C"], d["f"], d["g"], d["grad_f"], d["grad_g"], d["eps"], d["tau_a"],
            d["tau_b"], d.get("mask_a"), d.get("mask_b"), d["cg_max_iters"], d["cg_tol"])
    dC, da, db, n = O.implicit_gradient(*args)
    assert n == d["n64"]
    for out, key in ((dC, "dC"), (da, "da"), (db, "db")):
        ref = d[key + "64"]
        fin = np.isfinite(ref)
        assert (np.isfinite(out) == fin).all(), key
        if fin.any():
            np.testing.assert_allclose(out[fin], ref[fin], rtol=0,
                                       atol=1e-7 * np.abs(ref[fin]).max(), err_msg=key)
    # fp32 restatement against the reference's fp32 run, inside the fp32 budget
    dC, da, db, _ = O.implicit_gradient(*args, precision="f32")
    for out, key in ((dC, "dC"), (da, "da"), (db, "db")):
        ref32, fin = d[key], np.isfinite(d[key + "64"]) & np.isfinite(d[key])
        assert (np.isfinite(out) == np.isfinite(ref32)).all(), key
        if fin.any():
            tol = implicit_fp32_budget(d, key)
            np.testing.assert_allclose(out[fin], ref32[fin], rtol=0, atol=2 * tol,
                                       err_msg=key)
