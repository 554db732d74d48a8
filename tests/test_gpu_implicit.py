"""GPU parity of the implicit-differentiation adjoint (sinkhorn_b200.implicit_diff,
sk_implicit_* in the C ABI) against the reference's golden vectors and the
oracle's restatement of src/sinkhorn/pytorch/implicit_diff.py."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden_names, implicit_fp32_budget, load_golden
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def cu(x, dtype=torch.float32):
    if x is None:
        return None
    t = torch.from_numpy(np.ascontiguousarray(x))
    return t.to(torch.bool if t.dtype == torch.bool else dtype).cuda()


def npy(t):
    return t.detach().cpu().double().numpy()


def test_matvec_modes_dense_plan_match_reference():
    from sinkhorn_b200 import implicit_diff as I
    d = load_golden("imp_matvec")
    P, vf, vg = cu(d["P"]), cu(d["v_f"]), cu(d["v_g"])
    ma, mb = cu(d["mask_a"]), cu(d["mask_b"])
    outs = {
        "schur": I.schur_complement_matvec(vf, vg, P, d["rho_a"], d["rho_b"], d["reg"]),
        "vjp": I.vjp_sinkhorn(vf, vg, P, d["eps"], d["rho_a"], d["rho_b"], ma, mb),
        "jvp": I.jvp_sinkhorn(vf, vg, P, d["eps"], d["rho_a"], d["rho_b"], ma, mb),
    }
    for mode, (of, og) in outs.items():
        for out, ref in ((of, d[mode + "_f"]), (og, d[mode + "_g"])):
            np.testing.assert_allclose(npy(out), ref, rtol=0,
                                       atol=2e-6 * max(1.0, np.abs(ref).max()), err_msg=mode)


@pytest.mark.parametrize("masked", [False, True])
@pytest.mark.parametrize("shape", [(2, 37, 29), (1, 256, 200), (3, 96, 128)])
def test_plan_matvec_pfree_matches_oracle(shape, masked):
    from sinkhorn_b200 import _tensors as T
    B, N, M = shape
    rng = np.random.default_rng(N + M + masked)
    C = rng.random((B, N, M), dtype=np.float32)
    f = (0.1 * rng.standard_normal((B, N))).astype(np.float32)
    g = (0.1 * rng.standard_normal((B, M))).astype(np.float32)
    x = rng.standard_normal((B, M)).astype(np.float32)
    y = rng.standard_normal((B, N)).astype(np.float32)
    ma = rng.random((B, N)) > 0.25 if masked else None
    mb = rng.random((B, M)) > 0.25 if masked else None
    eps = 0.3
    P = O.transport_plan(C, f, g, eps, ma, mb)
    tC, tf, tg, tx, ty = cu(C), cu(f), cu(g), cu(x), cu(y)
    tma = None if ma is None else cu(ma.astype(np.uint8), torch.uint8)
    tmb = None if mb is None else cu(mb.astype(np.uint8), torch.uint8)
    outs = [torch.empty(B, N, device="cuda"), torch.empty(B, M, device="cuda"),
            torch.empty(B, N, device="cuda"), torch.empty(B, M, device="cuda")]
    lib = T.lib()
    ws = T.workspace(lib.sk_plan_matvec_workspace_bytes(B, N, M), tC.device)
    rc = lib.sk_plan_matvec(*T.cost_args(tC), tf.data_ptr(), tg.data_ptr(), eps, T.ptr(tma),
                            T.ptr(tmb), None, tx.data_ptr(), ty.data_ptr(),
                            *[o.data_ptr() for o in outs], ws.data_ptr(), ws.numel(),
                            T.stream_of(tC.device))
    T.check(rc, "sk_plan_matvec")
    want = [np.einsum("bnm,bm->bn", P, x), np.einsum("bnm,bn->bm", P, y), P.sum(2), P.sum(1)]
    for out, ref in zip(outs, want):
        np.testing.assert_allclose(npy(out), ref, rtol=0, atol=2e-5 * np.abs(ref).max())


def test_cg_solve_dense_short_matches_reference():
    from sinkhorn_b200 import implicit_diff as I
    d = load_golden("imp_cg_short")
    for it in (1, 2, 3):
        xf, xg, n = I.cg_solve(cu(d["rhs_f"]), cu(d["rhs_g"]), cu(d["P"]), 0.0, 0.0, it, 1e-5)
        assert n == d[f"n{it}"]
        for out, r32, r64 in ((xf, d[f"x_f{it}"], d[f"x64_f{it}"]),
                              (xg, d[f"x_g{it}"], d[f"x64_g{it}"])):
            tol = 4 * np.abs(r32 - r64).max() + 1e-5 * np.abs(r64).max()
            np.testing.assert_allclose(npy(out), r64, rtol=0, atol=tol)


@pytest.mark.parametrize("name", golden_names("imp_grad_"))
def test_implicit_gradient_matches_reference(name):
    """P-free implicit_gradient against the reference's fp64 run, inside the
    error budget the reference's own fp32 run shows on the same input; the
    batch items the reference's CG drives to NaN/inf are non-finite here too."""
    from sinkhorn_b200 import implicit_diff as I
    d = load_golden(name)
    dC, da, db = I.implicit_gradient(cu(d["C"]), cu(d["f"]), cu(d["g"]), cu(d["grad_f"]),
                                     cu(d["grad_g"]), d["eps"], d["tau_a"], d["tau_b"],
                                     cu(d.get("mask_a")), cu(d.get("mask_b")),
                                     d["cg_max_iters"], d["cg_tol"])
    for out, key in ((dC, "dC"), (da, "da"), (db, "db")):
        o, ref64 = npy(out), d[key + "64"]
        B = ref64.shape[0]
        for b in range(B):
            assert np.isfinite(o[b]).all() == np.isfinite(ref64[b]).all(), (key, b)
        fin = np.isfinite(ref64) & np.isfinite(d[key])
        if fin.any():
            np.testing.assert_allclose(o[fin], ref64[fin], rtol=0,
                                       atol=implicit_fp32_budget(d, key), err_msg=key)


def test_implicit_gradient_iterations_of_converging_case():
    """The on-device stopping test: the reference stops after 11 (fp64) / 16
    (fp32) iterations on this case; an fp32 solver with double dots lands in
    that range."""
    from sinkhorn_b200 import implicit_diff as I
    d = load_golden("imp_grad_balanced_conv")
    P = I.compute_transport_plan(cu(d["C"]), cu(d["f"]), cu(d["g"]), d["eps"])
    _, _, n = I.cg_solve(cu(d["grad_f"]), cu(d["grad_g"]), P, 0.0, 0.0, d["cg_max_iters"],
                         d["cg_tol"])
    assert d["n64"] <= n <= d["n32"] + 4, (n, d["n64"], d["n32"])


@pytest.mark.parametrize("masked", [False, True])
def test_implicit_gradient_pfree_matches_dense_and_oracle(masked):
    """A mid-size case: the P-free path, the dense-plan path and the fp64 oracle
    agree after a few CG iterations (before the reference's CG amplifies
    rounding)."""
    from sinkhorn_b200 import implicit_diff as I
    from sinkhorn_b200.cuda.forward import sinkhorn_forward_cuda
    gen = torch.Generator().manual_seed(5 + masked)
    B, N, M, eps = 2, 300, 260, 0.5
    C = torch.rand(B, N, M, generator=gen)
    ma = (torch.rand(B, N, generator=gen) > 0.2) if masked else None
    mb = (torch.rand(B, M, generator=gen) > 0.2) if masked else None
    gf = torch.randn(B, N, generator=gen)
    gg = torch.randn(B, M, generator=gen)
    tC, tma, tmb = C.cuda(), cu(ma), cu(mb)
    f, g, _, _ = sinkhorn_forward_cuda(tC, None, None, eps, 1.0, 1.0, tma, tmb, 500, 1e-7)
    iters = 3
    dC, da, db = I.implicit_gradient(tC, f, g, gf.cuda(), gg.cuda(), eps, 1.0, 1.0, tma, tmb,
                                     iters, 1e-5)
    rdC, rda, rdb, rn = O.implicit_gradient(C, f.cpu(), g.cpu(), gf, gg, eps, 1.0, 1.0, ma,
                                            mb, iters, 1e-5)
    assert rn == iters
    for out, ref in ((dC, rdC), (da, rda), (db, rdb)):
        np.testing.assert_allclose(npy(out), ref, rtol=0, atol=5e-4 * np.abs(ref).max())
    P = I.compute_transport_plan(tC, f, g, eps, tma, tmb)
    rho = eps / (eps + 1.0)
    lf, lg, n = I.cg_solve(gf.cuda(), gg.cuda(), P, rho, rho, iters, 1e-5)
    assert n == iters
    np.testing.assert_allclose(npy(lf) * eps, npy(da), rtol=0, atol=1e-4 * np.abs(rda).max())
    np.testing.assert_allclose(npy(lg) * eps, npy(db), rtol=0, atol=1e-4 * np.abs(rdb).max())


def test_zero_iterations_and_strided_cost():
    from sinkhorn_b200 import implicit_diff as I
    gen = torch.Generator().manual_seed(9)
    base = torch.rand(2, 40, 70, generator=gen).cuda()
    C = base[:, :, 3:67]  # rows not 16-byte aligned: the scalar band path
    f = torch.zeros(2, 40, device="cuda")
    g = torch.zeros(2, 64, device="cuda")
    gf = torch.randn(2, 40, generator=gen).cuda()
    gg = torch.randn(2, 64, generator=gen).cuda()
    dC, da, db = I.implicit_gradient(C, f, g, gf, gg, 1.0, cg_max_iters=0)
    assert not dC.any() and not da.any() and not db.any()
    dC, da, db = I.implicit_gradient(C, f, g, gf, gg, 1.0, cg_max_iters=3)
    rdC, rda, rdb, _ = O.implicit_gradient(C.cpu(), f.cpu(), g.cpu(), gf.cpu(), gg.cpu(), 1.0,
                                           cg_max_iters=3)
    for out, ref in ((dC, rdC), (da, rda), (db, rdb)):
        np.testing.assert_allclose(npy(out), ref, rtol=0, atol=2e-4 * np.abs(ref).max())


def test_large_problem_properties():
    """N = M = 4096: the dC of the P-free path equals -(1/eps) P (lf + lg) with
    the path's own lambda (grad_a / eps), and one CG step equals the closed
    form x1 = (r.r / p.Ap) rhs computed from the Schur matvec."""
    from sinkhorn_b200 import implicit_diff as I
    gen = torch.Generator(device="cuda").manual_seed(3)
    B, N, M, eps = 1, 4096, 4096, 0.1
    C = torch.rand(B, N, M, device="cuda", generator=gen)
    f = 0.01 * torch.randn(B, N, device="cuda", generator=gen)
    g = 0.01 * torch.randn(B, M, device="cuda", generator=gen)
    gf = torch.randn(B, N, device="cuda", generator=gen)
    gg = torch.randn(B, M, device="cuda", generator=gen)
    dC, da, db = I.implicit_gradient(C, f, g, gf, gg, eps, 2.0, 2.0, cg_max_iters=1)
    P = I.compute_transport_plan(C, f, g, eps)
    rho = eps / (eps + 2.0)
    Af, Ag = I.schur_complement_matvec(gf, gg, P, rho, rho, 1e-5)
    rr = (gf.double() ** 2).sum() + (gg.double() ** 2).sum()
    pap = (gf.double() * Af.double()).sum() + (gg.double() * Ag.double()).sum()
    alpha = rr / pap
    torch.testing.assert_close(da.double(), eps * alpha * gf.double(), rtol=1e-4, atol=1e-6)
    torch.testing.assert_close(db.double(), eps * alpha * gg.double(), rtol=1e-4, atol=1e-6)
    want = -(1.0 / eps) * P * (da / eps)[:, :, None] - (1.0 / eps) * P * (db / eps)[:, None, :]
    torch.testing.assert_close(dC, want, rtol=2e-5, atol=1e-6 * want.abs().max().item())


def test_errors():
    from sinkhorn_b200 import implicit_diff as I
    from sinkhorn_b200._lib import SinkhornCudaError
    C = torch.rand(1, 8, 8)
    with pytest.raises(RuntimeError, match="CUDA"):
        I.implicit_gradient(C, torch.zeros(1, 8), torch.zeros(1, 8), torch.zeros(1, 8),
                            torch.zeros(1, 8), 0.1)
    Cg = C.cuda()
    with pytest.raises(ValueError, match="shape"):
        I.implicit_gradient(Cg, torch.zeros(1, 7, device="cuda"), torch.zeros(1, 8,
                            device="cuda"), torch.zeros(1, 8, device="cuda"),
                            torch.zeros(1, 8, device="cuda"), 0.1)
    with pytest.raises(SinkhornCudaError, match="max_iters"):
        I.cg_solve(torch.zeros(1, 8, device="cuda"), torch.zeros(1, 8, device="cuda"), Cg,
                   max_iters=-1)
