"""Generate the golden fixtures in tests/golden/*.npz by running the reference.

This script imports the reference package (vv137/sinkhorn) from a source
checkout and runs it on seeded inputs:

* the PyTorch path (``sinkhorn.pytorch.unbalanced.sinkhorn_unbalanced``,
  convergence checked every iteration) on CPU;
* the Triton path (``sinkhorn.triton``: ``sinkhorn_forward_triton``,
  ``lse_row``, ``lse_col``, ``jvp_triton``; convergence checked every 10
  iterations) under ``TRITON_INTERPRET=1`` for tiny shapes;
* ``SinkhornOutput.transport_plan`` / ``.cost`` and
  ``sinkhorn.pytorch.balanced.compute_marginal_error``;
* ``sinkhorn_differentiable`` (truncated and full-recompute backward);
* ``sinkhorn.pytorch.implicit_diff`` (Schur / JVP / VJP matvecs, ``cg_solve``,
  ``implicit_gradient``) in fp32 and, as the fp32 error budget, fp64.

Usage (from the repository root):

    python tests/golden/make_golden.py --reference-src /root/reference/src

The fixtures are committed; the tests never import the reference.
"""

from __future__ import annotations

import argparse
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-src", default="/root/reference/src")
    ap.add_argument("--only", default=None, help="comma-separated case names")
    args = ap.parse_args()
    # The Triton interpreter must be selected before triton is imported.
    os.environ.setdefault("TRITON_INTERPRET", "1")
    sys.path.insert(0, args.reference_src)

    import numpy as np
    import torch

    from sinkhorn.autograd import sinkhorn_differentiable
    from sinkhorn.pytorch.balanced import compute_marginal_error
    from sinkhorn.pytorch.unbalanced import sinkhorn_unbalanced
    from sinkhorn.sinkhorn import SinkhornOutput
    from sinkhorn.triton.forward import sinkhorn_forward_triton
    from sinkhorn.triton.jvp_kernel import jvp_triton
    from sinkhorn.triton.lse_kernel import lse_col, lse_row

    torch.set_num_threads(min(8, os.cpu_count() or 1))
    only = set(args.only.split(",")) if args.only else None
    out_cases = {}

    def want(name):
        return only is None or name in only

    def t2n(x):
        if x is None:
            return None
        return x.detach().cpu().numpy()

    def save(name, **arrays):
        path = os.path.join(HERE, name + ".npz")
        clean = {k: v for k, v in arrays.items() if v is not None}
        np.savez_compressed(path, **clean)
        out_cases[name] = path
        print(f"wrote {path}")

    def sqdist(x, y):
        return ((x[:, :, None, :] - y[:, None, :, :]) ** 2).sum(-1)

    # ------------------------------------------------------------------
    # Forward, PyTorch path (check every iteration)
    def fwd_case(name, C, a, b, eps, tau_a, tau_b, mask_a, mask_b, iters, thr,
                 plan=False):
        f, g, n, conv = sinkhorn_unbalanced(C, a, b, eps, tau_a, tau_b, mask_a, mask_b,
                                            iters, thr)
        extra = {}
        if plan:
            out = SinkhornOutput(f=f, g=g, n_iters=n, converged=conv)
            extra["P"] = t2n(out.transport_plan(C, eps, mask_a, mask_b))
            extra["cost"] = t2n(out.cost(C, eps))
            # compute_marginal_error needs explicit marginals: the given ones,
            # else uniform over the valid entries (the solver's default)
            def marg(x, mask, n_):
                if x is not None:
                    return x
                if mask is None:
                    return torch.full((C.shape[0], n_), 1.0 / n_)
                m = mask.float()
                return m / m.sum(-1, keepdim=True).clamp(min=1.0)
            me_a = marg(a, mask_a, C.shape[1])
            me_b = marg(b, mask_b, C.shape[2])
            extra["me_a"] = t2n(me_a)
            extra["me_b"] = t2n(me_b)
            extra["marginal_err"] = t2n(compute_marginal_error(C, f, g, me_a, me_b, eps,
                                                               mask_a, mask_b))
        save(name, C=t2n(C), a=t2n(a), b=t2n(b), mask_a=t2n(mask_a), mask_b=t2n(mask_b),
             eps=eps, tau_a=np.nan if tau_a is None else tau_a,
             tau_b=np.nan if tau_b is None else tau_b, max_iters=iters, threshold=thr,
             check_every=1, f=t2n(f), g=t2n(g), n_iters=n, converged=conv, **extra)

    gen = torch.Generator().manual_seed(0)
    if want("cfg1"):
        # B=8, N=M=64, C ~ N(0,1), softmax marginals, eps=0.1, balanced
        C = torch.randn(8, 64, 64, generator=gen)
        a = torch.softmax(torch.randn(8, 64, generator=gen), -1)
        b = torch.softmax(torch.randn(8, 64, generator=gen), -1)
        fwd_case("cfg1", C, a, b, 0.1, None, None, None, None, 100, 1e-6)

    if want("cfg2_n256"):
        gen = torch.Generator().manual_seed(1)
        x = torch.rand(1, 256, 3, generator=gen)
        y = torch.rand(1, 256, 3, generator=gen)
        C = sqdist(x, y)
        C = C / C.max()
        fwd_case("cfg2_n256", C, None, None, 0.05, None, None, None, None, 100, 0.0,
                 plan=True)

    if want("cfg3_small"):
        gen = torch.Generator().manual_seed(2)
        B, N = 4, 96
        C = torch.randn(B, N, N, generator=gen)
        la = torch.randint(24, N + 1, (B,), generator=gen)
        lb = torch.randint(24, N + 1, (B,), generator=gen)
        ar = torch.arange(N)
        mask_a = ar[None, :] < la[:, None]
        mask_b = ar[None, :] < lb[:, None]
        za = torch.randn(B, N, generator=gen).masked_fill(~mask_a, float("-inf"))
        zb = torch.randn(B, N, generator=gen).masked_fill(~mask_b, float("-inf"))
        a = torch.softmax(za, -1)
        b = torch.softmax(zb, -1)
        fwd_case("cfg3_small", C, a, b, 0.1, 1.0, 1.0, mask_a, mask_b, 200, 1e-6,
                 plan=True)

    if want("rect_odd"):
        gen = torch.Generator().manual_seed(3)
        C = torch.randn(3, 17, 33, generator=gen).abs()
        fwd_case("rect_odd", C, None, None, 0.1, 0.5, None, None, None, 150, 1e-6,
                 plan=True)

    if want("identity_conv"):
        C = torch.ones(2, 8, 8) * 10
        for i in range(8):
            C[:, i, i] = 0.0
        a = torch.ones(2, 8) / 8
        b = torch.ones(2, 8) / 8
        fwd_case("identity_conv", C, a, b, 0.1, None, None, None, None, 100, 1e-6)

    if want("mask_edge"):
        gen = torch.Generator().manual_seed(4)
        B, N, M = 3, 20, 20
        C = torch.randn(B, N, M, generator=gen)
        mask_a = torch.rand(B, N, generator=gen) > 0.3
        mask_b = torch.rand(B, M, generator=gen) > 0.3
        mask_b[1, :] = False          # item 1: every column masked
        mask_a[2, 5] = False          # item 2: a masked row ...
        mask_b[2, 7] = False          # ... and a masked column
        fwd_case("mask_edge", C, None, None, 0.1, 2.0, None, mask_a, mask_b, 60, 1e-6,
                 plan=True)

    if want("sparse_marg"):
        gen = torch.Generator().manual_seed(5)
        a = torch.zeros(2, 16)
        a[:, :4] = 0.25
        b = torch.zeros(2, 16)
        b[:, :4] = 0.25
        C = torch.randn(2, 16, 16, generator=gen).abs()
        fwd_case("sparse_marg", C, a, b, 0.1, None, None, None, None, 100, 1e-6)

    if want("large_range"):
        C = torch.zeros(2, 64, 64)
        C[:, 0, 0] = -100
        C[:, -1, -1] = 100
        fwd_case("large_range", C, None, None, 1.0, None, None, None, None, 100, 1e-6)

    if want("unbal_conv"):
        gen = torch.Generator().manual_seed(6)
        C = torch.randn(2, 24, 20, generator=gen).abs()
        a = torch.softmax(torch.randn(2, 24, generator=gen), -1)
        b = torch.softmax(torch.randn(2, 20, generator=gen), -1)
        fwd_case("unbal_conv", C, a, b, 0.5, 1.0, 1.0, None, None, 300, 1e-6)

    # ------------------------------------------------------------------
    # Triton path under the interpreter (check every 10 iterations)
    def tri_case(name, C, a, b, eps, tau_a, tau_b, mask_a, mask_b, iters, thr):
        f, g, n, conv = sinkhorn_forward_triton(C, a, b, eps, tau_a, tau_b, mask_a,
                                                mask_b, iters, thr)
        save(name, C=t2n(C), a=t2n(a), b=t2n(b), mask_a=t2n(mask_a), mask_b=t2n(mask_b),
             eps=eps, tau_a=np.nan if tau_a is None else tau_a,
             tau_b=np.nan if tau_b is None else tau_b, max_iters=iters, threshold=thr,
             check_every=10, f=t2n(f), g=t2n(g), n_iters=n, converged=conv)

    if want("tri_identity_conv"):
        C = torch.ones(2, 8, 8) * 10
        for i in range(8):
            C[:, i, i] = 0.0
        tri_case("tri_identity_conv", C, None, None, 0.1, None, None, None, None, 100,
                 1e-6)

    if want("tri_masked_unbal"):
        gen = torch.Generator().manual_seed(7)
        C = torch.randn(2, 12, 12, generator=gen)
        mask_a = torch.ones(2, 12, dtype=torch.bool)
        mask_a[0, 9:] = False
        mask_a[1, 3] = False
        mask_b = torch.ones(2, 12, dtype=torch.bool)
        mask_b[0, :2] = False
        mask_b[1, 10:] = False
        tri_case("tri_masked_unbal", C, None, None, 0.2, 1.0, 0.5, mask_a, mask_b, 40,
                 1e-6)

    if want("tri_rect"):
        gen = torch.Generator().manual_seed(8)
        C = torch.randn(2, 9, 13, generator=gen).abs()
        a = torch.softmax(torch.randn(2, 9, generator=gen), -1)
        b = torch.softmax(torch.randn(2, 13, generator=gen), -1)
        tri_case("tri_rect", C, a, b, 0.1, None, None, None, None, 30, 1e-6)

    if want("tri_lse"):
        gen = torch.Generator().manual_seed(9)
        C = torch.randn(2, 7, 13, generator=gen)
        C[1, 2, :] = float("inf")     # an empty row: softmin 0
        C[0, :, 4] = float("inf")     # an empty column: softmin 0
        g = torch.randn(2, 13, generator=gen)
        f = torch.randn(2, 7, generator=gen)
        save("tri_lse", C=t2n(C), g=t2n(g), f=t2n(f), eps=0.1,
             row=t2n(lse_row(C, g, 0.1)), col=t2n(lse_col(C, f, 0.1)))

    if want("tri_jvp"):
        gen = torch.Generator().manual_seed(10)
        P = torch.rand(2, 6, 9, generator=gen)
        P[1, 4, :] = 0.0              # a zero row: clamp at 1e-38
        v_f = torch.randn(2, 6, generator=gen)
        v_g = torch.randn(2, 9, generator=gen)
        of, og = jvp_triton(v_f, v_g, P, 0.2, 0.0)
        save("tri_jvp", P=t2n(P), v_f=t2n(v_f), v_g=t2n(v_g), rho_a=0.2, rho_b=0.0,
             out_f=t2n(of), out_g=t2n(og))

    # ------------------------------------------------------------------
    # Backward (sinkhorn_differentiable, PyTorch forward inside)
    def bwd_case(name, C0, a0, b0, eps, tau_a, tau_b, mask_a, mask_b, iters, thr,
                 grad_iters, loss_kind, wgen=None, grad_ab=False):
        C = C0.clone().requires_grad_(True)
        a = None if a0 is None else a0.clone().requires_grad_(grad_ab)
        b = None if b0 is None else b0.clone().requires_grad_(grad_ab)
        f, g = sinkhorn_differentiable(C, a, b, eps, tau_a, tau_b, mask_a, mask_b, iters,
                                       thr, grad_iters, backend="pytorch")
        up = {}
        f.register_hook(lambda t: up.__setitem__("grad_f", t.detach().clone()))
        g.register_hook(lambda t: up.__setitem__("grad_g", t.detach().clone()))
        if loss_kind == "plan_cost":
            out = SinkhornOutput(f=f, g=g, n_iters=iters, converged=True)
            P = out.transport_plan(C, eps)
            loss = (P * C).sum()
        else:
            wf = torch.randn(f.shape, generator=wgen)
            wg = torch.randn(g.shape, generator=wgen)
            loss = (f * wf).sum() + (g * wg).sum()
        loss.backward()
        save(name, C=t2n(C0), a=t2n(a0), b=t2n(b0), mask_a=t2n(mask_a),
             mask_b=t2n(mask_b), eps=eps, tau_a=np.nan if tau_a is None else tau_a,
             tau_b=np.nan if tau_b is None else tau_b, max_iters=iters, threshold=thr,
             grad_iters=grad_iters, loss_kind=loss_kind, f=t2n(f), g=t2n(g),
             grad_f=t2n(up["grad_f"]), grad_g=t2n(up["grad_g"]), dC=t2n(C.grad),
             da=t2n(a.grad) if grad_ab else None, db=t2n(b.grad) if grad_ab else None)

    for gi in (10, 0):
        name = f"bwd_cfg4_small_k{gi}"
        if want(name):
            gen = torch.Generator().manual_seed(11)
            x = torch.randn(2, 32, 16, generator=gen)
            y = torch.randn(2, 32, 16, generator=gen)
            C = sqdist(x, y)
            C = C / C.mean()
            bwd_case(name, C, None, None, 1.0, None, None, None, None, 100, 1e-6, gi,
                     "plan_cost")

    if want("bwd_trunc_masked_unbal"):
        gen = torch.Generator().manual_seed(12)
        C = torch.randn(2, 16, 16, generator=gen)
        mask_a = torch.ones(2, 16, dtype=torch.bool)
        mask_a[0, 12:] = False
        mask_b = torch.ones(2, 16, dtype=torch.bool)
        mask_b[1, :3] = False
        a = torch.softmax(torch.randn(2, 16, generator=gen), -1)
        b = torch.softmax(torch.randn(2, 16, generator=gen), -1)
        bwd_case("bwd_trunc_masked_unbal", C, a, b, 0.3, 1.0, 1.0, mask_a, mask_b, 50,
                 1e-6, 5, "weights", wgen=gen, grad_ab=True)

    if want("bwd_full_unbal"):
        gen = torch.Generator().manual_seed(13)
        C = torch.randn(2, 12, 10, generator=gen).abs()
        a = torch.softmax(torch.randn(2, 12, generator=gen), -1)
        b = torch.softmax(torch.randn(2, 10, generator=gen), -1)
        bwd_case("bwd_full_unbal", C, a, b, 0.5, 1.0, None, None, None, 80, 1e-6, 0,
                 "weights", wgen=gen, grad_ab=True)

    # ------------------------------------------------------------------
    # Implicit-differentiation adjoint (sinkhorn.pytorch.implicit_diff), run in
    # the reference's fp32 and, for the error budget of fp32 arithmetic, fp64.
    from sinkhorn.pytorch import implicit_diff as imp

    def rho(eps, tau):
        return 0.0 if tau is None else eps / (eps + tau)

    def imp_problem(seed, B, N, M, eps, tau_a, tau_b, masked):
        gen = torch.Generator().manual_seed(seed)
        C = torch.rand(B, N, M, generator=gen)
        ma = mb = None
        if masked:
            ma = torch.rand(B, N, generator=gen) > 0.2
            mb = torch.rand(B, M, generator=gen) > 0.2
        f, g, _, _ = sinkhorn_unbalanced(C, None, None, eps, tau_a, tau_b, ma, mb, 1000, 1e-7)
        gf = torch.randn(B, N, generator=gen)
        gg = torch.randn(B, M, generator=gen)
        if ma is not None:
            gf = gf * ma
        if mb is not None:
            gg = gg * mb
        return C, f, g, ma, mb, gf, gg

    if want("imp_matvec"):
        C, f, g, ma, mb, vf, vg = imp_problem(3, 2, 24, 20, 1.0, 1.0, 0.5, True)
        P = imp.compute_transport_plan(C, f, g, 1.0, ma, mb)
        ra, rb = 0.2, 0.3
        sf, sg = imp.schur_complement_matvec(vf, vg, P, ra, rb, 1e-5)
        vjf, vjg = imp.vjp_sinkhorn(vf, vg, P, 1.0, ra, rb, ma, mb)
        jf, jg = imp.jvp_sinkhorn(vf, vg, P, 1.0, ra, rb, ma, mb)
        save("imp_matvec", C=t2n(C), f=t2n(f), g=t2n(g), mask_a=t2n(ma), mask_b=t2n(mb),
             eps=1.0, P=t2n(P), v_f=t2n(vf), v_g=t2n(vg), rho_a=ra, rho_b=rb, reg=1e-5,
             schur_f=t2n(sf), schur_g=t2n(sg), vjp_f=t2n(vjf), vjp_g=t2n(vjg), jvp_f=t2n(jf),
             jvp_g=t2n(jg))

    if want("imp_cg_short"):
        C, f, g, ma, mb, gf, gg = imp_problem(1, 2, 24, 20, 1.0, None, None, False)
        P = imp.compute_transport_plan(C, f, g, 1.0)
        arrays = {}
        for it in (1, 2, 3):
            xf, xg, n = imp.cg_solve(gf, gg, P, 0.0, 0.0, it, 1e-5)
            xf64, xg64, _ = imp.cg_solve(gf.double(), gg.double(), P.double(), 0.0, 0.0, it,
                                         1e-5)
            arrays.update({f"x_f{it}": t2n(xf), f"x_g{it}": t2n(xg), f"x64_f{it}": t2n(xf64),
                           f"x64_g{it}": t2n(xg64), f"n{it}": n})
        save("imp_cg_short", C=t2n(C), f=t2n(f), g=t2n(g), eps=1.0, P=t2n(P), rhs_f=t2n(gf),
             rhs_g=t2n(gg), **arrays)

    def imp_grad_case(name, seed, B, N, M, eps, tau_a, tau_b, masked, iters, tol):
        C, f, g, ma, mb, gf, gg = imp_problem(seed, B, N, M, eps, tau_a, tau_b, masked)
        out32 = imp.implicit_gradient(C, f, g, gf, gg, eps, tau_a, tau_b, ma, mb, iters, tol)
        out64 = imp.implicit_gradient(C.double(), f.double(), g.double(), gf.double(),
                                      gg.double(), eps, tau_a, tau_b, ma, mb, iters, tol)
        P = imp.compute_transport_plan(C, f, g, eps, ma, mb)
        _, _, n32 = imp.cg_solve(gf, gg, P, rho(eps, tau_a), rho(eps, tau_b), iters, tol)
        _, _, n64 = imp.cg_solve(gf.double(), gg.double(), P.double(), rho(eps, tau_a),
                                 rho(eps, tau_b), iters, tol)
        # fp32 noise floor: the reference's CG rerun on plans that differ from P
        # by at most one rounding (relative 2^-23), each result against fp64
        spread = {"dC": 0.0, "da": 0.0, "db": 0.0}
        for k in range(64):
            gk = torch.Generator().manual_seed(100 + k)
            Pk = P * (1 + (2 * torch.rand(P.shape, generator=gk) - 1) * 2.0 ** -23)
            lf, lg, _ = imp.cg_solve(gf, gg, Pk, rho(eps, tau_a), rho(eps, tau_b), iters, tol)
            runs = {"dC": -(1.0 / eps) * Pk * (lf.unsqueeze(-1) + lg.unsqueeze(-2)),
                    "da": eps * lf, "db": eps * lg}
            for key, ref64 in zip(("dC", "da", "db"), out64):
                r64, rk = t2n(ref64), t2n(runs[key]).astype(np.float64)
                fin = np.isfinite(r64) & np.isfinite(rk)
                if fin.any():
                    spread[key] = max(spread[key], float(np.abs(rk[fin] - r64[fin]).max()))
        save(name, C=t2n(C), f=t2n(f), g=t2n(g), mask_a=t2n(ma), mask_b=t2n(mb), eps=eps,
             tau_a=np.nan if tau_a is None else tau_a,
             tau_b=np.nan if tau_b is None else tau_b, grad_f=t2n(gf), grad_g=t2n(gg),
             cg_max_iters=iters, cg_tol=tol, dC=t2n(out32[0]), da=t2n(out32[1]),
             db=t2n(out32[2]), dC64=t2n(out64[0]), da64=t2n(out64[1]), db64=t2n(out64[2]),
             n32=n32, n64=n64, dC_spread=spread["dC"], da_spread=spread["da"],
             db_spread=spread["db"])

    if want("imp_grad_masked_unbal"):
        imp_grad_case("imp_grad_masked_unbal", 3, 2, 24, 20, 1.0, 1.0, 1.0, True, 50, 1e-5)
    if want("imp_grad_unbal"):
        imp_grad_case("imp_grad_unbal", 8, 1, 64, 48, 0.2, 0.05, 0.05, False, 50, 1e-5)
    if want("imp_grad_balanced_conv"):
        imp_grad_case("imp_grad_balanced_conv", 1, 1, 64, 64, 1.0, None, None, False, 200,
                      1e-6)
    if want("imp_grad_diverge"):
        imp_grad_case("imp_grad_diverge", 1, 2, 16, 12, 0.5, None, None, False, 50, 1e-5)

    # ------------------------------------------------------------------
    # Warm start: _sinkhorn_iters_from_init (autograd.py:134-178) from random
    # non-zero potentials, with and without masks / relaxation
    from sinkhorn.autograd import _sinkhorn_iters_from_init

    def warm_case(name, seed, B, N, M, eps, tau, masked, n_iters):
        gen = torch.Generator().manual_seed(seed)
        C = torch.rand(B, N, M, generator=gen)
        mask_a = mask_b = None
        if masked:
            mask_a = torch.rand(B, N, generator=gen) > 0.25
            mask_b = torch.rand(B, M, generator=gen) > 0.25
            a = mask_a.float() * torch.rand(B, N, generator=gen)
            b = mask_b.float() * torch.rand(B, M, generator=gen)
        else:
            a = torch.rand(B, N, generator=gen) + 0.1
            b = torch.rand(B, M, generator=gen) + 0.1
        a = a / a.sum(-1, keepdim=True)
        b = b / b.sum(-1, keepdim=True)
        f_init = 0.3 * torch.randn(B, N, generator=gen)
        g_init = 0.3 * torch.randn(B, M, generator=gen)
        with torch.no_grad():
            f, g = _sinkhorn_iters_from_init(C, a, b, eps, tau, tau, mask_a, mask_b,
                                             f_init, g_init, n_iters)
        save(name, C=t2n(C), a=t2n(a), b=t2n(b), mask_a=t2n(mask_a), mask_b=t2n(mask_b),
             eps=eps, tau_a=np.nan if tau is None else tau,
             tau_b=np.nan if tau is None else tau, f_init=t2n(f_init), g_init=t2n(g_init),
             n_iters=n_iters, f=t2n(f), g=t2n(g))

    if want("warm_init_balanced"):
        warm_case("warm_init_balanced", 21, 2, 48, 64, 0.1, None, False, 30)
    if want("warm_init_masked_unbal"):
        warm_case("warm_init_masked_unbal", 22, 3, 40, 56, 0.2, 1.0, True, 25)

    print(f"{len(out_cases)} fixtures written")


if __name__ == "__main__":
    main()
