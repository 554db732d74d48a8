"""Property tests of backend="cuda", the properties the reference's own suite
pins its solver with (tests/test_balanced.py, test_unbalanced.py,
test_numerical.py, test_gradients.py), restated against sinkhorn_b200's
public API on the GPU: convergence on easy problems, marginals, batch
independence, masks, the rho relaxation, numerical range, the plan's
structure, and gradients. Parity with the reference's exact outputs is in
the golden / oracle tests; these check behaviour."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _sinkhorn(*args, **kw):
    from sinkhorn_b200 import sinkhorn
    return sinkhorn(*args, backend="cuda", **kw)


def _rand(shape, seed, dist="rand"):
    gen = torch.Generator().manual_seed(seed)
    x = torch.rand(shape, generator=gen) if dist == "rand" else torch.randn(shape, generator=gen)
    return x.cuda()


def _marginals(out, C, eps, ma=None, mb=None):
    P = out.transport_plan(C, eps, ma, mb)
    return P, P.sum(-1), P.sum(-2)


def _identity_cost(B, n):
    C = torch.full((B, n, n), 10.0)
    C[:, torch.arange(n), torch.arange(n)] = 0.0
    return C.cuda()


def test_identity_cost_converges_and_concentrates_on_the_diagonal():
    C = _identity_cost(2, 16)
    out = _sinkhorn(C, epsilon=0.1, max_iters=100, threshold=1e-6)
    assert out.converged and out.n_iters < 100
    out2 = _sinkhorn(C, epsilon=0.01, max_iters=500)
    P = out2.transport_plan(C, 0.01)
    diag = torch.diagonal(P, dim1=-2, dim2=-1).sum(-1)
    assert (diag / P.sum((-2, -1)) > 0.8).all()
    assert torch.isfinite(P).all()


@pytest.mark.parametrize("N,M", [(48, 48), (40, 72)])
def test_balanced_marginals_match(N, M):
    C = _rand((3, N, M), 1)
    a = torch.softmax(_rand((3, N), 2, "randn"), -1)
    b = torch.softmax(_rand((3, M), 3, "randn"), -1)
    out = _sinkhorn(C, a, b, epsilon=0.1, max_iters=5000, threshold=1e-8, check_every=1)
    _, r, c = _marginals(out, C, 0.1)
    assert (r - a).abs().max().item() < 1e-4
    assert (c - b).abs().max().item() < 1e-4
    assert out.f.shape == (3, N) and out.g.shape == (3, M)


def test_default_marginals_are_uniform_and_plan_is_valid_at_small_eps():
    C = _rand((2, 30, 50), 4)
    small = _sinkhorn(C, epsilon=0.01, max_iters=200, threshold=1e-6)
    P = small.transport_plan(C, 0.01)
    assert (P >= 0).all() and torch.isfinite(P).all()
    assert torch.isfinite(small.f).all() and torch.isfinite(small.g).all()
    out = _sinkhorn(C, epsilon=0.1, max_iters=3000, threshold=1e-7)
    _, r, c = _marginals(out, C, 0.1)
    assert (r - 1.0 / 30).abs().max().item() < 1e-3 / 30
    assert (c - 1.0 / 50).abs().max().item() < 1e-3 / 50


def test_large_eps_converges_fast_and_faster_than_small_eps():
    C = _rand((2, 64, 64), 5)
    fast = _sinkhorn(C, epsilon=1.0, max_iters=1000, threshold=1e-6, check_every=1)
    slow = _sinkhorn(C, epsilon=0.05, max_iters=1000, threshold=1e-6, check_every=1)
    assert fast.converged and fast.n_iters < 30
    assert slow.n_iters > fast.n_iters


def test_batch_items_are_independent():
    """Each item of a batch solves like the item alone (a fixed number of
    iterations, since the reference's stopping test spans the batch)."""
    C = _rand((4, 50, 70), 6)
    a = torch.softmax(_rand((4, 50), 7, "randn"), -1)
    out = _sinkhorn(C, a, epsilon=0.1, tau_a=1.0, max_iters=80, threshold=0.0)
    for i in range(4):
        one = _sinkhorn(C[i:i + 1], a[i:i + 1], epsilon=0.1, tau_a=1.0, max_iters=80,
                        threshold=0.0)
        assert (one.f - out.f[i:i + 1]).abs().max().item() < 1e-5
        assert (one.g - out.g[i:i + 1]).abs().max().item() < 1e-5


def test_extreme_costs_and_sparse_marginals_keep_mass():
    C = _rand((2, 32, 32), 8) * 100.0
    a = torch.full((2, 32), 1e-6, device="cuda")
    a[:, 0] = 1.0
    a = a / a.sum(-1, keepdim=True)
    out = _sinkhorn(C, a, epsilon=1.0, max_iters=2000, threshold=1e-7)
    P = out.transport_plan(C, 1.0)
    assert torch.isfinite(P).all()
    assert (P.sum((-2, -1)) - 1.0).abs().max().item() < 1e-4


def test_cost_entries_of_plus_minus_100_stay_finite():
    C = (_rand((2, 40, 40), 9) * 200.0 - 100.0)
    out = _sinkhorn(C, epsilon=0.1, max_iters=200, threshold=1e-6)
    assert torch.isfinite(out.f).all() and torch.isfinite(out.g).all()
    assert torch.isfinite(out.transport_plan(C, 0.1)).all()


def test_unbalanced_relaxation():
    C = _rand((2, 40, 40), 10)
    a = torch.softmax(_rand((2, 40), 11, "randn"), -1)
    b = torch.softmax(_rand((2, 40), 12, "randn"), -1)
    bal = _sinkhorn(C, a, b, epsilon=0.1, tau_a=None, tau_b=None, max_iters=3000,
                    threshold=1e-8)
    _, r, c = _marginals(bal, C, 0.1)
    assert (r - a).abs().max().item() < 1e-3 and (c - b).abs().max().item() < 1e-3
    unb = _sinkhorn(C, a, b, epsilon=0.1, tau_a=1.0, tau_b=1.0, max_iters=3000, threshold=1e-7)
    assert unb.converged
    asym = _sinkhorn(C, a, b, epsilon=0.1, tau_a=0.1, tau_b=10.0, max_iters=3000,
                     threshold=1e-7)
    assert (asym.f - unb.f).abs().max().item() > 1e-3
    for tau in (0.1, 0.5, 1.0, 5.0, 10.0):
        o = _sinkhorn(C, a, b, epsilon=0.1, tau_a=tau, tau_b=tau, max_iters=500,
                      threshold=1e-6)
        assert torch.isfinite(o.f).all() and torch.isfinite(o.g).all()


def test_masked_entries_get_zero_potentials_and_no_mass():
    C = _rand((3, 40, 50), 13)
    ma = torch.ones(3, 40, dtype=torch.bool, device="cuda")
    mb = torch.ones(3, 50, dtype=torch.bool, device="cuda")
    ma[0, 30:] = False
    ma[2, :5] = False
    mb[1, 40:] = False
    mb[2, 10:20] = False
    out = _sinkhorn(C, epsilon=0.1, tau_a=1.0, tau_b=1.0, mask_a=ma, mask_b=mb,
                    max_iters=500, threshold=1e-6)
    assert (out.f[~ma] == 0).all() and (out.g[~mb] == 0).all()
    P = out.transport_plan(C, 0.1, ma, mb)
    assert P[~ma].abs().max().item() < 1e-10
    assert P.transpose(1, 2)[~mb].abs().max().item() < 1e-10


def test_variable_length_prefix_masks_produce_no_nan():
    gen = torch.Generator().manual_seed(14)
    B, N = 8, 128
    C = torch.randn(B, N, N, generator=gen).cuda()
    la = torch.randint(10, N + 1, (B,), generator=gen)
    ma = (torch.arange(N)[None, :] < la[:, None]).cuda()
    out = _sinkhorn(C, epsilon=0.1, tau_a=1.0, tau_b=1.0, mask_a=ma, mask_b=ma,
                    max_iters=200, threshold=1e-6)
    assert torch.isfinite(out.f).all() and torch.isfinite(out.g).all()


def test_delta_marginals_put_the_mass_on_the_cheap_entry():
    C = _rand((1, 16, 16), 15)
    C[0, 0, 0] = 0.0
    a = torch.zeros(1, 16, device="cuda")
    b = torch.zeros(1, 16, device="cuda")
    a[0, 0] = 1.0
    b[0, 0] = 1.0
    out = _sinkhorn(C, a, b, epsilon=0.05, max_iters=1000, threshold=1e-7)
    P = out.transport_plan(C, 0.05)
    assert P[0, 0, 0].item() > 0.9


def test_symmetric_problem_gives_potentials_of_equal_range():
    """A symmetric cost with uniform marginals: f and g are one potential up
    to the balanced problem's constant shift, so their ranges agree."""
    t = _rand((2, 40, 40), 16, "randn")
    C = (t + t.transpose(-2, -1)) / 2
    out = _sinkhorn(C, epsilon=0.1, max_iters=3000, threshold=1e-7, check_every=1)
    fr = out.f.amax(-1) - out.f.amin(-1)
    gr = out.g.amax(-1) - out.g.amin(-1)
    assert (fr - gr).abs().max().item() < 1e-3


def test_cost_grows_with_eps_and_dual_objective_increases():
    C = _rand((2, 32, 32), 17)
    costs = []
    for eps in (0.02, 0.1, 0.5):
        out = _sinkhorn(C, epsilon=eps, max_iters=3000, threshold=1e-7)
        costs.append(out.cost(C, eps))
    assert (costs[0] <= costs[1] + 1e-3).all() and (costs[1] <= costs[2] + 1e-3).all()

    def dual(it):
        # <f, a> + <g, b> - eps * sum(P) (compute_dual_objective, unbalanced.py:166-196)
        out = _sinkhorn(C, epsilon=0.1, max_iters=it, threshold=0.0)
        P = out.transport_plan(C, 0.1)
        return out.sinkhorn_divergence(C, 0.1) - 0.1 * P.sum((-2, -1))

    d1, d5, d50 = dual(1), dual(5), dual(50)
    assert (d5 >= d1 - 1e-6).all() and (d50 > d1).all()


def test_gradients_exist_are_finite_and_vanish_for_zero_upstream():
    from sinkhorn_b200 import sinkhorn_differentiable
    C0 = _rand((2, 24, 20), 18)
    for tau in (None, 1.0):
        C = C0.clone().requires_grad_(True)
        f, g = sinkhorn_differentiable(C, epsilon=0.5, tau_a=tau, tau_b=tau, max_iters=100,
                                       threshold=1e-6)
        (f.sum() + 2 * g.sum()).backward()
        gr = C.grad
        assert gr is not None and torch.isfinite(gr).all()
        assert 1e-10 < gr.norm().item() < 1e10
        C2 = C0.clone().requires_grad_(True)
        f2, g2 = sinkhorn_differentiable(C2, epsilon=0.5, tau_a=tau, tau_b=tau, max_iters=100,
                                         threshold=1e-6)
        (0.0 * f2.sum() + 0.0 * g2.sum()).backward()
        assert not C2.grad.any()


def test_gradient_matches_finite_differences():
    """fp32 stand-in for the reference's float64 gradcheck: the directional
    derivative of <f, w_f> + <g, w_g> along a random dC, against a centred
    difference (full-recompute backward)."""
    from sinkhorn_b200 import sinkhorn_differentiable
    C0 = _rand((1, 12, 10), 19)
    wf = _rand((1, 12), 20, "randn")
    wg = _rand((1, 10), 21, "randn")
    d = _rand((1, 12, 10), 22, "randn")
    kw = dict(epsilon=0.5, tau_a=1.0, tau_b=1.0, max_iters=200, threshold=0.0)

    def loss(C):
        f, g = sinkhorn_differentiable(C, **kw)
        return (f * wf).sum() + (g * wg).sum()

    C = C0.clone().requires_grad_(True)
    loss(C).backward()
    analytic = (C.grad * d).sum().item()
    h = 1e-2
    with torch.no_grad():
        numeric = (loss(C0 + h * d) - loss(C0 - h * d)).item() / (2 * h)
    assert abs(analytic - numeric) <= 2e-2 * max(1.0, abs(numeric))


def test_balanced_and_unbalanced_gradients_differ():
    from sinkhorn_b200 import sinkhorn_differentiable
    C0 = _rand((1, 16, 16), 23)
    wf = _rand((1, 16), 24, "randn")
    wg = _rand((1, 16), 25, "randn")
    grads = []
    for tau in (None, 0.5):
        C = C0.clone().requires_grad_(True)
        f, g = sinkhorn_differentiable(C, epsilon=0.5, tau_a=tau, tau_b=tau, max_iters=200,
                                       threshold=1e-6)
        ((f * wf).sum() + (g * wg).sum()).backward()
        grads.append(C.grad)
    assert (grads[0] - grads[1]).abs().max().item() > 1e-4
