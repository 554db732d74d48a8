"""Parity at the benchmarked sizes, against the oracle on the same inputs.

The problems are generated exactly as bench.py generates its workloads:

* the headline solve: B=1, N=M=16384 (C = 1 GiB), squared distances of
  x, y ~ U[0,1]^3 divided by max(C), uniform marginals, eps=0.05,
  threshold 0 (exactly 100 iterations), on the fused single-read iteration
  (74 row chunks merged per iteration); and the same problem run to
  convergence at threshold 1e-6, checked every 10 iterations (the
  ms-to-converge measurement);
* the masked, unbalanced batch: B=64, N=M=1024, C ~ N(0,1), prefix masks of
  lengths ~ U{256..1024}, softmax marginals over the valid entries, eps=0.1,
  tau_a=tau_b=1, max_iters=200, threshold 1e-6;
* the differentiable problem: B=16, N=M=2048, C = squared distances of
  x, y ~ N(0, I_16) scaled to mean 1, eps=1, loss = sum(P * C), dC through
  the truncated (grad_iters=10) and the full-recompute (grad_iters=0)
  backward.

Tolerances are the parity contract's: f, g within 1e-4 * max(1, eps)
absolute (plus 2e-6 relative against the oracle), identical iteration counts
(``iterations_agree``), dC within 1e-3 relative. The headline and the
differentiable problem use the oracle's fp32 build (the reference's own
arithmetic type) to keep the CPU side to tens of seconds on the host cores;
the masked batch uses the fp64 oracle.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import check_forward_parity
from oracle import oracle as O

pytestmark = [pytest.mark.gpu, pytest.mark.slow]


def _headline_cost(n=16384, seed=1234):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.rand(n, 3, device="cuda", generator=g)
    y = torch.rand(n, 3, device="cuda", generator=g)
    C = torch.cdist(x, y).pow_(2)
    C.div_(C.max())
    return C.unsqueeze(0).contiguous()


@pytest.fixture(scope="module")
def headline():
    C = _headline_cost()
    return C, C.cpu().numpy()


def test_headline_solve_matches_oracle(headline):
    """The benchmarked solve: 100 iterations of the fused single-read
    iteration (k_fused_iter + the 74-chunk merge of k_col_finish)."""
    from sinkhorn_b200.cuda.forward import sinkhorn_forward_cuda
    from sinkhorn_b200.cuda.solver import plan_query
    C, Cn = headline
    q = plan_query(C)
    assert q["forward_fused"] and q["chunks"] >= 8
    f, g, n, conv = sinkhorn_forward_cuda(C, None, None, 0.05, None, None, None, None, 100,
                                          0.0)
    assert (n, conv) == (100, False)
    check_forward_parity(f, g, n, conv, dict(C=Cn, eps=0.05, max_iters=100, threshold=0.0,
                                             check_every=10), precision="f32")
    # after the g-update every column of the plan sums to b = 1/M (exactly in
    # exact arithmetic): a size-independent property of the solve
    col = torch.exp((f[:, :, None] + g[:, None, :] - C) / 0.05).sum(dim=1)
    assert float((col * 16384 - 1).abs().max()) < 1e-4


def test_headline_converges_like_the_oracle(headline):
    """The same problem at threshold 1e-6, checked every 10 iterations: the
    iteration count at convergence and the potentials there."""
    from sinkhorn_b200.cuda.forward import sinkhorn_forward_cuda
    C, Cn = headline
    f, g, n, conv = sinkhorn_forward_cuda(C, None, None, 0.05, None, None, None, None, 500,
                                          1e-6, check_every=10)
    assert conv
    check_forward_parity(f, g, n, conv, dict(C=Cn, eps=0.05, max_iters=500, threshold=1e-6,
                                             check_every=10), precision="f32")


def _masked_batch():
    gen = torch.Generator().manual_seed(0)
    B, N, M = 64, 1024, 1024
    C = torch.randn(B, N, M, generator=gen)
    la = torch.randint(256, N + 1, (B,), generator=gen)
    lb = torch.randint(256, M + 1, (B,), generator=gen)
    mask_a = torch.arange(N)[None, :] < la[:, None]
    mask_b = torch.arange(M)[None, :] < lb[:, None]
    a = torch.softmax(torch.randn(B, N, generator=gen).masked_fill(~mask_a, float("-inf")), -1)
    b = torch.softmax(torch.randn(B, M, generator=gen).masked_fill(~mask_b, float("-inf")), -1)
    return C, a, b, mask_a, mask_b


def test_masked_unbalanced_batch_matches_oracle():
    """B=64, N=M=1024, prefix masks, tau=1, 200 iterations (the single-read
    k_rows_fused iteration with its per-item chunks)."""
    from sinkhorn_b200.cuda.forward import sinkhorn_forward_cuda
    from sinkhorn_b200.cuda.solver import plan_query
    C, a, b, ma, mb = _masked_batch()
    Cd = C.cuda()
    assert plan_query(Cd)["forward_fused"]
    f, g, n, conv = sinkhorn_forward_cuda(Cd, a.cuda(), b.cuda(), 0.1, 1.0, 1.0, ma.cuda(),
                                          mb.cuda(), 200, 1e-6)
    check_forward_parity(f, g, n, conv, dict(
        C=C.numpy(), a=a.numpy(), b=b.numpy(), eps=0.1, tau_a=1.0, tau_b=1.0,
        mask_a=ma.numpy(), mask_b=mb.numpy(), max_iters=200, threshold=1e-6,
        check_every=10))
    assert not f.cpu()[~ma].any() and not g.cpu()[~mb].any()


def _diff_cost():
    gen = torch.Generator().manual_seed(0)
    B, N, M, D = 16, 2048, 2048, 16
    x = torch.randn(B, N, D, generator=gen)
    y = torch.randn(B, M, D, generator=gen)
    C = torch.cdist(x, y).pow(2)
    return C / C.mean()


@pytest.fixture(scope="module")
def diff_problem():
    C = _diff_cost()
    Cn = C.numpy()
    # the oracle's forward (threshold 1e-6, check every 10: the cuda default)
    fs, gs, n, conv = O.forward(Cn, None, None, 1.0, None, None, None, None, 100, 1e-6, 10,
                                precision="f32")
    return C, Cn, (fs, gs, n, conv)


@pytest.mark.parametrize("grad_iters", [10, 0])
def test_differentiable_problem_dC_matches_oracle(diff_problem, grad_iters):
    """loss = sum(P * C) through sinkhorn_differentiable: forward potentials
    against the oracle, then dC = the loss's direct term P (1 - C/eps) plus
    the oracle's backward of the upstream gradients sum_j P C / eps and
    sum_i P C / eps."""
    from sinkhorn_b200.autograd import sinkhorn_differentiable
    from sinkhorn_b200.cuda.forward import sinkhorn_forward_cuda
    C, Cn, fwd = diff_problem
    eps = 1.0
    Cg = C.cuda().requires_grad_(True)
    # the forward the differentiable call runs (max_iters 100, threshold
    # 1e-6, checked every 10): here |f| ~ 8, so the threshold is about one
    # fp32 ulp of f and the stop is decided by rounding (iterations_agree);
    # the potentials are compared at the count the build reports
    f1, g1, n1, c1 = sinkhorn_forward_cuda(Cg.detach(), None, None, eps, None, None, None,
                                           None, 100, 1e-6, check_every=10)
    check_forward_parity(f1, g1, n1, c1, dict(C=Cn, eps=eps, max_iters=100, threshold=1e-6,
                                              check_every=10), oracle_out=fwd,
                         precision="f32")
    f, g = sinkhorn_differentiable(Cg, epsilon=eps, grad_iters=grad_iters)
    assert torch.equal(f.detach(), f1) and torch.equal(g.detach(), g1)
    fs, gs = f1.cpu().numpy(), g1.cpu().numpy()
    P = torch.exp((f[:, :, None] + g[:, None, :] - Cg) / eps)
    (P * Cg).sum().backward()
    dC = Cg.grad.cpu().numpy()

    f64, g64 = fs.astype(np.float64), gs.astype(np.float64)
    Pn = np.exp((f64[:, :, None] + g64[:, None, :] - Cn) / eps)
    PC = Pn * Cn
    grad_f = PC.sum(axis=2) / eps
    grad_g = PC.sum(axis=1) / eps
    direct = Pn - PC / eps
    del PC
    # the oracle's backward from the same (f*, g*) and upstream gradients
    edC, _, _, K = O.backward(Cn, None, None, eps, None, None, None, None, 100, 1e-6,
                              grad_iters, fs, gs, grad_f.astype(np.float32),
                              grad_g.astype(np.float32), precision="f32")
    ref = direct + edC
    err = float(np.abs(dC - ref).max() / np.abs(ref).max())
    assert err <= 1e-3, err
