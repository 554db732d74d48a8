"""The backward's single-read reverse step (k_bwd_rows, shapes with
512 <= M <= 4096 and contiguous rows; above 2048 a thread owns two column
groups of each row) against the fp64 oracle, and against the two-pass reverse
sweep the same call takes on a strided view of the same C.

Cases cover every threads-per-column variant (M = 512: 4, M <= 1024: 2,
M <= 2048: 1), row counts that leave a ragged last stage and chunk, masks
(full mode gives masked entries no term and masked rows / columns no
adjoint), unbalanced marginals, and both the truncated (grad_iters = 5) and
the full recompute (grad_iters = 0) modes. Tolerance: dC and the marginals'
gradients within 1e-3 of the oracle's largest magnitude, the parity contract
of the reference's autograd. Also the backward of rows 2048 < M < 8192,
whose recompute runs on the single-read step's one-CTA units."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _t(x):
    return None if x is None else torch.from_numpy(np.asarray(x)).cuda()


def _rel_err(x, ref):
    return float(np.abs(x - ref).max() / max(np.abs(ref).max(), 1e-30))


def _problem(B, N, M, masked, seed):
    rng = np.random.default_rng(seed)
    C = rng.random((B, N, M)).astype(np.float32)
    a = rng.random((B, N)).astype(np.float32) + 0.2
    b = rng.random((B, M)).astype(np.float32) + 0.2
    ma = mb = None
    if masked:
        ma = rng.random((B, N)) > 0.2
        mb = rng.random((B, M)) > 0.2
        a = np.where(ma, a, 0.0).astype(np.float32)
        b = np.where(mb, b, 0.0).astype(np.float32)
    a /= a.sum(axis=1, keepdims=True)
    b /= b.sum(axis=1, keepdims=True)
    gf = rng.standard_normal((B, N)).astype(np.float32)
    gg = rng.standard_normal((B, M)).astype(np.float32)
    return C, a, b, ma, mb, gf, gg


def _cuda_backward(C, a, b, eps, tau, ma, mb, iters, thr, grad_iters, fs, gs, gf, gg):
    from sinkhorn_b200.autograd import sinkhorn_backward_cuda
    dC, dla, dlb, K = sinkhorn_backward_cuda(C, _t(a), _t(b), eps, tau, tau, _t(ma), _t(mb),
                                             iters, thr, grad_iters, _t(fs), _t(gs), _t(gf),
                                             _t(gg), need_dlog=True)
    da = np.where(a > 0, dla.cpu().numpy() / np.maximum(a, 1e-38), 0.0)
    db = np.where(b > 0, dlb.cpu().numpy() / np.maximum(b, 1e-38), 0.0)
    return dC.cpu().numpy(), da, db, K


@pytest.mark.parametrize("shape", [(2, 130, 512), (3, 97, 1024), (2, 75, 640),
                                   (2, 201, 2048), (1, 37, 1500)])
@pytest.mark.parametrize("masked", [False, True])
@pytest.mark.parametrize("tau", [None, 1.0])
@pytest.mark.parametrize("grad_iters", [5, 0])
def test_single_read_reverse_matches_oracle(shape, masked, tau, grad_iters):
    B, N, M = shape
    C, a, b, ma, mb, gf, gg = _problem(B, N, M, masked, seed=N + M + (7 if masked else 0))
    eps, iters, thr = 0.1, 30, 0.0
    fs, gs, _, _ = O.forward(C, a, b, eps, tau, tau, ma, mb, iters, thr, 10)
    fs, gs = fs.astype(np.float32), gs.astype(np.float32)
    edC, eda, edb, eK = O.backward(C, a, b, eps, tau, tau, ma, mb, iters, thr, grad_iters,
                                   fs, gs, gf, gg)
    dC, da, db, K = _cuda_backward(_t(C), a, b, eps, tau, ma, mb, iters, thr, grad_iters,
                                   fs, gs, gf, gg)
    assert K == eK
    assert np.isfinite(dC).all()
    assert _rel_err(dC, edC) <= 1e-3
    assert _rel_err(da, eda) <= 1e-3
    assert _rel_err(db, edb) <= 1e-3


@pytest.mark.parametrize("shape", [(2, 96, 1024), (2, 65, 2048), (2, 70, 4096), (1, 44, 2052)])
def test_single_read_reverse_matches_two_pass(shape):
    """The same problem through the single-read reverse step (contiguous C)
    and through the band passes (C seen through a column-strided view, which
    the bulk copies cannot stage): the same vectors, summed in another order."""
    B, N, M = shape
    C, a, b, ma, mb, gf, gg = _problem(B, N, M, True, seed=3)
    eps, iters, thr = 0.05, 20, 0.0
    fs, gs, _, _ = O.forward(C, a, b, eps, None, None, ma, mb, iters, thr, 10)
    fs, gs = fs.astype(np.float32), gs.astype(np.float32)
    Cd = _t(C)
    Cs = torch.empty(B, M, N, device="cuda").transpose(1, 2)
    Cs.copy_(Cd)
    assert Cs.stride(2) != 1
    for gi in (4, 0):
        one = _cuda_backward(Cd, a, b, eps, None, ma, mb, iters, thr, gi, fs, gs, gf, gg)
        two = _cuda_backward(Cs, a, b, eps, None, ma, mb, iters, thr, gi, fs, gs, gf, gg)
        assert one[3] == two[3]
        for x, y in zip(one[:3], two[:3]):
            assert _rel_err(x, y) <= 1e-4


@pytest.mark.parametrize("shape", [(2, 100, 4096), (1, 90, 3000)])
@pytest.mark.parametrize("masked", [False, True])
@pytest.mark.parametrize("grad_iters", [5, 0])
def test_backward_with_one_cta_recompute_matches_oracle(shape, masked, grad_iters):
    """Rows of 2048 < M < 8192: the recompute runs on the single-read step's
    one-CTA units (the whole row in one CTA), the reverse steps on the band
    passes; dC and the marginals' gradients against the fp64 oracle."""
    B, N, M = shape
    C, a, b, ma, mb, gf, gg = _problem(B, N, M, masked, seed=N + M + (5 if masked else 0))
    eps, tau, iters, thr = 0.1, 1.0, 30, 0.0
    fs, gs, _, _ = O.forward(C, a, b, eps, tau, tau, ma, mb, iters, thr, 10)
    fs, gs = fs.astype(np.float32), gs.astype(np.float32)
    edC, eda, edb, eK = O.backward(C, a, b, eps, tau, tau, ma, mb, iters, thr, grad_iters,
                                   fs, gs, gf, gg)
    dC, da, db, K = _cuda_backward(_t(C), a, b, eps, tau, ma, mb, iters, thr, grad_iters,
                                   fs, gs, gf, gg)
    assert K == eK
    assert np.isfinite(dC).all()
    assert _rel_err(dC, edC) <= 1e-3
    assert _rel_err(da, eda) <= 1e-3
    assert _rel_err(db, edb) <= 1e-3
