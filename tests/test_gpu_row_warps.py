"""GPU parity of k_row_warps (the single-read iteration with a warp per row,
which sk_forward runs for 512 < M <= 1024) against the fp64 oracle, on the
cases its numerics branch on:

* the warp's pivot moves whenever a row's largest term lies more than 2^8
  above it (every solve's first rows; a warm start far from the solution);
* a column whose pivoted sum ends below 2^-72 of the pivot is summed again
  directly from C (a column every row of the chunk reaches only through
  terms far below its largest ones);
* masked rows inside the valid range, items with no valid row or column,
  and ragged column spans that end inside a float4.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import check_forward_parity

pytestmark = pytest.mark.gpu


def _t(x):
    return None if x is None else torch.from_numpy(np.asarray(x)).cuda()


def _sqdist(B, N, M, seed):
    rng = np.random.default_rng(seed)
    x = rng.random((B, N, 3), dtype=np.float32)
    y = rng.random((B, M, 3), dtype=np.float32)
    C = ((x[:, :, None, :] - y[:, None, :, :]) ** 2).sum(-1)
    return (C / C.max()).astype(np.float32), rng


def _run(C, eps, tau=None, ma=None, mb=None, iters=50, thr=0.0, ce=10, f_init=None,
         g_init=None):
    from sinkhorn_b200.cuda.forward import sinkhorn_forward_cuda
    from sinkhorn_b200.cuda.solver import plan_query
    Ct = _t(C)
    q = plan_query(Ct)
    assert q["forward_fused"], q  # sk_forward runs k_row_warps for these shapes
    f, g, n, conv = sinkhorn_forward_cuda(Ct, None, None, eps, tau, tau, _t(ma), _t(mb),
                                          iters, thr, check_every=ce, f_init=_t(f_init),
                                          g_init=_t(g_init))
    check_forward_parity(f, g, n, conv, dict(
        C=C, eps=eps, tau_a=tau, tau_b=tau, mask_a=ma, mask_b=mb, max_iters=iters,
        threshold=thr, check_every=ce, f_init=f_init, g_init=g_init))
    return f, g


@pytest.mark.parametrize("B,N,M,eps,tau", [
    (3, 1600, 1000, 0.05, None),  # one warp per row, spans ending inside a float4
    (2, 2400, 1020, 0.1, 1.0),    # every float4 slot of a lane, the last one ragged
    (10, 480, 516, 0.02, None),   # a short last slot
])
def test_random_masks_and_unbalanced(B, N, M, eps, tau):
    C, rng = _sqdist(B, N, M, seed=N + M)
    ma = rng.random((B, N)) > 0.2
    mb = rng.random((B, M)) > 0.2
    _run(C, eps, tau, ma, mb, iters=60, thr=1e-6, ce=10)


def test_warm_start_far_from_the_solution():
    """f_init = 40 and g_init = -40: the first iteration's row bounds lie
    far from the previous iteration's, so the pivot moves and rescales."""
    C, _ = _sqdist(2, 2400, 1024, seed=5)
    f0 = np.full((2, 2400), 40.0, dtype=np.float32)
    g0 = np.full((2, 1024), -40.0, dtype=np.float32)
    _run(C, 0.05, iters=30, f_init=f0, g_init=g0)


def test_starved_columns_are_summed_directly():
    """Columns 3 and 700 cost 60 more than the rest at eps = 0.05: against
    the pivot of the rows' largest terms their sums are below 2^-1000, far
    under the 2^-72 that sends a column to the direct sum."""
    C, _ = _sqdist(1, 4800, 1024, seed=9)
    C[:, :, 3] += 60.0
    C[:, :, 700] += 60.0
    f, g = _run(C, 0.05, iters=20)
    assert np.isfinite(g.cpu().numpy()).all()


def test_empty_items_and_masked_rows():
    C, rng = _sqdist(16, 300, 768, seed=11)
    ma = np.ones((16, 300), dtype=bool)
    mb = np.ones((16, 768), dtype=bool)
    ma[1] = False            # an item with no valid row
    mb[2] = False            # an item with no valid column
    ma[3, 100:180] = False   # masked rows inside the valid range
    mb[3, 5:9] = False
    f, g = _run(C, 0.1, None, ma, mb, iters=40)
    assert not f.cpu().numpy()[~ma].any() and not g.cpu().numpy()[~mb].any()
