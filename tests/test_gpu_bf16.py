"""GPU parity of the bfloat16-cost solve (sk_forward_bf16): an opt-in input
precision with no counterpart in the reference. The kernels widen every bf16
element exactly to fp32 and then run the fp32 arithmetic, so the contract is
the fp32 one against the fp64 oracle run on the same widened costs."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import ORACLE_RTOL, check_forward_parity, pot_tolerance

pytestmark = pytest.mark.gpu


def _t(x):
    return None if x is None else torch.from_numpy(np.asarray(x)).cuda()


def _problem(B, N, M, seed, masked):
    rng = np.random.default_rng(seed)
    x = rng.random((B, N, 3), dtype=np.float32)
    y = rng.random((B, M, 3), dtype=np.float32)
    C = ((x[:, :, None, :] - y[:, None, :, :]) ** 2).sum(-1).astype(np.float32)
    C /= C.max()
    Cb = torch.from_numpy(C).cuda().to(torch.bfloat16)
    ma = rng.random((B, N)) > 0.15 if masked else None
    mb = rng.random((B, M)) > 0.15 if masked else None
    return Cb, Cb.float().cpu().numpy(), ma, mb


@pytest.mark.parametrize("B,N,M,eps,tau,masked,iters,thr,ce", [
    (3, 200, 1024, 0.05, 1.0, True, 200, 1e-6, 10),   # two sweeps, masks, unbalanced
    (1, 256, 8192, 0.05, None, False, 40, 0.0, 10),   # the fused single-read iteration
    (2, 96, 8200, 0.1, None, False, 60, 1e-6, 1),     # M % 16 != 0: two sweeps at large M
    (1, 130, 1028, 0.2, 0.5, True, 80, 0.0, 10),      # odd row count, M % 8 != 0
])
def test_bf16_solve_matches_oracle_on_the_widened_costs(B, N, M, eps, tau, masked, iters,
                                                        thr, ce):
    from sinkhorn_b200.cuda.forward import sinkhorn_forward_cuda
    Cb, C32, ma, mb = _problem(B, N, M, seed=B * N + M, masked=masked)
    f, g, n, conv = sinkhorn_forward_cuda(Cb, None, None, eps, tau, tau, _t(ma), _t(mb),
                                          iters, thr, check_every=ce)
    assert f.dtype == torch.float32 and g.dtype == torch.float32
    check_forward_parity(f, g, n, conv, dict(
        C=C32, eps=eps, tau_a=tau, tau_b=tau, mask_a=ma, mask_b=mb, max_iters=iters,
        threshold=thr, check_every=ce))


def test_bf16_fused_solve_equals_the_fp32_solve_of_the_widened_costs():
    """On a fused shape the bf16 and fp32 kernels solve the same problem (the
    widened costs) with the same row arithmetic; the fp32 kernel's column
    fold reuses the row exponentials, the bf16 one (whose ring holds the
    narrow costs) takes its own, so the potentials agree to fp32 rounding."""
    from sinkhorn_b200.cuda.forward import sinkhorn_forward_cuda
    from sinkhorn_b200.cuda.solver import plan_query
    Cb, C32, _, _ = _problem(1, 300, 16384, seed=3, masked=False)
    Cf = torch.from_numpy(C32).cuda()
    assert plan_query(Cf)["forward_fused"]
    f1, g1, n1, _ = sinkhorn_forward_cuda(Cb, None, None, 0.05, None, None, None, None, 30, 0.0)
    f2, g2, n2, _ = sinkhorn_forward_cuda(Cf, None, None, 0.05, None, None, None, None, 30, 0.0)
    assert n1 == n2 == 30
    tol = pot_tolerance(0.05)
    torch.testing.assert_close(f1, f2, atol=tol, rtol=ORACLE_RTOL)
    torch.testing.assert_close(g1, g2, atol=tol, rtol=ORACLE_RTOL)


def test_bf16_layouts_without_a_4_wide_path_are_rejected():
    from sinkhorn_b200._lib import SinkhornCudaError
    from sinkhorn_b200.cuda.forward import sinkhorn_forward_cuda
    C = torch.rand(1, 64, 1030, device="cuda").to(torch.bfloat16)  # M % 4 != 0
    with pytest.raises(SinkhornCudaError):
        sinkhorn_forward_cuda(C, epsilon=0.1, max_iters=5)
    Ct = torch.rand(1, 512, 64, device="cuda").to(torch.bfloat16).transpose(1, 2)
    with pytest.raises(SinkhornCudaError):
        sinkhorn_forward_cuda(Ct, epsilon=0.1, max_iters=5)


def test_bf16_is_forward_only():
    from sinkhorn_b200 import sinkhorn
    C = torch.rand(1, 32, 32, device="cuda").to(torch.bfloat16).requires_grad_(True)
    with pytest.raises(TypeError):
        sinkhorn(C, epsilon=0.1, backend="cuda")
    with torch.no_grad():
        out = sinkhorn(C, epsilon=0.1, backend="cuda", max_iters=20)
    assert out.f.dtype == torch.float32
