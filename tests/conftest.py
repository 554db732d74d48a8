"""pytest configuration: the ``gpu`` marker and shared fixture helpers."""

from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200 / sm_100a)")
    config.addinivalue_line("markers", "slow: long-running case")


def load_golden(name: str) -> dict:
    """Load tests/golden/<name>.npz into a dict of numpy arrays / python scalars."""
    with np.load(os.path.join(GOLDEN, name + ".npz")) as z:
        out = {}
        for k in z.files:
            v = z[k]
            out[k] = v.item() if v.shape == () else v
    for k in ("tau_a", "tau_b"):
        if k in out and isinstance(out[k], float) and np.isnan(out[k]):
            out[k] = None
    return out


def golden_names(prefix: str = "") -> list[str]:
    return sorted(f[:-4] for f in os.listdir(GOLDEN)
                  if f.endswith(".npz") and f.startswith(prefix))


# fixtures that are not forward solves from zero potentials
NON_FORWARD = ("bwd_", "tri_lse", "tri_jvp", "imp_", "warm_")


def forward_golden_names() -> list[str]:
    """Fixtures of the reference's forward solve (sinkhorn_unbalanced or
    sinkhorn_forward_triton from f = g = 0)."""
    return [n for n in golden_names() if not n.startswith(NON_FORWARD)]


def pot_tolerance(eps: float) -> float:
    """Potential tolerance of the parity contract: 1e-4 * max(1, eps) absolute."""
    return 1e-4 * max(1.0, eps)


# Relative slack used only against the fp64 oracle: an fp32 solver (the
# reference's included) sits up to ~16 fp32 ulps from exact arithmetic once
# |f| is large (e.g. |f| ~ 100 in the large-range case), which the absolute
# 1e-4 bound alone does not allow for. Comparisons with the reference's own
# golden vectors use the absolute bound only.
ORACLE_RTOL = 2e-6


def fp32_noise(*arrays) -> float:
    """Four fp32 ulps at the largest potential magnitude: the resolution of a
    max|f_new - f| residual computed in fp32."""
    mx = max(float(np.abs(np.asarray(x)).max()) for x in arrays if np.size(x))
    return 4.0 * float(np.spacing(np.float32(max(mx, 1e-30))))


def iterations_agree(n, conv, ref: dict, residual_at) -> bool:
    """Convergence-count parity.

    Counts must be identical, unless the exact (fp64) residual at the
    reference's stopping iteration lies within the fp32 resolution of the
    threshold -- then any fp32 implementation may stop a few checks earlier or
    later, and a difference of up to 3 check periods is accepted.
    ``residual_at(k)`` returns the fp64 residual of iteration k.

    A threshold at or below that resolution itself (4 fp32 ulps of the
    largest potential) cannot be resolved by a residual computed in fp32:
    whether and when an fp32 solver stops is then decided by rounding, so the
    counts are not compared (the potentials still are, at the count each
    side reports).
    """
    n_ref, conv_ref = int(ref["n_iters"]), bool(ref["converged"])
    if n == n_ref and conv == conv_ref:
        return True
    band = fp32_noise(ref["f"], ref["g"])
    if 0.0 < float(ref["threshold"]) <= band:
        return True
    if not (conv and conv_ref):
        return False
    period = int(ref.get("check_every", 1))
    if abs(n - n_ref) > 3 * period:
        return False
    return abs(residual_at(n_ref) - float(ref["threshold"])) <= band


def _np(x):
    if x is None:
        return None
    if hasattr(x, "detach"):
        x = x.detach().cpu().numpy()
    return np.asarray(x)


def oracle_residual(p: dict, precision: str = "f64"):
    """residual_at(k) for ``iterations_agree``: the oracle's residual
    max(|f_k - f_{k-1}|, |g_k - g_{k-1}|) of iteration k of problem ``p``
    (k - 1 iterations, then one more started from them)."""
    from oracle import oracle as O

    def at(k):
        args = (p["C"], p.get("a"), p.get("b"), p["eps"], p.get("tau_a"), p.get("tau_b"),
                p.get("mask_a"), p.get("mask_b"))
        f0, g0, _, _ = O.forward(*args, k - 1, 0.0, 1, precision=precision,
                                 f_init=p.get("f_init"), g_init=p.get("g_init"))
        f1, g1, _, _ = O.forward(*args, 1, 0.0, 1, precision=precision, f_init=f0,
                                 g_init=g0)
        return max(np.abs(f1 - f0).max(), np.abs(g1 - g0).max())
    return at


def check_forward_parity(f, g, n, conv, p: dict, oracle_out=None, atol=None,
                         rtol=ORACLE_RTOL, precision="f64"):
    """Forward parity of a build's (f, g, n_iters, converged) against the
    oracle on problem ``p`` (keys C, a, b, eps, tau_a, tau_b, mask_a, mask_b,
    max_iters, threshold, check_every and optionally f_init / g_init).

    The iteration counts must pass ``iterations_agree`` (identical, or apart
    only inside the documented fp32 band around the threshold), and the
    potentials are always compared: against the oracle's own stop when the
    counts agree, else against the oracle run for exactly the build's count.
    Returns the oracle's (f, g, n, converged)."""
    from oracle import oracle as O
    args = (p["C"], p.get("a"), p.get("b"), p["eps"], p.get("tau_a"), p.get("tau_b"),
            p.get("mask_a"), p.get("mask_b"))
    warm = dict(f_init=p.get("f_init"), g_init=p.get("g_init"))
    if oracle_out is None:
        oracle_out = O.forward(*args, p["max_iters"], p["threshold"], p["check_every"],
                               precision=precision, **warm)
    fo, go, no, co = oracle_out
    ref = dict(f=fo, g=go, n_iters=no, converged=co, threshold=p["threshold"],
               check_every=p["check_every"])
    assert iterations_agree(int(n), bool(conv), ref, oracle_residual(p, precision)), \
        (int(n), bool(conv), no, co)
    if int(n) != no:
        fo, go, _, _ = O.forward(*args, int(n), 0.0, p["check_every"], precision=precision,
                                 **warm)
    tol = pot_tolerance(p["eps"]) if atol is None else atol
    np.testing.assert_allclose(_np(f), fo, atol=tol, rtol=rtol)
    np.testing.assert_allclose(_np(g), go, atol=tol, rtol=rtol)
    return oracle_out


def marginal_err_tolerance(me_a, me_b) -> float:
    """Absolute tolerance of a marginal error: fp32 row / column sums of the
    plan carry a few ulps of the largest marginal (the reference's own value
    for a converged case sits at that noise level)."""
    import numpy as np
    return 4e-6 * float(max(np.abs(me_a).max(), np.abs(me_b).max()))


def implicit_fp32_budget(d: dict, key: str) -> float:
    """Tolerance for an fp32 implicit-gradient output against the reference's
    fp64 run (fixture keys ``key`` = the reference's fp32 run, ``key + "64"`` =
    fp64, ``key + "_spread"`` = the largest deviation from fp64 among 64
    reruns of the reference's fp32 CG on plans perturbed by one rounding).

    The reference's CG runs on a near-singular, non-symmetric system (the
    balanced gauge direction is held only by reg = 1e-5), so fp32 rounding is
    amplified by ~1e3-1e4 and where a given fp32 run lands is a matter of
    rounding order: an fp32 implementation is within tolerance when it is no
    further from fp64 than twice the worst of those fp32 runs, plus 1e-5 of the
    output's magnitude. Finite entries only."""
    ref64, ref32 = np.asarray(d[key + "64"]), np.asarray(d[key])
    fin = np.isfinite(ref64) & np.isfinite(ref32)
    if not fin.any():
        return 0.0
    dev = float(np.abs(ref32[fin].astype(np.float64) - ref64[fin]).max())
    dev = max(dev, float(d.get(key + "_spread", 0.0)))
    return 2.0 * dev + 1e-5 * float(np.abs(ref64[fin]).max())
