"""numpy front end of the C Sinkhorn oracle (``oracle/sk_oracle.c``).

TEST INFRASTRUCTURE ONLY. Imported by ``tests/``, ``__graft_entry__.smoke()``
and the CPU-baseline / reference leg of ``bench.py``; never by the product
package ``sinkhorn_b200``, which has no CPU fallback.

Parity pin: ``tests/test_oracle_golden.py`` checks every function here against
golden vectors produced by running the reference package itself
(``tests/golden/make_golden.py``).

The front end restates the reference's host-side prologue before calling the
C loops:

* rho = eps/(eps+tau), 0 for tau None/inf
  (src/sinkhorn/pytorch/unbalanced.py:13-25, src/sinkhorn/triton/forward.py:124-129);
* default marginals: uniform 1/N in fp32, or mask/count(mask).clamp(1) in fp32
  (unbalanced.py:48-57, forward.py:132-142);
* log(clamp(a, 1e-38)) with 1e-38 rounded to fp32 (a subnormal)
  (unbalanced.py:59-60, forward.py:144-145).

``precision="f64"`` (default) runs the fp64 oracle; ``"f32"`` runs the same
loops in fp32, the arithmetic type of the reference, and is what the CPU
baseline times.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
import threading

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "_build", "libsk_oracle.so")
_LOCK = threading.Lock()
_LIB = None

F32_TINY = float(np.float32(1e-38))  # the fp32 value of the reference's clamp

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_D = ctypes.c_double
_INT = ctypes.c_int


def build() -> str:
    """Compile the oracle with its Makefile; returns the library path."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _SO


def lib() -> ctypes.CDLL:
    global _LIB
    with _LOCK:
        if _LIB is None:
            if not os.path.exists(_SO):
                build()
            L = ctypes.CDLL(_SO)
            for pfx in ("sko64_", "sko32_"):
                getattr(L, pfx + "lse_row").argtypes = [_P, _I64, _I64, _I64, _P, _D, _P]
                getattr(L, pfx + "lse_col").argtypes = [_P, _I64, _I64, _I64, _P, _D, _P]
                fw = getattr(L, pfx + "forward")
                fw.argtypes = [_P, _I64, _I64, _I64, _P, _P, _P, _P, _D, _D, _D,
                               _INT, _D, _INT, _P, _P, _P]
                fw.restype = _INT
                bw = getattr(L, pfx + "backward")
                bw.argtypes = [_P, _I64, _I64, _I64, _P, _P, _P, _P, _D, _D, _D,
                               _INT, _INT, _INT, _D, _P, _P, _P, _P, _P, _P, _P]
                bw.restype = _INT
                getattr(L, pfx + "iterate").argtypes = [_P, _I64, _I64, _I64, _P, _P, _P, _P,
                                                        _D, _D, _D, _INT, _INT, _P, _P]
                getattr(L, pfx + "plan").argtypes = [_P, _I64, _I64, _I64, _P, _P, _D,
                                                     _P, _P, _P]
                getattr(L, pfx + "cost").argtypes = [_P, _I64, _I64, _I64, _P, _P, _D, _P]
                getattr(L, pfx + "jvp").argtypes = [_P, _I64, _I64, _I64, _P, _P, _D, _D,
                                                    _P, _P]
            _LIB = L
    return _LIB


def _np(x):
    if x is None:
        return None
    if hasattr(x, "detach"):  # torch tensor
        x = x.detach().cpu().numpy()
    return np.asarray(x)


def _real(precision):
    if precision == "f64":
        return np.float64, "sko64_"
    if precision == "f32":
        return np.float32, "sko32_"
    raise ValueError(f"precision must be 'f64' or 'f32', got {precision!r}")


def _arr(x, dt):
    return np.ascontiguousarray(_np(x), dtype=dt)


def _mask(m):
    if m is None:
        return None
    return np.ascontiguousarray(_np(m).astype(np.uint8))


def _ptr(x):
    return None if x is None else x.ctypes.data_as(ctypes.c_void_p)


def compute_rho(epsilon: float, tau) -> float:
    """unbalanced.py:13-25."""
    if tau is None or tau == float("inf"):
        return 0.0
    return epsilon / (epsilon + tau)


def default_marginal(mask, B: int, n: int) -> np.ndarray:
    """fp32 default marginal of forward.py:132-142."""
    if mask is not None:
        m = _np(mask).astype(np.float32)
        cnt = np.maximum(m.sum(axis=-1, keepdims=True, dtype=np.float32), np.float32(1))
        return (m / cnt).astype(np.float32)
    return np.full((B, n), np.float32(1) / np.float32(n), dtype=np.float32)


def log_marginal(a) -> np.ndarray:
    """log(a.clamp(min=1e-38)) with the fp32 clamp value, in float64."""
    a64 = _np(a).astype(np.float64)
    return np.log(np.maximum(a64, F32_TINY))


def forward(C, a=None, b=None, epsilon=0.1, tau_a=None, tau_b=None, mask_a=None,
            mask_b=None, max_iters=100, threshold=1e-6, check_every=1,
            precision="f64", f_init=None, g_init=None):
    """Forward solve. check_every=1: PyTorch path (unbalanced.py:125-163);
    check_every=10: Triton path (forward.py:161-186).

    ``f_init`` / ``g_init`` (optional, (B,N) / (B,M)) start the loop from
    those potentials instead of zeros -- the warm start of
    ``_sinkhorn_iters_from_init`` (autograd.py:134-178) with the forward's
    masking, guard and checks: the first iteration's rho-mix uses f_init /
    g_init as they are (masked entries included) and the first residual is
    measured against them.
    Returns (f, g, n_iters, converged) as numpy arrays in the oracle's dtype."""
    dt, pfx = _real(precision)
    C = _arr(C, dt)
    B, N, M = C.shape
    if a is None:
        a = default_marginal(mask_a, B, N)
    if b is None:
        b = default_marginal(mask_b, B, M)
    la = _arr(log_marginal(a), dt)
    lb = _arr(log_marginal(b), dt)
    ma, mb = _mask(mask_a), _mask(mask_b)
    f = np.zeros((B, N), dt) if f_init is None else _arr(f_init, dt).reshape(B, N).copy()
    g = np.zeros((B, M), dt) if g_init is None else _arr(g_init, dt).reshape(B, M).copy()
    conv = ctypes.c_int(0)
    n = getattr(lib(), pfx + "forward")(
        _ptr(C), B, N, M, _ptr(la), _ptr(lb), _ptr(ma), _ptr(mb), float(epsilon),
        compute_rho(epsilon, tau_a), compute_rho(epsilon, tau_b), int(max_iters),
        float(threshold), int(check_every), _ptr(f), _ptr(g), ctypes.byref(conv))
    return f, g, int(n), bool(conv.value)


def iters_from_init(C, a, b, epsilon, tau_a, tau_b, mask_a, mask_b, f_init, g_init,
                    n_iters, precision="f64", masked=False):
    """``_sinkhorn_iters_from_init`` (autograd.py:134-178): n_iters Gauss-Seidel
    iterations from (f_init, g_init) on raw C, with log(clamp(a, 1e-38)) and
    the rho of autograd.py:150-157, no guard, masks applied to the final f / g
    only. ``a`` / ``b`` None take the defaults of sinkhorn_differentiable
    (autograd.py:223-233). ``masked=True`` runs the forward iteration
    (C masked, guard, masked_fill after every iteration) instead, with no
    convergence check. Returns (f, g) in the oracle's dtype."""
    dt, pfx = _real(precision)
    C = _arr(C, dt)
    B, N, M = C.shape
    if a is None:
        a = default_marginal(mask_a, B, N)
    if b is None:
        b = default_marginal(mask_b, B, M)
    la = _arr(log_marginal(a), dt)
    lb = _arr(log_marginal(b), dt)
    f = _arr(f_init, dt).reshape(B, N).copy()
    g = _arr(g_init, dt).reshape(B, M).copy()
    getattr(lib(), pfx + "iterate")(
        _ptr(C), B, N, M, _ptr(la), _ptr(lb), _ptr(_mask(mask_a)), _ptr(_mask(mask_b)),
        float(epsilon), compute_rho(epsilon, tau_a), compute_rho(epsilon, tau_b),
        int(bool(masked)), int(n_iters), _ptr(f), _ptr(g))
    return f, g


def lse_row(C, g, epsilon, precision="f64"):
    """Row softmin of lse_kernel.py:210-250 (0 for an empty row)."""
    dt, pfx = _real(precision)
    C = _arr(C, dt)
    B, N, M = C.shape
    g = _arr(g, dt)
    out = np.empty((B, N), dt)
    getattr(lib(), pfx + "lse_row")(_ptr(C), B, N, M, _ptr(g), float(epsilon), _ptr(out))
    return out


def lse_col(C, f, epsilon, precision="f64"):
    """Column softmin of lse_kernel.py:253-293 (0 for an empty column)."""
    dt, pfx = _real(precision)
    C = _arr(C, dt)
    B, N, M = C.shape
    f = _arr(f, dt)
    out = np.empty((B, M), dt)
    getattr(lib(), pfx + "lse_col")(_ptr(C), B, N, M, _ptr(f), float(epsilon), _ptr(out))
    return out


def transport_plan(C, f, g, epsilon, mask_a=None, mask_b=None, precision="f64"):
    """sinkhorn.py:27-54."""
    dt, pfx = _real(precision)
    C = _arr(C, dt)
    B, N, M = C.shape
    P = np.empty_like(C)
    getattr(lib(), pfx + "plan")(_ptr(C), B, N, M, _ptr(_arr(f, dt)), _ptr(_arr(g, dt)),
                                 float(epsilon), _ptr(_mask(mask_a)), _ptr(_mask(mask_b)),
                                 _ptr(P))
    return P


def cost(C, f, g, epsilon, precision="f64"):
    """sinkhorn.py:56-67 (masks ignored, as in the reference)."""
    dt, pfx = _real(precision)
    C = _arr(C, dt)
    B, N, M = C.shape
    out = np.empty((B,), dt)
    getattr(lib(), pfx + "cost")(_ptr(C), B, N, M, _ptr(_arr(f, dt)), _ptr(_arr(g, dt)),
                                 float(epsilon), _ptr(out))
    return out


def jvp(P, v_f, v_g, rho_a=0.0, rho_b=0.0, precision="f64"):
    """jvp_kernel.py:113-182 on a materialised plan."""
    dt, pfx = _real(precision)
    P = _arr(P, dt)
    B, N, M = P.shape
    of = np.empty((B, N), dt)
    og = np.empty((B, M), dt)
    getattr(lib(), pfx + "jvp")(_ptr(P), B, N, M, _ptr(_arr(v_f, dt)), _ptr(_arr(v_g, dt)),
                                float(rho_a), float(rho_b), _ptr(of), _ptr(og))
    return of, og


def backward(C, a=None, b=None, epsilon=0.1, tau_a=None, tau_b=None, mask_a=None,
             mask_b=None, max_iters=100, threshold=1e-6, grad_iters=0, f_star=None,
             g_star=None, grad_f=None, grad_g=None, precision="f64"):
    """SinkhornFunction.backward (autograd.py:61-131) for the cost matrix and
    the marginals. ``a``/``b`` None means the defaults of
    sinkhorn_differentiable (autograd.py:223-233), which carry no gradient.

    Returns (dC, da, db, K) where K is the number of recorded iterations.
    The full-recompute mode is used when grad_iters is outside (0, max_iters)
    (autograd.py:76)."""
    dt, pfx = _real(precision)
    C = _arr(C, dt)
    B, N, M = C.shape
    if a is None:
        a = default_marginal(mask_a, B, N)
    if b is None:
        b = default_marginal(mask_b, B, M)
    a64 = _np(a).astype(np.float64)
    b64 = _np(b).astype(np.float64)
    la = _arr(log_marginal(a64), dt)
    lb = _arr(log_marginal(b64), dt)
    full = not (0 < grad_iters < max_iters)
    if f_star is None:
        f_star = np.zeros((B, N))
    if g_star is None:
        g_star = np.zeros((B, M))
    if grad_f is None:
        grad_f = np.zeros((B, N))
    if grad_g is None:
        grad_g = np.zeros((B, M))
    dC = np.empty_like(C)
    dla = np.empty((B, N), dt)
    dlb = np.empty((B, M), dt)
    K = getattr(lib(), pfx + "backward")(
        _ptr(C), B, N, M, _ptr(la), _ptr(lb), _ptr(_mask(mask_a)), _ptr(_mask(mask_b)),
        float(epsilon), compute_rho(epsilon, tau_a), compute_rho(epsilon, tau_b),
        int(full), int(grad_iters), int(max_iters), float(threshold),
        _ptr(_arr(f_star, dt)), _ptr(_arr(g_star, dt)), _ptr(_arr(grad_f, dt)),
        _ptr(_arr(grad_g, dt)), _ptr(dC), _ptr(dla), _ptr(dlb))
    # d/da log(clamp(a, tiny)) = 1/a where a >= tiny (clamp_min backward), else 0
    da = np.where(a64 >= F32_TINY, dla / np.maximum(a64, F32_TINY), 0.0).astype(dt)
    db = np.where(b64 >= F32_TINY, dlb / np.maximum(b64, F32_TINY), 0.0).astype(dt)
    return dC, da, db, int(K)


def plan_backward(C, f, g, epsilon, grad_P, mask_a=None, mask_b=None):
    """Adjoint of P = exp((f+g-C)/eps) for an upstream gradient grad_P:
    dC = -grad_P*P/eps, df = sum_j grad_P*P/eps, dg = sum_i grad_P*P/eps
    (masked entries of P are constants and pass nothing). float64 numpy."""
    P = transport_plan(C, f, g, epsilon, mask_a, mask_b)
    w = _np(grad_P).astype(np.float64) * P / epsilon
    return -w, w.sum(axis=2), w.sum(axis=1)


def marginal_error(C, f, g, a, b, epsilon, mask_a=None, mask_b=None):
    """compute_marginal_error (pytorch/balanced.py:183-213): the largest of
    max |P 1 - a| (0 at masked rows) and max |P^T 1 - b| (0 at masked
    columns) over the whole batch, P the masked plan. float64 numpy."""
    P = transport_plan(C, f, g, epsilon, mask_a, mask_b)
    re = np.abs(P.sum(axis=2) - _np(a).astype(np.float64))
    ce = np.abs(P.sum(axis=1) - _np(b).astype(np.float64))
    if mask_a is not None:
        re = np.where(_np(mask_a).astype(bool), re, 0.0)
    if mask_b is not None:
        ce = np.where(_np(mask_b).astype(bool), ce, 0.0)
    return float(max(re.max(), ce.max()))


# ---------------------------------------------------------------------------
# Implicit-differentiation adjoint (src/sinkhorn/pytorch/implicit_diff.py),
# restated in numpy. ``precision`` "f64" (default) or "f32" (the reference's
# arithmetic type for fp32 inputs).

_SUM_FLOOR = 1e-30  # row_sum / col_sum and dot clamps, implicit_diff.py:83-84,168,187


def _plan_sums(P):
    """Row and column sums clamped at 1e-30 (implicit_diff.py:83-84)."""
    fl = P.dtype.type(_SUM_FLOOR)
    return np.maximum(P.sum(axis=2), fl), np.maximum(P.sum(axis=1), fl)


def implicit_matvec(v_f, v_g, P, rho_a=0.0, rho_b=0.0, reg=1e-5, mode="schur", mask_a=None,
                    mask_b=None, precision="f64"):
    """One Jacobian product on a dense plan:
    "schur": (1+reg) v - J_T^T v   (schur_complement_matvec, implicit_diff.py:45-104)
    "vjp":   J_T^T v, 0 at masked   (vjp_sinkhorn, :281-309)
    "jvp":   J_T v, 0 at masked     (jvp_sinkhorn, :253-278)"""
    dt, _ = _real(precision)
    P = _arr(P, dt)
    vf, vg = _arr(v_f, dt), _arr(v_g, dt)
    r, c = _plan_sums(P)
    if mode == "jvp":
        of = rho_a * vf + (1 - rho_a) * np.einsum("bnm,bm->bn", P, vg) / r
        og = rho_b * vg + (1 - rho_b) * np.einsum("bnm,bn->bm", P, vf) / c
    else:
        jf = rho_a * vf + (1 - rho_b) * np.einsum("bnm,bm->bn", P, vg / c)
        jg = rho_b * vg + (1 - rho_a) * np.einsum("bnm,bn->bm", P, vf / r)
        if mode == "schur":
            return ((1 + reg) * vf - jf).astype(dt), ((1 + reg) * vg - jg).astype(dt)
        of, og = jf, jg
    if mask_a is not None:
        of = np.where(_np(mask_a).astype(bool), of, 0)
    if mask_b is not None:
        og = np.where(_np(mask_b).astype(bool), og, 0)
    return of.astype(dt), og.astype(dt)


def cg_solve(rhs_f, rhs_g, P, rho_a=0.0, rho_b=0.0, max_iters=50, tol=1e-5, reg=1e-5,
             precision="f64"):
    """Batched CG on (I - J_T^T + reg I) lambda = rhs (cg_solve,
    implicit_diff.py:107-193): x0 = 0; alpha = r.r / max(p.Ap, 1e-30); stop
    after the first iteration whose max_b |r_b| < tol * max_b |rhs_b| (NaN
    never stops); beta = r'.r' / max(r.r, 1e-30). Returns (x_f, x_g, n_iters)."""
    dt, _ = _real(precision)
    P = _arr(P, dt)
    r_f, r_g = _arr(rhs_f, dt).copy(), _arr(rhs_g, dt).copy()
    x_f, x_g = np.zeros_like(r_f), np.zeros_like(r_g)
    p_f, p_g = r_f.copy(), r_g.copy()

    def dot(a_f, a_g, b_f, b_g):
        return (a_f * b_f).sum(axis=-1) + (a_g * b_g).sum(axis=-1)

    def clamp(v):
        return np.where(v < _SUM_FLOOR, dt(_SUM_FLOOR), v)  # keeps NaN, as torch.clamp

    def nanmax(v):
        return np.nan if np.isnan(v).any() else v.max()

    r_dot = dot(r_f, r_g, r_f, r_g)
    rhs_norm = nanmax(np.sqrt(r_dot))
    n = 0
    with np.errstate(all="ignore"):
        for i in range(max_iters):
            Ap_f, Ap_g = implicit_matvec(p_f, p_g, P, rho_a, rho_b, reg, "schur",
                                         precision=precision)
            alpha = (r_dot / clamp(dot(p_f, p_g, Ap_f, Ap_g)))[:, None]
            x_f, x_g = x_f + alpha * p_f, x_g + alpha * p_g
            r_f, r_g = r_f - alpha * Ap_f, r_g - alpha * Ap_g
            n = i + 1
            r_new = dot(r_f, r_g, r_f, r_g)
            if nanmax(np.sqrt(r_new)) < tol * rhs_norm:
                break
            beta = (r_new / clamp(r_dot))[:, None]
            p_f, p_g = r_f + beta * p_f, r_g + beta * p_g
            r_dot = r_new
    return x_f.astype(dt), x_g.astype(dt), n


def implicit_gradient(C, f, g, grad_f, grad_g, epsilon, tau_a=None, tau_b=None, mask_a=None,
                      mask_b=None, cg_max_iters=50, cg_tol=1e-5, precision="f64"):
    """implicit_gradient (implicit_diff.py:196-249): the masked plan, CG with
    reg 1e-5 on the upstream (grad_f, grad_g), then
    dC = -(1/eps) P (lambda_f[:, None] + lambda_g[None, :]), da = eps lambda_f,
    db = eps lambda_g. Returns (dC, da, db, n_iters)."""
    dt, _ = _real(precision)
    P = transport_plan(C, f, g, epsilon, mask_a, mask_b, precision)
    lf, lg, n = cg_solve(grad_f, grad_g, P, compute_rho(epsilon, tau_a),
                         compute_rho(epsilon, tau_b), cg_max_iters, cg_tol, 1e-5, precision)
    with np.errstate(all="ignore"):
        dC = -(1.0 / epsilon) * P * (lf[:, :, None] + lg[:, None, :])
    return dC.astype(dt), (epsilon * lf).astype(dt), (epsilon * lg).astype(dt), n


def ensure_threads(n: int | None = None) -> int:
    """Number of OpenMP threads the oracle will use: ``n`` if given (set in
    the OpenMP runtime, so it holds even where a launcher exported
    OMP_NUM_THREADS=1), else OMP_NUM_THREADS or all cores in this process's
    affinity set."""
    if n is None:
        n = int(os.environ.get("OMP_NUM_THREADS", "0")) or len(os.sched_getaffinity(0))
    else:
        L = lib()
        L.sko64_set_threads.argtypes = [_INT]
        L.sko64_set_threads(int(n))
    return n


__all__ = [
    "build", "lib", "compute_rho", "default_marginal", "log_marginal", "forward",
    "lse_row", "lse_col", "transport_plan", "cost", "jvp", "backward",
    "plan_backward", "marginal_error", "implicit_matvec", "cg_solve", "implicit_gradient",
    "ensure_threads",
]
