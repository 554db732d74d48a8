"""CPU checks of the C ABI: the library loads, exports every symbol the
header declares, sizes workspaces and rejects bad arguments before touching a
device (no compute calls here)."""

from __future__ import annotations

import ctypes
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "sinkhorn_b200.h")


def declared_symbols() -> list[str]:
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(sk_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_entry_points():
    names = declared_symbols()
    for must in ("sk_forward", "sk_lse_row", "sk_lse_col", "sk_transport_plan", "sk_cost",
                 "sk_jvp", "sk_jvp_plan", "sk_plan_backward", "sk_backward",
                 "sk_last_error", "sk_version"):
        assert must in names


def test_library_exports_every_declared_symbol():
    from sinkhorn_b200 import _lib
    lib = ctypes.CDLL(_lib.LIB_PATH)
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, missing


def test_python_binding_covers_the_header():
    from sinkhorn_b200 import _lib
    assert set(declared_symbols()) <= set(_lib.SIGNATURES)


def test_version_and_error_string():
    from sinkhorn_b200 import _lib
    lib = _lib.load()
    assert lib.sk_version() >= 100
    assert lib.sk_last_error() is not None


def test_workspace_sizes_are_positive_and_monotone():
    from sinkhorn_b200 import _lib
    lib = _lib.load()
    small = lib.sk_forward_workspace_bytes(1, 64, 64)
    big = lib.sk_forward_workspace_bytes(1, 16384, 16384)
    assert 0 < small < big
    assert lib.sk_forward_workspace_bytes(0, 4, 4) == 0
    assert lib.sk_backward_workspace_bytes(2, 32, 32, 10) > lib.sk_backward_workspace_bytes(2, 32, 32, 1)
    assert lib.sk_lse_col_workspace_bytes(1, 128, 128) > 0
    assert lib.sk_cost_workspace_bytes(1, 128, 128) > 0
    assert lib.sk_jvp_workspace_bytes(1, 128, 128) > 0


def _fwd(lib, C=1, B=1, N=4, M=4, eps=0.1, f=1, g=1, ws=1, wsb=1 << 30, iters=10, ce=10):
    n = ctypes.c_int(-1)
    c = ctypes.c_int(-1)
    return lib.sk_forward(C, B, N, M, N * M, M, 1, None, None, None, None, eps,
                          float("inf"), float("inf"), iters, 1e-6, ce, f, g, ws, wsb,
                          ctypes.byref(n), ctypes.byref(c), None)


@pytest.mark.parametrize("kw,code", [
    (dict(C=None), 1), (dict(N=0), 1), (dict(eps=0.0), 1), (dict(eps=float("nan")), 1),
    (dict(iters=-1), 1), (dict(ce=0), 1), (dict(f=None), 1), (dict(ws=None), 3),
    (dict(wsb=16), 3),
])
def test_forward_rejects_bad_arguments_without_a_device(kw, code):
    from sinkhorn_b200 import _lib
    lib = _lib.load()
    assert _fwd(lib, **kw) == code
    assert lib.sk_last_error().decode()


@pytest.mark.parametrize("B,N,M,base,vec,fused,chunks", [
    # single-read iteration k_fused_iter (M >= 8192): 74 two-CTA clusters
    (1, 16384, 16384, 4096, 4, 2, 74),
    # one-CTA units of k_fused_iter (2048 < M < 8192, rows of M % 4 == 0): one
    # wave of 148; short chunks take the fewest that fill the SMs within 5%
    (1, 65536, 4096, 4096, 4, 2, 148),
    (16, 2048, 2560, 4096, 4, 2, 9),
    (1, 4096, 2052, 4096, 4, 2, 137),
    # k_rows_fused (M = 512 and 1024 < M <= 2048, B*N >= 4736): one wave of 9
    # chunks per item where it fills the SMs within 5% of four waves of 37
    (16, 2048, 2048, 4096, 4, 2, 9),
    (64, 2048, 512, 4096, 4, 2, 9),
    # k_row_warps (512 < M <= 1024): about two waves of 2 CTAs per SM over the
    # batch, chunks at least 64 rows deep
    (64, 1024, 1024, 4096, 4, 2, 10),
    (32, 1024, 1024, 4096, 4, 2, 16),
    # the iteration exists but sk_forward keeps two sweeps (too few rows)
    (1, 300, 1024, 4096, 4, 1, 5),
    # M below the rows kernel: two sweeps only
    (8, 64, 64, 4096, 4, 0, 0),
    # a base address off the 16-byte grid: the strided scalar path
    (1, 16384, 16384, 4100, 1, 0, 0),
])
def test_plan_query_selects_kernels_without_a_device(B, N, M, base, vec, fused, chunks):
    """sk_plan_query is host logic over the shape, the strides and the base
    address's alignment (the address is never dereferenced)."""
    from sinkhorn_b200 import _lib
    lib = _lib.load()
    v, f, c = ctypes.c_int(-1), ctypes.c_int(-1), ctypes.c_int64(-1)
    rc = lib.sk_plan_query(ctypes.c_void_p(base), B, N, M, N * M, M, 1, ctypes.byref(v),
                           ctypes.byref(f), ctypes.byref(c))
    assert rc == 0
    assert (v.value, f.value, c.value) == (vec, fused, chunks)


def test_implicit_workspace_sizes():
    from sinkhorn_b200 import _lib
    lib = _lib.load()
    assert lib.sk_implicit_workspace_bytes(0, 8, 8) == 0
    assert 0 < lib.sk_implicit_workspace_bytes(2, 64, 64) < \
        lib.sk_implicit_workspace_bytes(16, 2048, 2048)
    assert 0 < lib.sk_plan_matvec_workspace_bytes(1, 40, 64)


def _cg(lib, C=1, f=1, g=1, P=None, rf=1, rg=1, lf=1, lg=1, it=5, eps=0.5, ga=None,
        ws=1, wsb=1 << 30):
    n = ctypes.c_int(-1)
    return lib.sk_implicit_cg(C, 2, 8, 8, 64, 8, 1, f, g, eps, None, None, P, rf, rg, 0.0,
                              0.0, it, 1e-5, 1e-5, lf, lg, ga, None, ws, wsb,
                              ctypes.byref(n), None)


@pytest.mark.parametrize("kw,code", [
    (dict(C=None), 1), (dict(f=None), 1), (dict(rf=None), 1), (dict(lg=None), 1),
    (dict(it=-1), 1), (dict(eps=0.0), 1), (dict(ws=None), 3), (dict(wsb=64), 3),
    (dict(C=None, f=None, g=None, P=None), 1),
])
def test_implicit_cg_rejects_bad_arguments_without_a_device(kw, code):
    from sinkhorn_b200 import _lib
    lib = _lib.load()
    assert _cg(lib, **kw) == code
    assert lib.sk_last_error().decode()


def test_implicit_matvec_rejects_bad_mode_without_a_device():
    from sinkhorn_b200 import _lib
    lib = _lib.load()
    rc = lib.sk_implicit_matvec(1, 1, 8, 8, 64, 8, 1, 1, 1, 0.5, None, None, None, 1, 1, 0.0,
                                0.0, 1e-5, 3, 1, 1, 1, 1 << 30, None)
    assert rc == 1 and "mode" in lib.sk_last_error().decode()


# Every entry point checks its problem (C, B, N, M, epsilon), its pointers and
# its workspace before any CUDA call; these cases stop there (pointers are
# never dereferenced), so they run without a device.
_P = 1          # a non-NULL pointer that is never read
_W = 1 << 40    # workspace bytes larger than any requirement
_ERR_ARG, _ERR_WS = 1, 3


def _entry_cases():
    inf = float("inf")
    n, c, k = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    return [
        ("lse_row C=NULL", lambda L: L.sk_lse_row(None, 1, 4, 4, 16, 4, 1, _P, 0.1, _P, None),
         _ERR_ARG),
        ("lse_row out=NULL", lambda L: L.sk_lse_row(_P, 1, 4, 4, 16, 4, 1, _P, 0.1, None, None),
         _ERR_ARG),
        ("lse_row M=0", lambda L: L.sk_lse_row(_P, 1, 4, 0, 0, 0, 1, _P, 0.1, _P, None),
         _ERR_ARG),
        ("lse_col eps<0", lambda L: L.sk_lse_col(_P, 1, 4, 4, 16, 4, 1, _P, -1.0, _P, _P, _W,
                                                 None), _ERR_ARG),
        ("lse_col no workspace", lambda L: L.sk_lse_col(_P, 1, 4, 4, 16, 4, 1, _P, 0.1, _P,
                                                        None, 0, None), _ERR_WS),
        ("lse_col_noalloc beyond its scratch",
         lambda L: L.sk_lse_col_noalloc(_P, 1, 4, 1 << 22, 4 << 22, 1 << 22, 1, _P, 0.1, _P,
                                        None), _ERR_WS),
        ("transport_plan P=NULL",
         lambda L: L.sk_transport_plan(_P, 1, 4, 4, 16, 4, 1, _P, _P, 0.1, None, None, None,
                                       None), _ERR_ARG),
        ("transport_plan eps=inf",
         lambda L: L.sk_transport_plan(_P, 1, 4, 4, 16, 4, 1, _P, _P, inf, None, None, _P,
                                       None), _ERR_ARG),
        ("cost g=NULL", lambda L: L.sk_cost(_P, 1, 4, 4, 16, 4, 1, _P, None, 0.1, _P, _P, _W,
                                            None), _ERR_ARG),
        ("cost small workspace", lambda L: L.sk_cost(_P, 1, 4, 4, 16, 4, 1, _P, _P, 0.1, _P, _P,
                                                     4, None), _ERR_WS),
        ("marginal_error b=NULL",
         lambda L: L.sk_marginal_error(_P, 1, 4, 4, 16, 4, 1, _P, _P, _P, None, 0.1, None, None,
                                       _P, _P, _W, None), _ERR_ARG),
        ("marginal_error no workspace",
         lambda L: L.sk_marginal_error(_P, 1, 4, 4, 16, 4, 1, _P, _P, _P, _P, 0.1, None, None,
                                       _P, None, 0, None), _ERR_WS),
        ("jvp v_g=NULL", lambda L: L.sk_jvp(_P, 1, 4, 4, 16, 4, 1, _P, _P, 0.1, _P, None, 1.0,
                                            1.0, _P, _P, _P, _W, None), _ERR_ARG),
        ("jvp small workspace", lambda L: L.sk_jvp(_P, 1, 4, 4, 16, 4, 1, _P, _P, 0.1, _P, _P,
                                                   1.0, 1.0, _P, _P, _P, 4, None), _ERR_WS),
        ("jvp_plan P=NULL", lambda L: L.sk_jvp_plan(None, 1, 4, 4, _P, _P, 1.0, 1.0, _P, _P, _P,
                                                    _W, None), _ERR_ARG),
        ("plan_backward grad_P=NULL",
         lambda L: L.sk_plan_backward(_P, 1, 4, 4, 16, 4, 1, _P, _P, 0.1, None, None, None, _P,
                                      _P, _P, _P, _W, None), _ERR_ARG),
        ("backward dC=NULL",
         lambda L: L.sk_backward(_P, 1, 4, 4, 16, 4, 1, None, None, None, None, 0.1, inf, inf,
                                 10, 1e-6, 0, None, None, _P, _P, None, None, None, _P, _W,
                                 ctypes.byref(k), None), _ERR_ARG),
        ("backward max_iters<0",
         lambda L: L.sk_backward(_P, 1, 4, 4, 16, 4, 1, None, None, None, None, 0.1, inf, inf,
                                 -1, 1e-6, 0, None, None, _P, _P, _P, None, None, _P, _W,
                                 ctypes.byref(k), None), _ERR_ARG),
        ("backward truncated without f*, g*",
         lambda L: L.sk_backward(_P, 1, 4, 4, 16, 4, 1, None, None, None, None, 0.1, inf, inf,
                                 10, 1e-6, 3, None, None, _P, _P, _P, None, None, _P, _W,
                                 ctypes.byref(k), None), _ERR_ARG),
        ("backward no workspace",
         lambda L: L.sk_backward(_P, 1, 4, 4, 16, 4, 1, None, None, None, None, 0.1, inf, inf,
                                 10, 1e-6, 0, None, None, _P, _P, _P, None, None, None, 0,
                                 ctypes.byref(k), None), _ERR_WS),
        ("forward_warm N=0",
         lambda L: L.sk_forward_warm(_P, 1, 0, 4, 0, 4, 1, None, None, None, None, 0.1, inf,
                                     inf, 10, 1e-6, 10, _P, _P, _P, _W, ctypes.byref(n),
                                     ctypes.byref(c), None), _ERR_ARG),
        ("col_finish_peer P=9",
         lambda L: L.sk_solver_col_finish_peer(_P, 9, 1, 4, 4, None, 0.1, inf, _P, _P, _W,
                                               None), _ERR_ARG),
    ]


@pytest.mark.parametrize("case", _entry_cases(), ids=lambda c: c[0])
def test_entry_points_reject_bad_arguments_without_a_device(case):
    from sinkhorn_b200 import _lib
    lib = _lib.load()
    _, call, code = case
    assert call(lib) == code
    assert lib.sk_last_error().decode()


def test_peer_buffer_sizes_cover_one_to_eight_ranks():
    from sinkhorn_b200 import _lib
    lib = _lib.load()
    sizes = [lib.sk_peer_buffer_bytes(p, 1, 16384) for p in range(1, 9)]
    assert all(s > 0 for s in sizes) and sizes == sorted(sizes)
    assert lib.sk_peer_buffer_bytes(0, 1, 16384) == 0
    assert lib.sk_peer_buffer_bytes(9, 1, 16384) == 0


def test_integration_guide_names_every_entry_point():
    doc = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    named = set(re.findall(r"sk_[a-z0-9_]+", doc))
    missing = [n for n in declared_symbols()
               if n not in named and not n.endswith(("_workspace_bytes", "_scratch_bytes"))]
    assert not missing, missing
