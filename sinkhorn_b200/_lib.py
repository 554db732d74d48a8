"""ctypes binding of libsinkhorn_b200.so (the C ABI in include/sinkhorn_b200.h).

The library is loaded from the package's _lib/ directory. There is no
fallback: if the library is missing or a call fails, a RuntimeError says so.
"""

from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "libsinkhorn_b200.so")

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_D = ctypes.c_double
_INT = ctypes.c_int
_SZ = ctypes.c_size_t
_IP = ctypes.POINTER(ctypes.c_int)

# name -> (restype, argtypes); mirrors include/sinkhorn_b200.h
SIGNATURES = {
    "sk_version": (_INT, []),
    "sk_last_error": (ctypes.c_char_p, []),
    "sk_forward_workspace_bytes": (_SZ, [_I64, _I64, _I64]),
    "sk_forward": (_INT, [_P, _I64, _I64, _I64, _I64, _I64, _I64, _P, _P, _P, _P, _D, _D,
                          _D, _INT, _D, _INT, _P, _P, _P, _SZ, _IP, _IP, _P]),
    "sk_forward_warm": (_INT, [_P, _I64, _I64, _I64, _I64, _I64, _I64, _P, _P, _P, _P, _D,
                               _D, _D, _INT, _D, _INT, _P, _P, _P, _SZ, _IP, _IP, _P]),
    "sk_forward_bf16": (_INT, [_P, _I64, _I64, _I64, _I64, _I64, _I64, _P, _P, _P, _P, _D,
                               _D, _D, _INT, _D, _INT, _P, _P, _P, _SZ, _IP, _IP, _P]),
    "sk_solver_init": (_INT, [_P, _I64, _I64, _I64, _I64, _I64, _I64, _P, _P, _P, _P, _INT,
                              _D, _INT, _INT, _P, _P, _P, _SZ, _P]),
    "sk_solver_row_sweep": (_INT, [_P, _I64, _I64, _I64, _I64, _I64, _I64, _P, _D, _D, _P,
                                   _P, _SZ, _P]),
    "sk_solver_col_sweep": (_INT, [_P, _I64, _I64, _I64, _I64, _I64, _I64, _P, _D, _D, _P,
                                   _P, _SZ, _P]),
    "sk_solver_col_partial": (_INT, [_P, _I64, _I64, _I64, _I64, _I64, _I64, _D, _P, _P,
                                     _SZ, _P]),
    "sk_solver_col_finish": (_INT, [_P, _INT, _I64, _I64, _I64, _P, _D, _D, _P, _P, _SZ,
                                    _P]),
    "sk_solver_chunk_merge": (_INT, [_P, _I64, _I64, _I64, _I64, _I64, _I64, _P, _P, _SZ,
                                     _P]),
    "sk_solver_rank_rescale": (_INT, [_P, _P, _P, _I64, _P]),
    "sk_solver_col_finish_pairs": (_INT, [_P, _P, _I64, _I64, _I64, _P, _D, _D, _P, _P, _SZ,
                                          _P]),
    "sk_solver_decide": (_INT, [_P, _P]),
    "sk_peer_buffer_bytes": (_SZ, [_INT, _I64, _I64]),
    "sk_peer_buffer_alloc": (_INT, [_SZ, ctypes.POINTER(_P)]),
    "sk_peer_buffer_free": (_INT, [_P]),
    "sk_peer_handle": (_INT, [_P, _P]),
    "sk_peer_open": (_INT, [_P, ctypes.POINTER(_P)]),
    "sk_peer_close": (_INT, [_P]),
    "sk_peer_reset": (_INT, [_P, _INT, _I64, _I64, _P]),
    "sk_solver_chunk_merge_peer": (_INT, [_P, _I64, _I64, _I64, _I64, _I64, _I64,
                                          ctypes.POINTER(_P), _INT, _INT, _P, _SZ, _P]),
    "sk_solver_col_finish_peer": (_INT, [_P, _INT, _I64, _I64, _I64, _P, _D, _D, _P, _P, _SZ,
                                         _P]),
    "sk_solver_fused_step": (_INT, [_P, _I64, _I64, _I64, _I64, _I64, _I64, _P, _D, _D, _P,
                                    _P, _SZ, _P]),
    "sk_solver_fused_finish": (_INT, [_P, _I64, _I64, _I64, _I64, _I64, _I64, _P, _D, _D,
                                      _P, _P, _SZ, _P]),
    "sk_solver_solve": (_INT, [_P, _I64, _I64, _I64, _I64, _I64, _I64, _P, _P, _D, _D, _D,
                               _P, _P, _P, _SZ, _P]),
    "sk_probe_ex2_scratch_bytes": (_SZ, []),
    "sk_probe_ex2_rate": (_INT, [_P, _SZ, ctypes.POINTER(ctypes.c_double), _P]),
    "sk_probe_wait_scratch_bytes": (_SZ, []),
    "sk_probe_wait_timeout": (_INT, [_INT, _INT, ctypes.c_uint, _P, _SZ, _P]),
    "sk_marginal_error_workspace_bytes": (_SZ, [_I64, _I64, _I64]),
    "sk_marginal_error": (_INT, [_P, _I64, _I64, _I64, _I64, _I64, _I64, _P, _P, _P, _P, _D,
                                 _P, _P, _P, _P, _SZ, _P]),
    "sk_plan_matvec_workspace_bytes": (_SZ, [_I64, _I64, _I64]),
    "sk_plan_matvec": (_INT, [_P, _I64, _I64, _I64, _I64, _I64, _I64, _P, _P, _D, _P, _P, _P,
                              _P, _P, _P, _P, _P, _P, _P, _SZ, _P]),
    "sk_implicit_workspace_bytes": (_SZ, [_I64, _I64, _I64]),
    "sk_implicit_matvec": (_INT, [_P, _I64, _I64, _I64, _I64, _I64, _I64, _P, _P, _D, _P, _P,
                                  _P, _P, _P, _D, _D, _D, _INT, _P, _P, _P, _SZ, _P]),
    "sk_implicit_cg": (_INT, [_P, _I64, _I64, _I64, _I64, _I64, _I64, _P, _P, _D, _P, _P, _P,
                              _P, _P, _D, _D, _INT, _D, _D, _P, _P, _P, _P, _P, _SZ, _IP,
                              _P]),
    "sk_implicit_dC": (_INT, [_P, _I64, _I64, _I64, _I64, _I64, _I64, _P, _P, _D, _P, _P, _P,
                              _P, _P, _P]),
    "sk_plan_query": (_INT, [_P, _I64, _I64, _I64, _I64, _I64, _I64, _IP, _IP,
                             ctypes.POINTER(ctypes.c_int64)]),
    "sk_solver_status": (_INT, [_P, _IP, _IP, _IP, _IP, ctypes.POINTER(ctypes.c_float), _P]),
    "sk_lse_row": (_INT, [_P, _I64, _I64, _I64, _I64, _I64, _I64, _P, _D, _P, _P]),
    "sk_lse_col_workspace_bytes": (_SZ, [_I64, _I64, _I64]),
    "sk_lse_col": (_INT, [_P, _I64, _I64, _I64, _I64, _I64, _I64, _P, _D, _P, _P, _SZ,
                          _P]),
    "sk_lse_col_noalloc": (_INT, [_P, _I64, _I64, _I64, _I64, _I64, _I64, _P, _D, _P, _P]),
    "sk_transport_plan": (_INT, [_P, _I64, _I64, _I64, _I64, _I64, _I64, _P, _P, _D, _P,
                                 _P, _P, _P]),
    "sk_cost_workspace_bytes": (_SZ, [_I64, _I64, _I64]),
    "sk_cost": (_INT, [_P, _I64, _I64, _I64, _I64, _I64, _I64, _P, _P, _D, _P, _P, _SZ,
                       _P]),
    "sk_jvp_workspace_bytes": (_SZ, [_I64, _I64, _I64]),
    "sk_jvp": (_INT, [_P, _I64, _I64, _I64, _I64, _I64, _I64, _P, _P, _D, _P, _P, _D, _D,
                      _P, _P, _P, _SZ, _P]),
    "sk_jvp_plan": (_INT, [_P, _I64, _I64, _I64, _P, _P, _D, _D, _P, _P, _P, _SZ, _P]),
    "sk_plan_backward": (_INT, [_P, _I64, _I64, _I64, _I64, _I64, _I64, _P, _P, _D, _P,
                                _P, _P, _P, _P, _P, _P, _SZ, _P]),
    "sk_backward_workspace_bytes": (_SZ, [_I64, _I64, _I64, _I64]),
    "sk_backward": (_INT, [_P, _I64, _I64, _I64, _I64, _I64, _I64, _P, _P, _P, _P, _D, _D,
                           _D, _INT, _D, _INT, _P, _P, _P, _P, _P, _P, _P, _P, _SZ, _IP,
                           _P]),
}

_lock = threading.Lock()
_lib = None


class SinkhornCudaError(RuntimeError):
    """A libsinkhorn_b200 entry point returned an error status."""


def load() -> ctypes.CDLL:
    """Load the library (once). Raises RuntimeError if it has not been built."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with `python -m sinkhorn_b200.build` "
                    "(nvcc, sm_100a). sinkhorn_b200 has no CPU fallback.")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name, None)
                if fn is None:
                    continue
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def exported_symbols() -> list[str]:
    lib = load()
    return [n for n in SIGNATURES if getattr(lib, n, None) is not None]


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = load().sk_last_error()
        msg = msg.decode() if msg else ""
        raise SinkhornCudaError(f"{what} failed (status {rc}): {msg}")
