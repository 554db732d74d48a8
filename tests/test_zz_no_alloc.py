"""GPU test of sk_lse_col_noalloc, the column softmin for callers that cannot
allocate device memory when they call in (its scratch is a fixed array inside
the library instead of a caller workspace).

Checked through the C ABI against the workspace entry point sk_lse_col, on two
calls in a row with different shapes (the second call must not see the first
call's tickets), and for the size limit of the built-in scratch. This file is
named to be collected last.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from sinkhorn_b200 import _lib
    return _lib.load()


def _lse_col_workspace(lib, C, f, eps):
    B, N, M = C.shape
    out = torch.empty(B, M, device=C.device, dtype=torch.float32)
    ws = torch.empty(max(lib.sk_lse_col_workspace_bytes(B, N, M), 256), dtype=torch.uint8,
                     device=C.device)
    rc = lib.sk_lse_col(C.data_ptr(), B, N, M, *C.stride(), f.data_ptr(), float(eps),
                        out.data_ptr(), ws.data_ptr(), ws.numel(),
                        torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.sk_last_error()
    return out


def _lse_col_noalloc(lib, C, f, eps):
    B, N, M = C.shape
    out = torch.empty(B, M, device=C.device, dtype=torch.float32)
    rc = lib.sk_lse_col_noalloc(C.data_ptr(), B, N, M, *C.stride(), f.data_ptr(),
                                float(eps), out.data_ptr(),
                                torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.sk_last_error()
    return out


def test_noalloc_matches_workspace_entry_point_on_two_calls_in_a_row():
    lib = _lib()
    torch.cuda.set_device(0)
    gen = torch.Generator(device="cuda").manual_seed(7)
    for shape, eps in (((1, 2048, 4096), 0.05), ((3, 300, 1000), 0.5)):
        B, N, M = shape
        C = torch.rand(shape, device="cuda", generator=gen)
        f = 0.1 * torch.randn(B, N, device="cuda", generator=gen)
        got = _lse_col_noalloc(lib, C, f, eps)
        ref = _lse_col_workspace(lib, C, f, eps)
        torch.cuda.synchronize()
        np.testing.assert_allclose(got.cpu().numpy(), ref.cpu().numpy(),
                                   atol=2e-5 * max(1.0, eps), rtol=1e-5)


def test_noalloc_rejects_problems_larger_than_its_scratch():
    lib = _lib()
    small = torch.zeros(4, device="cuda")
    # B=1024, N=M=2048 needs ~8.25 MiB of scratch; rejected before any launch
    rc = lib.sk_lse_col_noalloc(small.data_ptr(), 1024, 2048, 2048, 2048 * 2048, 2048, 1,
                                small.data_ptr(), 0.1, small.data_ptr(),
                                torch.cuda.current_stream().cuda_stream)
    assert rc == 3  # SK_ERR_WORKSPACE
    assert b"8 MiB" in lib.sk_last_error()
