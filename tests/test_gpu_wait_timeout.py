"""Bounded device-side waits end with an error instead of hanging.

Every pipelined kernel here waits on mbarriers (its own copies, its peer CTA
in a cluster) or on a grid barrier, and every such wait gives up after a
bounded number of polls, records error 2 in its status and returns, which the
host reports as SK_ERR_TIMEOUT. sk_probe_wait_timeout runs the same wait
primitives with a short poll limit against a partner that never arrives (a
flag that nothing sets): the call must return SK_ERR_TIMEOUT promptly and the
context must stay usable. With the partner present the same waits complete.
"""

from __future__ import annotations

import time

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

SK_ERR_TIMEOUT = 6
KINDS = {0: "local mbarrier", 1: "cluster peer st.async", 2: "grid barrier"}


def _probe(kind, partner, polls):
    from sinkhorn_b200 import _tensors as T
    lib = T.lib()
    n = int(lib.sk_probe_wait_scratch_bytes())
    scratch = torch.zeros(n, dtype=torch.uint8, device="cuda")
    rc = lib.sk_probe_wait_timeout(kind, partner, polls, scratch.data_ptr(), n,
                                   torch.cuda.current_stream().cuda_stream)
    return rc, lib.sk_last_error()


@pytest.mark.parametrize("kind", sorted(KINDS))
def test_wait_without_partner_times_out_and_returns(kind):
    t0 = time.time()
    rc, msg = _probe(kind, 0, 2000)
    assert rc == SK_ERR_TIMEOUT, (KINDS[kind], rc, msg)
    assert b"gave up" in msg
    assert time.time() - t0 < 30.0
    # the same wait completes when its partner arrives
    rc, msg = _probe(kind, 1, 1 << 20)
    assert rc == 0, (KINDS[kind], rc, msg)


def test_context_is_usable_after_a_timeout():
    from sinkhorn_b200.cuda.forward import sinkhorn_forward_cuda
    from oracle import oracle as O
    rc, _ = _probe(1, 0, 1000)
    assert rc == SK_ERR_TIMEOUT
    C = np.random.default_rng(0).random((1, 64, 8192), dtype=np.float32)
    f, g, n, conv = sinkhorn_forward_cuda(torch.from_numpy(C).cuda(), epsilon=0.1,
                                          max_iters=20, threshold=0.0)
    fo, go, _, _ = O.forward(C, epsilon=0.1, max_iters=20, threshold=0.0, check_every=10)
    assert n == 20
    np.testing.assert_allclose(f.cpu().numpy(), fo, atol=1e-4, rtol=2e-6)
    np.testing.assert_allclose(g.cpu().numpy(), go, atol=1e-4, rtol=2e-6)
