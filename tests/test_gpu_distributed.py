"""GPU tests of the sharded drivers (sinkhorn_b200.distributed) through the
sk_solver_* ABI: a single-rank NCCL group on one GPU, and -- when two or more
GPUs are visible -- a torchrun run of tests/dist_check.py on two ranks.

With one rank the peer exchange's finish waits only for the flag its own
merge kernel raised, and that kernel has completed before the finish's wait
begins (the finish waits for its predecessor first), so no kernel waits for
another one running on the same GPU."""

from __future__ import annotations

import datetime
import os
import socket
import subprocess
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist

from conftest import ROOT, check_forward_parity

pytestmark = pytest.mark.gpu


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.fixture
def single_rank_group():
    torch.cuda.set_device(0)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{_port()}", rank=0,
                            world_size=1, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", 0))
    yield
    dist.destroy_process_group()


@pytest.mark.parametrize("merge", ["allreduce", "gather", "peer"])
@pytest.mark.parametrize("B,N,M,masked", [
    (2, 300, 260, False),    # two sweeps per iteration on the rank's rows
    (2, 300, 260, True),
    (1, 300, 8192, True),    # the single-read step and the chunk merge
    (1, 200, 32768, False),  # single read on 4-CTA clusters
])
def test_row_sharded_single_rank_matches_forward(single_rank_group, merge, B, N, M, masked):
    from sinkhorn_b200.cuda.forward import sinkhorn_forward_cuda
    from sinkhorn_b200.distributed import sinkhorn_row_sharded
    gen = torch.Generator().manual_seed(1)
    C = torch.rand(B, N, M, generator=gen).cuda()
    ma = (torch.rand(B, N, generator=gen) > 0.2).cuda() if masked else None
    mb = (torch.rand(B, M, generator=gen) > 0.2).cuda() if masked else None
    f, g, n, conv = sinkhorn_row_sharded(C, None, None, 0.05, 1.0, None, ma, mb, 200, 1e-6,
                                         10, merge=merge)
    fr, gr, nr, cr = sinkhorn_forward_cuda(C, None, None, 0.05, 1.0, None, ma, mb, 200, 1e-6)
    # both against the oracle, each at the count it reports (the sharded merge
    # sums in another order, so a stop inside the fp32 band of the threshold
    # may land one check apart; anything else fails)
    p = dict(C=C.cpu().numpy(), eps=0.05, tau_a=1.0, tau_b=None,
             mask_a=None if ma is None else ma.cpu().numpy(),
             mask_b=None if mb is None else mb.cpu().numpy(), max_iters=200,
             threshold=1e-6, check_every=10)
    out = check_forward_parity(f, g, n, conv, p)
    check_forward_parity(fr, gr, nr, cr, p, oracle_out=out)


def test_batch_sharded_single_rank_matches_forward(single_rank_group):
    from sinkhorn_b200.cuda.forward import sinkhorn_forward_cuda
    from sinkhorn_b200.distributed import sinkhorn_batch_sharded
    gen = torch.Generator().manual_seed(2)
    C = torch.randn(3, 128, 96, generator=gen).cuda()
    f, g, n, conv = sinkhorn_batch_sharded(C, None, None, 0.1, None, None, None, None, 300,
                                           1e-6, 10)
    fr, gr, nr, cr = sinkhorn_forward_cuda(C, None, None, 0.1, None, None, None, None, 300,
                                           1e-6)
    assert (n, conv) == (nr, cr)
    # the driver runs the sweep kernels, sk_forward the on-chip solver at this
    # size: same iterations, fp32 summation orders differ
    np.testing.assert_allclose(f.cpu().numpy(), fr.cpu().numpy(), atol=1e-5)
    np.testing.assert_allclose(g.cpu().numpy(), gr.cpu().numpy(), atol=1e-5)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_ranks_nccl():
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(_port()),
           os.path.join(ROOT, "tests", "dist_check.py")]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(["timeout", "-k", "30", "300"] + cmd, capture_output=True, text=True,
                       env=env)
    print(r.stdout[-3000:], r.stderr[-3000:])
    assert r.returncode == 0
