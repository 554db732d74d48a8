"""Multi-GPU check of the sharded drivers, run under torchrun (one rank per GPU).

Every rank builds the same seeded problems, solves its shard with the
drivers in sinkhorn_b200.distributed (NCCL), and rank 0 compares the gathered
result with the one-GPU solve. Exit code 0 on agreement. Used by
tests/test_gpu_distributed.py when two or more GPUs are visible:

    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 \
        --master-port 29511 tests/dist_check.py
"""

from __future__ import annotations

import datetime
import os
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))


def main() -> int:
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    P, rank = dist.get_world_size(), dist.get_rank()
    from sinkhorn_b200.cuda.forward import sinkhorn_forward_cuda
    from sinkhorn_b200.distributed import sinkhorn_batch_sharded, sinkhorn_row_sharded

    ok = True
    gen = torch.Generator().manual_seed(0)
    # row sharded: masked, unbalanced problems, uneven shards, every merge
    # (the peer exchange on the single-read shape; the two-sweep shape falls
    # back to the all-gather); a two-sweep shape and a single-read one
    from conftest import check_forward_parity
    for (B, N, M, iters, thr) in ((2, 1000, 772, 300, 1e-6), (1, 1000, 8192, 40, 0.0)):
        C = torch.randn(B, N, M, generator=gen).to(dev)
        ma = (torch.rand(B, N, generator=gen) > 0.1).to(dev)
        mb = (torch.rand(B, M, generator=gen) > 0.1).to(dev)
        cuts = [round(N * r / P) for r in range(P + 1)]
        rows = slice(cuts[rank], cuts[rank + 1])
        for merge in ("allreduce", "gather", "peer"):
            f, g, n, conv = sinkhorn_row_sharded(C[:, rows].contiguous(), None, None, 0.2, 1.0,
                                                 None, ma[:, rows].contiguous(), mb, iters,
                                                 thr, 10, merge=merge)
            f_all = [torch.empty(B, cuts[r + 1] - cuts[r], device=dev) for r in range(P)]
            dist.all_gather(f_all, f.contiguous())
            if rank == 0:
                fr, gr, nr, cr = sinkhorn_forward_cuda(C, None, None, 0.2, 1.0, None, ma, mb,
                                                       iters, thr)
                err_f = (torch.cat(f_all, 1) - fr).abs().max().item()
                err_g = (g - gr).abs().max().item()
                print(f"row-sharded {merge} P={P} M={M}: n={n}/{nr} conv={conv}/{cr} "
                      f"|df|={err_f:.2e} |dg|={err_g:.2e}")
                # both against the oracle, each at the count it reports
                p = dict(C=C.cpu().numpy(), eps=0.2, tau_a=1.0, tau_b=None,
                         mask_a=ma.cpu().numpy(), mask_b=mb.cpu().numpy(), max_iters=iters,
                         threshold=thr, check_every=10)
                try:
                    out = check_forward_parity(torch.cat(f_all, 1), g, n, conv, p)
                    check_forward_parity(fr, gr, nr, cr, p, oracle_out=out)
                except AssertionError as e:
                    print(f"row-sharded parity failed: {e}")
                    ok = False
    # batch sharded: P*2 items, two per rank
    Cb = torch.randn(2 * P, 300, 300, generator=gen).to(dev)
    mine = Cb[2 * rank:2 * rank + 2].contiguous()
    f, g, n, conv = sinkhorn_batch_sharded(mine, None, None, 0.1, None, None, None, None,
                                           300, 1e-6, 10)
    ref = sinkhorn_forward_cuda(Cb, None, None, 0.1, None, None, None, None, 300, 1e-6)
    err = (f - ref[0][2 * rank:2 * rank + 2]).abs().max().item()
    t = torch.tensor([err, float(n != ref[2])], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    if rank == 0:
        print(f"batch-sharded P={P}: n={n}/{ref[2]} max|df|={t[0].item():.2e}")
        ok &= t[0].item() < 1e-5 and t[1].item() == 0.0
    flag = torch.tensor([int(ok)], device=dev)
    dist.broadcast(flag, 0)
    dist.destroy_process_group()
    return 0 if flag.item() else 1


if __name__ == "__main__":
    sys.exit(main())
