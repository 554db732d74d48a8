#!/usr/bin/env python
"""Sinkhorn iterations/sec on B200 (sm_100a) -- benchmark harness.

Default workload (one GPU): balanced Sinkhorn, B=1, N=M=16384, fp32,
C = squared distances of x, y ~ U[0,1]^{N x 3} divided by max(C), uniform
marginals, eps=0.05, threshold=0 so every solve runs exactly 100 iterations.
A step is one solve (100 iterations = 100 row sweeps + 100 column sweeps);
``value`` is whole-job Sinkhorn iterations per second with C resident in HBM.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl cuda|reference]

With N > 1 (launched by torchrun, one rank per GPU, NCCL) every rank solves its
own seeded problem of the same size (batch sharding, weak scaling); the
convergence test of a sharded batch is global (all-reduce MAX of the residual),
which a zero threshold never reaches.

``--impl reference`` times the reference's CPU algorithm (the C restatement in
oracle/, fp32, all host threads) on the same workload and metric.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "Sinkhorn iters/sec & C-sweep GB/s at B=1 N=M=16384 fp32; ms-to-converge; 1/2/4/8 GPU"
UNIT = "iter/s"
CONVERGE_THR = 1e-6  # the ms-to-converge measurement (check every 10 iterations)
SOLVE_KERNEL = "k_fused_iter (solve mode)"


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["cuda", "reference"], default="cuda")
    ap.add_argument("--n", type=int, default=16384, help="N = M of the workload")
    ap.add_argument("--iters", type=int, default=100, help="iterations per solve")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--dtype", choices=["f32", "bf16"], default="f32",
                    help="bf16: the default workload with C stored as bfloat16 (opt-in "
                         "input precision, fp32 arithmetic; one JSON line, single GPU)")
    ap.add_argument("--no-reference", action="store_true",
                    help="sweep/cfg3/cfg4: time this build only (not the reference beside it)")
    ap.add_argument("--merge", choices=["peer", "allreduce", "gather"], default="peer",
                    help="row-sharded runs: how the ranks merge their column LSEs each "
                         "iteration (stores into the other ranks' buffers over NVLink with "
                         "device-side flags; two NCCL all-reduces; one NCCL all-gather)")
    ap.add_argument("--scaling", choices=["weak", "strong"], default="weak",
                    help="N > 1 on the default workload: weak = a (16384 N) x 16384 problem "
                         "row-sharded one 16384 x 16384 block (1 GiB) per GPU; strong = the "
                         "one N=M=16384 problem row-sharded over the GPUs")
    ap.add_argument("--cpu-torch-iters", type=int, default=2,
                    help="iterations of the reference's own PyTorch CPU path timed beside "
                         "the C restatement (0: skip)")
    ap.add_argument("--cpu-seconds", type=float, default=15.0,
                    help="budget of the CPU-baseline sample")
    ap.add_argument("--workload", choices=["batch", "rowshard", "sweep", "cfg3", "cfg4",
                                           "implicit", "f1", "solve", "bwd", "mid"],
                    default="batch",
                    help="batch: the default workload above (one problem per GPU); "
                         "rowshard: one N=M=65536 problem (16 GiB C, x,y ~ U[0,1]^8, "
                         "eps=0.01, 50 iterations) split by rows over the GPUs; "
                         "sweep: N=M in {128, 1024, 4096, 16384} on one GPU, fixed 100 "
                         "iterations and ms-to-converge (threshold 1e-6), beside the "
                         "reference's Triton path when baseline/_ref holds it; "
                         "cfg3: B=64 N=M=1024 masked unbalanced forward; cfg4: B=16 "
                         "N=M=2048 differentiable forward + backward (grad_iters 10 and 0); "
                         "implicit: implicit_gradient (50 CG iterations) at B=16 N=M=2048 "
                         "and B=1 N=M=16384; f1: transport_plan, cost, marginal error and "
                         "the P-free JVP at the same two shapes; mid: rows of 2048 < M < 8192, "
                         "sk_forward against the two sweeps (with --profile: B=4 N=M=4096)")
    ap.add_argument("--grad-iters-profile", type=int, default=-1, metavar="G",
                    help="with --workload cfg4 --profile K: K whole differentiable steps "
                         "(forward, loss, backward) with grad_iters G instead of K iterations")
    ap.add_argument("--profile", type=int, default=0, metavar="K",
                    help="profiling case: build C, then only the solver prologue and K "
                         "iterations (a few launches, for ncu; --workload solve: one "
                         "persistent launch of K iterations); prints nothing")
    return ap.parse_args(argv)


def run_profile_case(args):
    """A short, self-contained launch sequence for ncu captures: input
    generation, one sk_solver_init and K iterations of the default workload;
    with --workload cfg3, K single-read iterations of the masked batch; with
    --workload implicit, one implicit_gradient call of K CG iterations at
    B=16, N=M=2048 (C ~ U[0,1), f = g = 0, eps = 1); with --workload cfg4,
    K single-read iterations (k_rows_fused + k_col_finish) of the balanced
    B=16, N=M=2048 solve (C = squared distances of U[0,1]^3 points over max,
    eps = 0.05)."""
    import torch
    from sinkhorn_b200.cuda.solver import SinkhornSolver
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    if args.workload == "implicit":
        from sinkhorn_b200 import implicit_diff as I
        gen = torch.Generator(device=dev).manual_seed(0)
        B, n = 16, 2048
        C = torch.rand(B, n, n, device=dev, generator=gen)
        f = torch.zeros(B, n, device=dev)
        gf = torch.randn(B, n, device=dev, generator=gen)
        I.implicit_gradient(C, f, f, gf, gf, 1.0, None, None, None, None, args.profile, 0.0)
        torch.cuda.synchronize()
        return
    if args.workload == "bwd":
        # one truncated backward of K iterations at B=16, N=M=2048 (its
        # single-read recompute steps, single-read reverse steps and the dC pass)
        from sinkhorn_b200.autograd import sinkhorn_backward_cuda
        gen = torch.Generator(device=dev).manual_seed(0)
        x = torch.randn(16, 2048, 16, device=dev, generator=gen)
        y = torch.randn(16, 2048, 16, device=dev, generator=gen)
        C = torch.cdist(x, y).pow(2)
        C = C / C.mean()
        f = torch.zeros(16, 2048, device=dev)
        gf = torch.randn(16, 2048, device=dev, generator=gen)
        sinkhorn_backward_cuda(C, None, None, 1.0, None, None, None, None, 100, 1e-6,
                               args.profile, f, f, gf, gf)
        torch.cuda.synchronize()
        return
    if args.workload == "rowshard":
        # one rank's shard of the row-sharded N=M=65536 problem at 8 ranks
        # (8192 rows x 65536 columns, 2 GiB): K single-read iterations on
        # 8-CTA clusters + k_col_finish
        n = 65536
        gen = torch.Generator(device=dev).manual_seed(99)
        x = torch.rand(n // 8, 8, device=dev, generator=gen)
        y = torch.rand(n, 8, device=dev, generator=gen)
        C = torch.empty(1, n // 8, n, device=dev)
        for s0 in range(0, n // 8, 2048):
            C[0, s0:s0 + 2048] = torch.cdist(x[s0:s0 + 2048], y).pow_(2)
        C.div_(C.max())
        solver = SinkhornSolver(C, epsilon=ROWSHARD_EPS, max_iters=10 ** 9, threshold=0.0)
        solver.iterate(args.profile, fused=True)
        torch.cuda.synchronize()
        return
    if args.workload == "mid":
        # K single-read iterations on one-CTA units (k_fused_iter with the whole
        # row in one CTA + k_col_finish): B=4, N=M=4096 (256 MiB of C)
        gen = torch.Generator(device=dev).manual_seed(0)
        x = torch.rand(4, 4096, 3, device=dev, generator=gen)
        y = torch.rand(4, 4096, 3, device=dev, generator=gen)
        C = torch.cdist(x, y).pow(2)
        C = C / C.amax()
        solver = SinkhornSolver(C, epsilon=EPS, max_iters=10 ** 9, threshold=0.0)
        solver.iterate(args.profile, fused=True)
        torch.cuda.synchronize()
        return
    if args.workload == "cfg3":
        # K single-read iterations (k_row_warps + k_col_finish) of the masked,
        # unbalanced batch (the cfg3 leg's inputs)
        C, a, b, mask_a, mask_b = (t.to(dev) for t in _cfg3_inputs())
        solver = SinkhornSolver(C, a, b, 0.1, 1.0, 1.0, mask_a, mask_b, max_iters=10 ** 9,
                                threshold=0.0)
        solver.iterate(args.profile, fused=True)
        torch.cuda.synchronize()
        return
    if args.workload == "cfg4" and args.grad_iters_profile >= 0:
        # K full differentiable steps of the cfg4 leg (sinkhorn_differentiable
        # forward, the loss sum(P * C), backward to dC) after two warm-up steps
        from sinkhorn_b200.autograd import sinkhorn_differentiable
        gen = torch.Generator().manual_seed(0)
        x = torch.randn(16, 2048, 16, generator=gen)
        y = torch.randn(16, 2048, 16, generator=gen)
        C0 = torch.cdist(x, y).pow(2)
        C0 = (C0 / C0.mean()).to(dev)
        for _ in range(2 + args.profile):
            C = C0.clone().requires_grad_(True)
            f, g = sinkhorn_differentiable(C, epsilon=1.0, grad_iters=args.grad_iters_profile)
            (torch.exp(f[:, :, None] + g[:, None, :] - C) * C).sum().backward()
        torch.cuda.synchronize()
        return
    if args.workload == "cfg4":
        gen = torch.Generator(device=dev).manual_seed(0)
        x = torch.rand(16, 2048, 3, device=dev, generator=gen)
        y = torch.rand(16, 2048, 3, device=dev, generator=gen)
        C = torch.cdist(x, y).pow(2)
        C = C / C.amax()
        solver = SinkhornSolver(C, epsilon=EPS, max_iters=10 ** 9, threshold=0.0)
        solver.iterate(args.profile, fused=True)
        torch.cuda.synchronize()
        return
    C = make_cost_gpu(args.n, seed=1234, device=dev)
    if args.workload == "solve":
        # the persistent solve: one k_init and one solve-mode launch of K iterations
        solver = SinkhornSolver(C, epsilon=EPS, max_iters=args.profile, threshold=0.0)
        solver.solve()
        torch.cuda.synchronize()
        return
    solver = SinkhornSolver(C, epsilon=EPS, max_iters=10 ** 9, threshold=0.0)
    solver.iterate(args.profile)
    torch.cuda.synchronize()


# ---------------------------------------------------------------------------
# workload

EPS = 0.05


def make_cost_gpu(n: int, seed: int, device):
    import torch
    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.rand(n, 3, device=device, generator=g)
    y = torch.rand(n, 3, device=device, generator=g)
    C = torch.cdist(x, y).pow_(2)
    C.div_(C.max())
    return C.unsqueeze(0).contiguous()


def make_cost_cpu(n: int, seed: int):
    import torch
    g = torch.Generator().manual_seed(seed)
    x = torch.rand(n, 3, generator=g)
    y = torch.rand(n, 3, generator=g)
    C = torch.cdist(x, y).pow_(2)
    C.div_(C.max())
    return C.unsqueeze(0).contiguous()


def workload_config(args, n_gpus):
    return {
        "workload": f"balanced Sinkhorn B=1 N=M={args.n} fp32 per GPU, C=sqdist(U[0,1]^3)/max, "
                    f"uniform marginals, eps={EPS}, threshold=0, {args.iters} iterations per solve",
        "B": 1, "N": args.n, "M": args.n, "epsilon": EPS, "iters_per_solve": args.iters,
        "parallelism": f"batch-sharded x{n_gpus}" if n_gpus > 1 else "single GPU",
        "l2": f"inputs larger than L2: C is {4 * args.n * args.n / 2**30:.2f} GiB per GPU"
              if 4 * args.n * args.n > 126e6 else "C fits in L2 (no flush)",
    }


def weak_rowshard_workload(n, world, iters):
    """The weak row-sharded problem of `world` GPUs: one n x n block per GPU."""
    gib = 4 * n * n / 2**30
    return {"workload": f"balanced Sinkhorn B=1, N={n * world} x M={n} fp32 row-sharded one "
                        f"{n} x {n} block ({gib:.2f} GiB of C) per GPU, C=sqdist(U[0,1]^3)/max, "
                        f"uniform marginals, eps={EPS}, threshold=0, {iters} iterations per "
                        f"solve; value = {n} x {n} block-iterations per second, all GPUs",
            "N": n * world}


# ---------------------------------------------------------------------------
# clocks sampled during the timed region

REASONS = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]


class ClockSampler:
    def __init__(self, device_index: int, uuid: str | None):
        self.sel = uuid if uuid else str(device_index)
        self.rows: list[list[str]] = []
        self.proc = None
        self.thread = None

    def __enter__(self):
        q = ("clocks.sm,clocks.max.sm,power.draw,"
             + ",".join(f"clocks_event_reasons.{r}" for r in REASONS))
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.sel, f"--query-gpu={q}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            # nvidia-smi takes a moment to emit its first row: start the timed
            # region only once sampling is live (bounded wait)
            t0 = time.time()
            while not self.rows and time.time() - t0 < 5.0 and self.proc.poll() is None:
                time.sleep(0.02)
            self.rows.clear()
        except (OSError, ValueError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            if self.thread is not None:
                self.thread.join(timeout=5)

    def summary(self) -> dict:
        sm, mx, reasons = [], [], set()
        for r in self.rows:
            try:
                sm.append(float(r[0]))
                mx.append(float(r[1]))
            except (ValueError, IndexError):
                continue
            for name, val in zip(REASONS, r[3:]):
                if val.strip().lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx),
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# peaks and ncu-measured traffic (committed summaries)

def hbm_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as fh:
            return float(json.load(fh)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def ncu_traffic(kernel: str, n: int):
    """DRAM bytes per launch of `kernel` at N=M=n from profiles/ncu_traffic.json."""
    p = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    try:
        with open(p) as fh:
            d = json.load(fh)
        return d.get(f"{kernel}@{n}")
    except (OSError, ValueError):
        return None


# ---------------------------------------------------------------------------

def run_cuda(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1:
        return run_cuda_sharded(args)
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.gpus != world:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE={world}; using {world}",
              file=sys.stderr)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=dev)

    from sinkhorn_b200 import sinkhorn
    from sinkhorn_b200.cuda.forward import sinkhorn_forward_cuda
    from sinkhorn_b200.cuda.solver import SinkhornSolver, ex2_rate

    n, iters = args.n, args.iters
    ex2_per_s = ex2_rate(dev)  # the exponential floor, measured on this GPU now
    C = make_cost_gpu(n, seed=1234 + rank, device=dev)
    torch.cuda.synchronize()

    def solve():
        return sinkhorn_forward_cuda(C, None, None, EPS, None, None, None, None, iters, 0.0)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(max(args.warmup, 3)):
        f, g, n_it, _ = solve()
    assert n_it == iters
    torch.cuda.synchronize()

    # ---- headline: device-resident C, CUDA events, max over ranks ------
    uuid = None
    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:  # noqa: BLE001 - older torch has no uuid
        uuid = None
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local, uuid) as clocks:
        e0.record()
        for _ in range(args.steps):
            solve()
        e1.record()
        torch.cuda.synchronize()
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1))
    ms_per_step = ms / args.steps
    value = world * args.steps * iters / (ms / 1e3)
    sweep_gbs = world * args.steps * iters * 8.0 * n * n / (ms / 1e3) / 1e9

    # ---- the dominant kernel's duration (roofline) on its launching stream
    c_bytes = 4.0 * n * n  # one read of C (vectors and partials are negligible)
    peak, peak_kind = hbm_peak()
    stream = torch.cuda.current_stream(dev)
    kernels = {}
    # the step kernels of one iteration (sk_solver_fused_step / _finish, or
    # the two sweeps), each timed on the stream it runs on
    R = 20
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(R)]
    step = SinkhornSolver(C, epsilon=EPS, max_iters=10 ** 9, threshold=0.0)
    step.iterate(2)
    torch.cuda.synchronize()
    fused = step.forward_fused
    first, second = ((step.fused_step, step.fused_finish) if fused
                     else (step.row_sweep, step.col_sweep))
    for r in range(R):
        evs[r][0].record(stream)
        first()
        evs[r][1].record(stream)
        second()
        evs[r][2].record(stream)
    torch.cuda.synchronize()
    a_ms = max_over_ranks(sum(e[0].elapsed_time(e[1]) for e in evs) / R)
    b_ms = max_over_ranks(sum(e[1].elapsed_time(e[2]) for e in evs) / R)
    if fused:
        kernels["k_fused_iter"] = {"ms": a_ms, "GB/s": c_bytes / (a_ms / 1e3) / 1e9,
                                   "role": "one single-read step (sk_solver_fused_step)"}
        kernels["k_col_finish"] = {"ms": b_ms, "GB/s": None,
                                   "role": "its chunk merge (sk_solver_fused_finish); in the "
                                           "solve it overlaps the next step's start "
                                           "(programmatic dependent launch)"}
    else:
        kernels["k_row_sweep"] = {"ms": a_ms, "GB/s": c_bytes / (a_ms / 1e3) / 1e9}
        kernels["k_col_sweep"] = {"ms": b_ms, "GB/s": c_bytes / (b_ms / 1e3) / 1e9}
    if step.persist:
        # the opt-in one-launch solve (sk_solver_solve), not on sk_forward's
        # path: K iterations in one persistent launch of k_fused_iter, timed
        # alone after its k_init, for comparison with the loop
        solver = SinkhornSolver(C, epsilon=EPS, max_iters=iters, threshold=0.0)
        durs = []
        for r in range(6):
            solver.init()
            ea = torch.cuda.Event(enable_timing=True)
            eb = torch.cuda.Event(enable_timing=True)
            ea.record(stream)
            solver.solve()
            eb.record(stream)
            torch.cuda.synchronize()
            if r:
                durs.append(ea.elapsed_time(eb))
        k_ms = max_over_ranks(sum(durs) / len(durs))
        kernels[SOLVE_KERNEL] = {
            "ms": k_ms, "iterations_per_launch": iters, "ms_per_iteration": k_ms / iters,
            "GB/s": c_bytes * iters / (k_ms / 1e3) / 1e9,
            "role": "opt-in sk_solver_solve, not what sk_forward runs"}
        del solver
    dom = "k_fused_iter" if fused else max(("k_row_sweep", "k_col_sweep"),
                                            key=lambda k: kernels[k]["ms"])
    iter_bytes = c_bytes if fused else 2 * c_bytes
    # the whole iteration as the timed solve runs it (init and the status
    # read-back included, spread over its iterations)
    iter_ms = ms_per_step / iters
    launch_bytes = c_bytes
    achieved = kernels[dom]["GB/s"]
    roofline = {"bound": "hbm", "kernel": dom, "achieved": round(achieved, 1),
                "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind ==
                "measured" else "fallback 6.65 TB/s",
                "algorithmic_bytes_per_launch": launch_bytes,
                "algorithmic_model": "one read of C (4*N*M bytes) per launch",
                "traffic": ncu_traffic(dom, n),
                "iteration_ms": round(iter_ms, 4),
                "iteration_ms_source": "ms_per_solve / iterations (the timed solves)",
                "iteration_frac": round(iter_bytes / (iter_ms / 1e3) / 1e9 / peak, 4),
                "iteration_model": "one read of C per iteration (fused)" if fused else
                                   "two reads of C per iteration (row + column sweep)",
                # the iteration's two floors: bytes at the HBM peak and its 2*N*M
                # exponentials at the ex2 rate measured live (sk_probe_ex2_rate)
                "ex2_per_s": round(ex2_per_s, -6),
                "floor_ms_hbm": round(iter_bytes / (peak * 1e9) * 1e3, 4),
                "floor_ms_ex2": round(2.0 * n * n / ex2_per_s * 1e3, 4),
                "iteration_floor_frac": round(
                    max(iter_bytes / (peak * 1e9), 2.0 * n * n / ex2_per_s) * 1e3 / iter_ms, 4)}
    for k in kernels:
        if kernels[k]["GB/s"] is not None:
            kernels[k]["frac"] = round(kernels[k]["GB/s"] / peak, 4)
            kernels[k]["GB/s"] = round(kernels[k]["GB/s"], 1)
        for key in ("ms", "ms_per_iteration"):
            if key in kernels[k]:
                kernels[k][key] = round(kernels[k][key], 4)
    del step

    # ---- ms-to-converge: the same problem at threshold 1e-6 -------------
    def converge():
        return sinkhorn_forward_cuda(C, None, None, EPS, None, None, None, None, 5000,
                                     CONVERGE_THR)

    conv_ms, (_, _, conv_n, conv_ok) = _events_ms(converge, 5, warm=1)
    conv_ms = max_over_ranks(conv_ms)
    ms_to_converge = {"ms": round(conv_ms, 3), "n_iters": conv_n, "converged": bool(conv_ok),
                      "threshold": CONVERGE_THR, "check_every": 10,
                      "timed": "one sinkhorn_forward_cuda call (init, solve, status "
                               "read-back), C resident; CUDA events, mean of 5"}

    # ---- e2e: pinned host C -> device, public API, f/g -> host ----------
    # Every step copies its own C from pinned host memory and reads f, g
    # back. The copies are double-buffered: step k+1's host-to-device copy
    # runs on a copy stream while step k solves (what a serving pipeline
    # does); the first step's copy is inside the timed region too.
    e2e = None
    if not args.no_e2e:
        C_host = C.cpu().pin_memory()
        C_dev = [torch.empty_like(C), torch.empty_like(C)]
        f_host = torch.empty(1, n, dtype=torch.float32).pin_memory()
        g_host = torch.empty(1, n, dtype=torch.float32).pin_memory()
        main = torch.cuda.current_stream(dev)
        copy_stream = torch.cuda.Stream(dev)
        ev_copied = [torch.cuda.Event(), torch.cuda.Event()]
        ev_used = [torch.cuda.Event(), torch.cuda.Event()]

        def copy_in(k):
            with torch.cuda.stream(copy_stream):
                if k >= 2:
                    copy_stream.wait_event(ev_used[k % 2])  # step k-2 is done with it
                C_dev[k % 2].copy_(C_host, non_blocking=True)
                ev_copied[k % 2].record(copy_stream)

        def e2e_steps(k_steps):
            copy_in(0)
            for k in range(k_steps):
                if k + 1 < k_steps:
                    copy_in(k + 1)
                main.wait_event(ev_copied[k % 2])
                out = sinkhorn(C_dev[k % 2], epsilon=EPS, max_iters=iters, threshold=0.0)
                ev_used[k % 2].record(main)
                f_host.copy_(out.f, non_blocking=True)
                g_host.copy_(out.g, non_blocking=True)

        e2e_steps(2)
        torch.cuda.synchronize()
        k_e2e = max(3, min(args.steps, 10))
        barrier()
        torch.cuda.synchronize()
        e0.record()
        e2e_steps(k_e2e)
        e1.record()
        torch.cuda.synchronize()
        barrier()
        ms_e2e = max_over_ranks(e0.elapsed_time(e1))
        e2e = {"value": round(world * k_e2e * iters / (ms_e2e / 1e3), 2), "unit": UNIT,
               "h2d_bytes_per_step": C_host.numel() * 4,
               "d2h_bytes_per_step": (f_host.numel() + g_host.numel()) * 4,
               "ms_per_step": round(ms_e2e / k_e2e, 3),
               "api": "sinkhorn_b200.sinkhorn (C ABI sk_forward)",
               "pipeline": "double-buffered: step k+1's host-to-device copy (copy stream) "
                           "overlaps step k's solve; every step's copy is timed"}
        C_dev = None
    else:
        C_host = None

    # ---- CPU baseline (rank 0, one GPU only) ------------------------------
    cpu = cpu_torch = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        if C_host is None:
            C_host = C.cpu()
        cpu = cpu_sample(C_host.numpy(), args.cpu_seconds)
        cpu_torch = cpu_reference_torch(C_host, args.cpu_torch_iters)

    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": max(args.warmup, 3),
        "ms_per_step": round(ms_per_step, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(args, world),
        "c_sweep_gbs": round(sweep_gbs / 2 if fused else sweep_gbs, 1),
        "c_sweep_gbs_model": "bytes of C actually read per second: one read of C per "
                             "iteration (fused)" if fused else
                             "bytes of C actually read per second: two reads per iteration",
        "c_sweep_gbs_two_read_equivalent": round(sweep_gbs, 1),
        "c_sweep_gbs_two_read_equivalent_model": "8*N*M bytes per iteration, the two sweeps "
                                                 "the reference's row + column passes read; "
                                                 "not a physical bandwidth",
        "ms_per_solve": round(ms_per_step, 4),
        "ms_to_converge": ms_to_converge,
        "roofline": roofline, "kernels": kernels, "cpu_baseline": cpu,
        "cpu_reference_torch": cpu_torch, "e2e": e2e,
        "clocks": clocks.summary(),
        "gpu_launches": args.steps * (1 + 2 * iters),
        "iteration_kernels": ("fused single read (k_fused_iter + k_col_finish, chained by "
                              "programmatic dependent launch)" if fused else
                              "row sweep + column sweep"),
    }
    print(json.dumps(line))


SWEEP_SIZES = (128, 1024, 4096, 16384)
SWEEP_THR = 1e-6
SWEEP_MAX_ITERS = 5000  # bounds the reference's converge run (~2.8 ms/iteration at 16384)


def run_sweep(args):
    """cfg2's size sweep on one GPU: per size, iterations/s of a fixed
    100-iteration solve and the time to converge at threshold 1e-6 (check
    every 10 iterations), with C resident; the same for the reference's own
    Triton path (sinkhorn.triton.forward, installed under baseline/_ref) when
    it is importable, with the largest potential difference between the two.
    One JSON line per size (informational: the driver's reference arm is the
    CPU restatement, --impl reference)."""
    import torch
    from sinkhorn_b200.cuda.forward import sinkhorn_forward_cuda
    ref = None
    ref_dir = os.path.join(ROOT, "baseline", "_ref")
    if os.path.isdir(ref_dir) and not args.no_reference:
        sys.path.insert(0, ref_dir)
        try:
            from sinkhorn.triton.forward import sinkhorn_forward_triton as ref
        except Exception as exc:  # noqa: BLE001 - report, keep measuring our side
            print(f"reference Triton path unavailable: {exc}", file=sys.stderr)
            ref = None
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)

    def timed(fn, reps, warm=2):
        for _ in range(warm):
            out = fn()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            out = fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps, out

    for n in SWEEP_SIZES:
        C = make_cost_gpu(n, seed=1234, device=dev)
        reps = 3 if n >= 16384 else 10
        line = {"workload": "sweep", "N": n, "M": n, "B": 1, "epsilon": EPS, "dtype": "f32",
                "data": "synthetic", "C_bytes": 4 * n * n,
                "c_resident": "C fits in L2" if 4 * n * n <= 126e6 else "C larger than L2"}
        fixed = lambda: sinkhorn_forward_cuda(C, None, None, EPS, None, None, None, None,  # noqa: E731
                                              100, 0.0)
        conv = lambda: sinkhorn_forward_cuda(C, None, None, EPS, None, None, None, None,  # noqa: E731
                                             SWEEP_MAX_ITERS, SWEEP_THR)
        ms, (f, g, _, _) = timed(fixed, reps)
        ms_c, (_, _, n_c, ok_c) = timed(conv, 1 if n >= 16384 else 3, warm=1)
        line["sinkhorn_b200"] = {"ms_per_100_iterations": round(ms, 4),
                                 "iterations_per_s": round(100 / ms * 1e3, 1),
                                 "ms_to_converge": round(ms_c, 3), "n_iters": n_c,
                                 "converged": bool(ok_c)}
        if ref is not None:
            rfix = lambda: ref(C, None, None, EPS, None, None, None, None, 100, 0.0)  # noqa: E731
            rconv = lambda: ref(C, None, None, EPS, None, None, None, None,  # noqa: E731
                                SWEEP_MAX_ITERS, SWEEP_THR)
            rms, (fr, gr, _, _) = timed(rfix, reps)
            rms_c, (_, _, rn_c, rok_c) = timed(rconv, 1, warm=1)
            line["reference_triton"] = {"ms_per_100_iterations": round(rms, 4),
                                        "iterations_per_s": round(100 / rms * 1e3, 1),
                                        "ms_to_converge": round(rms_c, 3), "n_iters": rn_c,
                                        "converged": bool(rok_c)}
            line["speedup_fixed"] = round(rms / ms, 2)
            line["speedup_to_converge"] = round(rms_c / ms_c, 2)
            line["max_abs_df"] = float((f - fr).abs().max())
            line["max_abs_dg"] = float((g - gr).abs().max())
        print(json.dumps(line), flush=True)
        del C


def _reference_module(name: str):
    """The reference package installed under baseline/_ref, or None."""
    ref_dir = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(ref_dir):
        return None
    if ref_dir not in sys.path:
        sys.path.insert(0, ref_dir)
    try:
        import importlib
        return importlib.import_module(name)
    except Exception as exc:  # noqa: BLE001 - report, keep measuring our side
        print(f"reference module {name} unavailable: {exc}", file=sys.stderr)
        return None


def _events_ms(fn, reps, warm=2):
    import torch
    out = None
    for _ in range(warm):
        out = fn()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        out = fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps, out


def run_mid(args):
    """Rows of 2048 < M < 8192 (the one-CTA single read): per shape, sk_forward
    (100 iterations, threshold 0) against the two sweeps it ran there before
    (the same solver stepping row and column sweeps), C = squared distances of
    U[0,1]^3 points over the max, eps = 0.05; best of 3 after a warm-up."""
    import torch
    from sinkhorn_b200.cuda.forward import sinkhorn_forward_cuda
    from sinkhorn_b200.cuda.solver import SinkhornSolver, plan_query
    dev = torch.device("cuda", 0)
    it = 100
    for (B, N, M) in ((16, 2048, 2560), (16, 2048, 4096), (4, 4096, 4096), (1, 65536, 4096),
                      (8, 3000, 3000), (1, 4096, 2052), (64, 512, 3072), (2, 8192, 7168),
                      (1, 2000, 6000)):
        gen = torch.Generator(device=dev).manual_seed(0)
        x = torch.rand(B, N, 3, device=dev, generator=gen)
        y = torch.rand(B, M, 3, device=dev, generator=gen)
        C = torch.cdist(x, y).pow_(2)
        C.div_(C.amax())
        C = C.contiguous()

        def fwd():
            return sinkhorn_forward_cuda(C, None, None, EPS, None, None, None, None, it, 0.0)

        solver = SinkhornSolver(C, epsilon=EPS, max_iters=10 ** 9, threshold=0.0)

        def sweeps():
            solver.init()
            solver.iterate(it, fused=False)

        t1 = min(_events_ms(fwd, 1, warm=1 if r == 0 else 0)[0] for r in range(3)) / it
        t2 = min(_events_ms(sweeps, 1, warm=1 if r == 0 else 0)[0] for r in range(3)) / it
        q = plan_query(C)
        gbs = 4.0 * B * N * M / (t1 * 1e-3) / 1e9
        print(json.dumps({"workload": "mid", "B": B, "N": N, "M": M, "epsilon": EPS,
                          "iters": it, "sk_forward_us_per_iter": round(t1 * 1e3, 1),
                          "two_sweeps_us_per_iter": round(t2 * 1e3, 1),
                          "speedup": round(t2 / t1, 2), "one_read_GBps": round(gbs),
                          "single_read": bool(q["forward_fused"]), "chunks": q["chunks"]}),
              flush=True)
        del solver, C
        torch.cuda.empty_cache()


def run_bf16(args):
    """The default workload with C stored as bfloat16 (sk_forward_bf16): the
    same solve on the widened costs, half the bytes of C per read. Reports
    iterations/s and the iteration's roofline (its two floors: C's bytes at
    the HBM peak, 2*N*M exponentials at the measured ex2 rate)."""
    import torch
    from sinkhorn_b200.cuda.forward import sinkhorn_forward_cuda
    from sinkhorn_b200.cuda.solver import ex2_rate, plan_query
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    n, iters = args.n, args.iters
    ex2_per_s = ex2_rate(dev)
    C32 = make_cost_gpu(n, seed=1234, device=dev)
    fused = plan_query(C32)["forward_fused"] and n % 16 == 0
    C = C32.to(torch.bfloat16)
    del C32

    def solve():
        return sinkhorn_forward_cuda(C, None, None, EPS, None, None, None, None, iters, 0.0)

    for _ in range(max(args.warmup, 3)):
        solve()
    torch.cuda.synchronize()
    with ClockSampler(0, None) as clocks:
        ms, _ = _events_ms(solve, args.steps, warm=0)
    peak, kind = hbm_peak()
    it_ms = ms / iters
    reads = 1 if fused else 2
    it_bytes = reads * 2.0 * n * n
    floor = max(it_bytes / (peak * 1e9), 2.0 * n * n / ex2_per_s) * 1e3
    print(json.dumps({
        "workload": "bf16", "metric": METRIC, "value": round(1e3 / it_ms, 2),
        "unit": UNIT, "n_gpus": 1, "steps": args.steps, "warmup": max(args.warmup, 3),
        "ms_per_solve": round(ms, 4), "dtype": "bf16 C, f32 arithmetic", "data": "synthetic",
        "config": dict(workload_config(args, 1), C_dtype="bfloat16"),
        "iteration_kernels": "fused single read" if fused else "row sweep + column sweep",
        "roofline": {"iteration_ms": round(it_ms, 4), "bytes_per_iteration": it_bytes,
                     "achieved_gbs": round(it_bytes / (it_ms * 1e-3) / 1e9, 1), "peak": peak,
                     "peak_source": kind, "floor_ms_hbm": round(it_bytes / (peak * 1e9) * 1e3, 4),
                     "floor_ms_ex2": round(2.0 * n * n / ex2_per_s * 1e3, 4),
                     "iteration_floor_frac": round(floor / it_ms, 4)},
        "clocks": clocks.summary()}), flush=True)


def _cfg3_inputs():
    """The masked, unbalanced batch on the CPU: B=64, N=M=1024, C ~ N(0,1),
    valid lengths ~ U{256..1024} (prefix masks), a, b = softmax over the
    valid entries (torch.Generator().manual_seed(0))."""
    import torch
    gen = torch.Generator().manual_seed(0)
    B, N, M = 64, 1024, 1024
    C = torch.randn(B, N, M, generator=gen)
    la = torch.randint(256, N + 1, (B,), generator=gen)
    lb = torch.randint(256, M + 1, (B,), generator=gen)
    mask_a = torch.arange(N)[None, :] < la[:, None]
    mask_b = torch.arange(M)[None, :] < lb[:, None]
    a = torch.softmax(torch.randn(B, N, generator=gen).masked_fill(~mask_a, float("-inf")), -1)
    b = torch.softmax(torch.randn(B, M, generator=gen).masked_fill(~mask_b, float("-inf")), -1)
    return C, a, b, mask_a, mask_b


def run_cfg3(args):
    """Unbalanced, masked, batched forward: B=64, N=M=1024, C ~ N(0,1), valid
    lengths ~ U{256..1024} (prefix masks), a, b = softmax over the valid
    entries, eps=0.1, tau_a=tau_b=1, max_iters=200, threshold=1e-6. Inputs
    from torch.Generator().manual_seed(0) on the CPU, then copied. Under
    torchrun the 64 items are split over the ranks (batch sharding, strong
    scaling): each check all-reduces the residual (MAX) so every rank stops at
    the same global iteration; time = max over ranks."""
    import torch
    import torch.distributed as dist
    from sinkhorn_b200.cuda.forward import sinkhorn_forward_cuda
    from sinkhorn_b200.distributed import sinkhorn_batch_sharded
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    C, a, b, mask_a, mask_b = _cfg3_inputs()
    B, N, M = C.shape
    la, lb = mask_a.sum(-1), mask_b.sum(-1)  # valid lengths of the whole batch
    i0, i1 = B * rank // world, B * (rank + 1) // world
    C, a, b, mask_a, mask_b = (t[i0:i1].to(dev) for t in (C, a, b, mask_a, mask_b))
    args_ = (C, a, b, 0.1, 1.0, 1.0, mask_a, mask_b, 200, 1e-6)
    if world > 1:
        def solve():
            return sinkhorn_batch_sharded(*args_)
    else:
        def solve():
            return sinkhorn_forward_cuda(*args_)
    solve()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier(device_ids=[local])
    ms, (f, g, n_it, conv) = _events_ms(solve, 5, warm=1)
    if world > 1:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    dense = 8.0 * B * N * M
    lav, lbv = la.to(torch.float64), lb.to(torch.float64)
    valid = 8.0 * float((lav * lbv).sum())
    line = {"workload": "cfg3", "B": B, "N": N, "M": M, "epsilon": 0.1, "tau": 1.0,
            "max_iters": 200, "threshold": 1e-6, "dtype": "f32", "data": "synthetic",
            "n_gpus": world, "scaling": "strong",
            "parallelism": f"batch-sharded x{world}, residual all-reduce (MAX) per check"
                           if world > 1 else "single GPU",
            "sinkhorn_b200": {"ms_per_solve": round(ms, 3), "n_iters": n_it,
                              "converged": bool(conv),
                              "iterations_per_s": round(n_it / ms * 1e3, 1),
                              "dense_gbs": round(dense * n_it / (ms * 1e-3) / 1e9, 1),
                              "valid_gbs": round(valid * n_it / (ms * 1e-3) / 1e9, 1)},
            "bytes_model": "8*B*N*M per iteration (dense) and 8*sum(valid rows*valid cols)"}
    fwd = None if (args.no_reference or world > 1) else \
        _reference_module("sinkhorn.triton.forward")
    if fwd is not None:
        rms, (fr, gr, rn, rc) = _events_ms(lambda: fwd.sinkhorn_forward_triton(*args_), 3, warm=1)
        line["reference_triton"] = {"ms_per_solve": round(rms, 3), "n_iters": rn,
                                    "converged": bool(rc)}
        line["speedup"] = round(rms / ms, 2)
        line["max_abs_df"] = float((f - fr).abs().max())
        line["max_abs_dg"] = float((g - gr).abs().max())
    if world > 1:
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_cfg4(args):
    """Differentiable forward + backward: B=16, N=M=2048, x, y ~ N(0, I_16),
    C = sqdist / mean(C) with requires_grad, uniform marginals, eps=1.0,
    loss = sum(P * C) with P = exp((f + g - C)/eps), backprop to dC; for
    grad_iters 10 (truncated) and 0 (full recompute)."""
    import torch
    from sinkhorn_b200.autograd import sinkhorn_differentiable
    dev = torch.device("cuda", 0)
    gen = torch.Generator().manual_seed(0)
    B, N, M, D = 16, 2048, 2048, 16
    x = torch.randn(B, N, D, generator=gen)
    y = torch.randn(B, M, D, generator=gen)
    C0 = torch.cdist(x, y).pow(2)
    C0 = (C0 / C0.mean()).to(dev)
    eps = 1.0
    ref = None if args.no_reference else _reference_module("sinkhorn.autograd")

    def step(fn, gi, **kw):
        C = C0.clone().requires_grad_(True)
        f, g = fn(C, epsilon=eps, grad_iters=gi, **kw)
        P = torch.exp((f[:, :, None] + g[:, None, :] - C) / eps)
        (P * C).sum().backward()
        return C.grad

    from sinkhorn_b200.autograd import sinkhorn_backward_cuda
    from sinkhorn_b200.cuda.forward import sinkhorn_forward_cuda
    from sinkhorn_b200.cuda.solver import ex2_rate
    peak, _ = hbm_peak()
    ex2_per_s = ex2_rate(dev)
    fs, gs, _, _ = sinkhorn_forward_cuda(C0, None, None, eps, None, None, None, None, 100, 1e-6)
    Pl = torch.exp((fs[:, :, None] + gs[:, None, :] - C0) / eps)
    grad_f = (Pl * C0).sum(2) / eps
    grad_g = (Pl * C0).sum(1) / eps
    del Pl
    bnm = float(B * N * M)
    for gi in (10, 0):
        ms, dC = _events_ms(lambda: step(sinkhorn_differentiable, gi), 3, warm=1)
        # the backward alone (sk_backward: recompute, reverse band passes, dC)
        bms, out = _events_ms(lambda: sinkhorn_backward_cuda(
            C0, None, None, eps, None, None, None, None, 100, 1e-6, gi, fs, gs, grad_f, grad_g),
            3, warm=1)
        K = int(out[3])
        # per unrolled iteration one read of C for the recompute (the
        # single-read step) and one for the reverse step (k_bwd_rows), each
        # with 2 B*N*M exponentials; then one read of C, one write of dC and
        # 2K exponentials per element for dC. The algorithm's two-pass form
        # (2 recompute sweeps + 2 reverse passes per iteration) moves
        # (16 K + 8) B N M bytes: reported beside it.
        bwd_bytes = (8.0 * K + 8.0) * bnm
        two_pass_bytes = (16.0 * K + 8.0) * bnm
        bwd_exps = 6.0 * K * bnm
        floor_ms = max(bwd_bytes / (peak * 1e9), bwd_exps / ex2_per_s) * 1e3
        line = {"workload": "cfg4", "B": B, "N": N, "M": M, "epsilon": eps, "grad_iters": gi,
                "dtype": "f32", "data": "synthetic",
                "timed": "forward (max_iters 100, threshold 1e-6) + loss + backward to dC",
                "sinkhorn_b200": {"ms_per_step": round(ms, 2)},
                "backward": {"ms": round(bms, 3), "K": K,
                             "roofline": {"bound": "hbm" if bwd_bytes / (peak * 1e9) >=
                                          bwd_exps / ex2_per_s else "ex2",
                                          "bytes_model": "(8 K + 8) B N M: per unrolled "
                                                         "iteration one read of C for the "
                                                         "recompute and one for the reverse "
                                                         "step, then read C + write dC",
                                          "exp_model": "6 K B N M",
                                          "floor_ms": round(floor_ms, 3),
                                          "achieved_GBps": round(bwd_bytes / (bms / 1e3) / 1e9,
                                                                 1),
                                          "peak_GBps": peak, "ex2_per_s": round(ex2_per_s, -6),
                                          "frac": round(floor_ms / bms, 4),
                                          "two_pass_equiv_GBps": round(
                                              two_pass_bytes / (bms / 1e3) / 1e9, 1)}}}
        if ref is not None:
            rms, dCr = _events_ms(lambda: step(ref.sinkhorn_differentiable, gi), 2, warm=1)
            line["reference"] = {"ms_per_step": round(rms, 2),
                                 "path": "reference sinkhorn_differentiable (Triton forward, "
                                         "PyTorch autograd backward)"}
            line["speedup"] = round(rms / ms, 2)
            line["dC_max_rel_err"] = float((dC - dCr).abs().max() / dCr.abs().max())
        print(json.dumps(line), flush=True)
        torch.cuda.empty_cache()


def run_implicit(args):
    """Implicit-differentiation adjoint (implicit_gradient): B=16, N=M=2048
    (the differentiable workload's shape) and B=1, N=M=16384, C = sqdist /
    mean, potentials from a converged forward solve (eps=1.0, balanced, and
    tau=1 unbalanced), upstream grads ~ N(0,1), cg_max_iters=50 with
    cg_tol=0 so every call runs all 50 CG iterations. A CG iteration is one
    band pass over C (4*B*N*M bytes) plus the CG vector update; the call adds
    the row/column-sum pass and the dC pass (read C, write dC)."""
    import torch
    from sinkhorn_b200 import implicit_diff as I
    from sinkhorn_b200.cuda.forward import sinkhorn_forward_cuda
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    ref = None if args.no_reference else _reference_module("sinkhorn.pytorch.implicit_diff")
    peak, kind = hbm_peak()
    cg_iters = 50
    for B, n, tau in ((16, 2048, None), (16, 2048, 1.0), (1, 16384, None)):
        gen = torch.Generator().manual_seed(0)
        x = torch.randn(B, n, 16, generator=gen)
        y = torch.randn(B, n, 16, generator=gen)
        C = torch.cdist(x, y).pow(2)
        C = (C / C.mean()).to(dev)
        del x, y
        eps = 1.0
        f, g, _, _ = sinkhorn_forward_cuda(C, None, None, eps, tau, tau, None, None, 200, 1e-6)
        gf = torch.randn(B, n, generator=gen).to(dev)
        gg = torch.randn(B, n, generator=gen).to(dev)

        def call():
            return I.implicit_gradient(C, f, g, gf, gg, eps, tau, tau, None, None, cg_iters, 0.0)

        def call_short():
            return I.implicit_gradient(C, f, g, gf, gg, eps, tau, tau, None, None, 0, 0.0)

        ms, out = _events_ms(call, 3, warm=1)
        ms0, _ = _events_ms(call_short, 3, warm=1)
        it_ms = (ms - ms0) / cg_iters
        it_bytes = 4.0 * B * n * n
        line = {"workload": "implicit", "B": B, "N": n, "M": n, "epsilon": eps, "tau": tau,
                "cg_max_iters": cg_iters, "cg_tol": 0.0, "dtype": "f32", "data": "synthetic",
                "sinkhorn_b200": {
                    "ms_per_call": round(ms, 3), "ms_fixed (sums + dC passes)": round(ms0, 3),
                    "ms_per_cg_iteration": round(it_ms, 4),
                    "cg_iteration_gbs": round(it_bytes / (it_ms * 1e-3) / 1e9, 1),
                    "cg_iteration_hbm_frac": round(it_bytes / (it_ms * 1e-3) / 1e9 / peak, 3),
                    "peak_gbs": peak, "peak_source": kind},
                "bytes_model": "4*B*N*M per CG iteration (C read once; P never stored)"}
        if ref is not None and B * n * n * 4 <= (1 << 31):
            def ref_call():
                return ref.implicit_gradient(C, f, g, gf, gg, eps, tau, tau, None, None,
                                             cg_iters, 0.0)
            rms, rout = _events_ms(ref_call, 2, warm=1)
            line["reference_pytorch"] = {"ms_per_call": round(rms, 3),
                                         "path": "reference implicit_gradient on the GPU "
                                                 "(dense P, torch.bmm matvecs)"}
            line["speedup"] = round(rms / ms, 2)
            errs = {}
            for k, a_, b_ in zip(("dC", "da", "db"), out, rout):
                fin = torch.isfinite(b_) & torch.isfinite(a_)
                errs[k] = float((a_[fin] - b_[fin]).abs().max() / b_[fin].abs().max()) \
                    if bool(fin.any()) else None
            line["max_rel_dev_vs_reference"] = errs
        print(json.dumps(line), flush=True)
        del C, out
        torch.cuda.empty_cache()


def run_f1(args):
    """The plan-side entry points on C resident in HBM, B=16 N=M=2048 and
    B=1 N=M=16384 (C = squared distances over max, f, g from 50 iterations at
    eps=0.05): transport_plan (1 read of C + 1 write of P), cost (1 read),
    marginal error (1 read), the P-free JVP (1 read). Each against the
    reference's own implementation on the same GPU where baseline/_ref holds
    it (SinkhornOutput.transport_plan / .cost, compute_marginal_error;
    jvp_triton needs the plan materialised first, so its time includes it)."""
    import torch
    from sinkhorn_b200.cuda.forward import sinkhorn_forward_cuda
    from sinkhorn_b200.cuda.plan import cost, jvp_cuda_free, marginal_error, transport_plan
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    peak, kind = hbm_peak()
    ref_out = None if args.no_reference else _reference_module("sinkhorn.sinkhorn")
    ref_bal = None if args.no_reference else _reference_module("sinkhorn.pytorch.balanced")
    ref_jvp = None if args.no_reference else _reference_module("sinkhorn.triton.jvp_kernel")
    for B, n in ((16, 2048), (1, 16384)):
        gen = torch.Generator(device=dev).manual_seed(0)
        x = torch.rand(B, n, 3, device=dev, generator=gen)
        y = torch.rand(B, n, 3, device=dev, generator=gen)
        C = torch.cdist(x, y).pow(2)
        C = C / C.amax()
        del x, y
        eps = 0.05
        f, g, _, _ = sinkhorn_forward_cuda(C, None, None, eps, None, None, None, None, 50, 0.0)
        a = torch.full((B, n), 1.0 / n, device=dev)
        v = torch.randn(B, n, device=dev, generator=gen)
        c_bytes = 4.0 * B * n * n
        ops = {
            "transport_plan": (lambda: transport_plan(C, f, g, eps), 2 * c_bytes),
            "cost": (lambda: cost(C, f, g, eps), c_bytes),
            "marginal_error": (lambda: marginal_error(C, f, g, a, a, eps), c_bytes),
            "jvp_pfree": (lambda: jvp_cuda_free(v, v, C, f, g, eps, 0.0, 0.0), c_bytes),
        }
        line = {"workload": "f1", "B": B, "N": n, "M": n, "dtype": "f32", "data": "synthetic",
                "peak_gbs": peak, "peak_source": kind, "sinkhorn_b200": {}}
        for name, (fn, nbytes) in ops.items():
            ms, _ = _events_ms(fn, 5, warm=2)
            line["sinkhorn_b200"][name] = {"ms": round(ms, 4),
                                           "gbs": round(nbytes / (ms * 1e-3) / 1e9, 1),
                                           "hbm_frac": round(nbytes / (ms * 1e-3) / 1e9 / peak, 3)}
        ref = {}
        if ref_out is not None and B * n * n * 4 <= (1 << 31):
            out = ref_out.SinkhornOutput(f=f, g=g, n_iters=50, converged=False)
            ms, _ = _events_ms(lambda: out.transport_plan(C, eps), 3, warm=1)
            ref["transport_plan"] = round(ms, 4)
            ms, _ = _events_ms(lambda: out.cost(C, eps), 3, warm=1)
            ref["cost"] = round(ms, 4)
        if ref_bal is not None and B * n * n * 4 <= (1 << 31):
            ms, _ = _events_ms(lambda: ref_bal.compute_marginal_error(C, f, g, a, a, eps), 3,
                               warm=1)
            ref["marginal_error"] = round(ms, 4)
        if ref_jvp is not None and B * n * n * 4 <= (1 << 31):
            def ref_jvp_call():
                P = torch.exp((f[:, :, None] + g[:, None, :] - C) / eps)
                return ref_jvp.jvp_triton(v, v, P, 0.0, 0.0)
            ms, _ = _events_ms(ref_jvp_call, 3, warm=1)
            ref["jvp_with_plan"] = round(ms, 4)
        if ref:
            line["reference_ms"] = ref
            line["speedup"] = {k: round(ref[k] / line["sinkhorn_b200"][k]["ms"], 2)
                               for k in ("transport_plan", "cost", "marginal_error") if k in ref}
            if "jvp_with_plan" in ref:
                line["speedup"]["jvp"] = round(ref["jvp_with_plan"] /
                                               line["sinkhorn_b200"]["jvp_pfree"]["ms"], 2)
        print(json.dumps(line), flush=True)
        del C
        torch.cuda.empty_cache()


ROWSHARD_EPS = 0.01
ROWSHARD_ITERS = 50


def _rowshard_breakdown(engine, merge, group_size, dev, reps=10):
    """Per-iteration device time of one rank's phases of the row-sharded
    iteration: the local partial (single-read step + chunk merge, or the two
    sweeps), the collectives, and the g-update -- CUDA events on the stream
    they run on (mean of `reps` iterations)."""
    import torch
    import torch.distributed as dist
    stream = torch.cuda.current_stream(dev)
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(reps)]
    P = group_size
    parts = gmax = None
    if merge == "peer":
        engine.peer_begin()
    for r in range(reps):
        ev[r][0].record(stream)
        if merge == "peer":
            # the step and the push (stores into every rank's buffer); the
            # finish then waits for the other ranks' flags on the device
            engine.peer_step()
            ev[r][1].record(stream)
            ev[r][2].record(stream)
            engine.peer_finish()
            ev[r][3].record(stream)
            continue
        part = engine.partial()
        ev[r][1].record(stream)
        if merge == "gather":
            if parts is None:
                parts = part.new_empty((P * part.numel(),))
            dist.all_gather_into_tensor(parts, part)
            ev[r][2].record(stream)
            engine.col_finish(parts.view(P, -1))
        else:
            if gmax is None:
                gmax = part.new_empty(part.shape)
            gmax.copy_(part)
            dist.all_reduce(gmax, op=dist.ReduceOp.MAX)
            ssum = engine.rescale(part, gmax)
            dist.all_reduce(ssum, op=dist.ReduceOp.SUM)
            ev[r][2].record(stream)
            engine.col_finish_pairs(gmax, ssum)
        ev[r][3].record(stream)
    torch.cuda.synchronize()
    out = {}
    for name, i, j in (("partial_ms", 0, 1), ("collectives_ms", 1, 2), ("finish_ms", 2, 3),
                       ("iteration_ms", 0, 3)):
        out[name] = round(sum(e[i].elapsed_time(e[j]) for e in ev) / reps, 4)
    out["comm_share"] = round(out["collectives_ms"] / out["iteration_ms"], 4)
    if merge == "peer":
        out["phases"] = ("partial_ms: the step and the push of the rank's vector into every "
                         "rank's buffer; finish_ms: the wait for the ranks' flags and the "
                         "merge; no collective call")
    return out


def _merge_text(merge):
    return {"peer": "the ranks' column LSE vectors stored into every rank's buffer over "
                    "NVLink peer memory each iteration, merged on every rank after a "
                    "device-side flag wait (no collective call)",
            "allreduce": "allreduce merge of the ranks' column LSEs per iteration (NCCL: MAX, "
                         "then SUM)",
            "gather": "all-gather of the ranks' column LSEs per iteration (NCCL)"}[merge]


def _rowshard_launches(merge, iters):
    """Kernels of this library per solve: k_init, then per iteration the step
    and the merge (+ the rescale for the all-reduce merge) and the finish; the
    peer exchange adds one flag reset per solve."""
    if merge == "peer":
        return 2 + 3 * iters
    return 1 + (4 if merge == "allreduce" else 3) * iters


def run_cuda_sharded(args):
    """The default workload on N > 1 GPUs, row-sharded: every rank runs the
    single-read step on its rows and its chunk merge, the ranks merge their
    column LSE vectors (--merge: stores into every rank's buffer over NVLink
    with device-side flags, the default; or NCCL: two all-reduces, MAX then
    SUM, or one all-gather), and every rank applies the g-update.

    --scaling weak (default): the problem grows with the GPUs, one 16384 x
    16384 block of C (1 GiB, the single-GPU workload) per rank: x ~
    U[0,1]^{16384 N x 3} (rank 0's rows are the single-GPU problem's), y ~
    U[0,1]^{16384 x 3} shared, C = sqdist / max over all ranks, a = 1/(16384
    N); value = block-iterations per second over all ranks (one iteration of
    the N-rank problem is N blocks). --scaling strong: the one N=M=16384
    problem split by rows; value = its iterations per second."""
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    from sinkhorn_b200.distributed import CudaRowEngine, sinkhorn_row_sharded

    n, iters = args.n, args.iters
    weak = args.scaling == "weak"
    if weak:
        n_global = n * world
        r0, r1 = n * rank, n * (rank + 1)
        g0 = torch.Generator(device=dev).manual_seed(1234)
        x = torch.rand(n, 3, device=dev, generator=g0)
        y = torch.rand(n, 3, device=dev, generator=g0)
        if rank > 0:
            gr = torch.Generator(device=dev).manual_seed(1234 + 7919 * rank)
            x = torch.rand(n, 3, device=dev, generator=gr)
        C = torch.cdist(x, y).pow_(2).unsqueeze(0).contiguous()
        del x, y
        mx = C.max().reshape(1)
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        C.div_(mx)
    else:
        n_global = n
        r0, r1 = n * rank // world, n * (rank + 1) // world
        C_full = make_cost_gpu(n, seed=1234, device=dev)  # the same problem on every rank
        C = C_full[:, r0:r1].contiguous()
        del C_full
    torch.cuda.synchronize()
    a_rows = torch.full((1, r1 - r0), 1.0 / n_global, device=dev)
    engine = CudaRowEngine(C, a_rows, None, EPS, None, None, None, None, iters, 0.0, 10)

    def solve():
        engine.reset()
        return sinkhorn_row_sharded(C, a_rows, None, EPS, None, None, None, None, iters, 0.0,
                                    10, n_global=n_global, engine=engine, merge=args.merge)

    for _ in range(max(args.warmup, 3)):
        _, _, n_it, _ = solve()
    assert n_it == iters
    uuid = None
    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:  # noqa: BLE001
        uuid = None
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    dist.barrier(device_ids=[local])
    torch.cuda.synchronize()
    with ClockSampler(local, uuid) as clocks:
        e0.record()
        for _ in range(args.steps):
            solve()
        e1.record()
        torch.cuda.synchronize()
    dist.barrier(device_ids=[local])

    def max_over_ranks(x):
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    ms = max_over_ranks(e0.elapsed_time(e1))
    # per-iteration phases (device time, max over ranks)
    engine.reset()
    bd = _rowshard_breakdown(engine, args.merge, world, dev)
    bd = {k: (max_over_ranks(v) if k.endswith("_ms") else v) for k, v in bd.items()}
    bd["comm_share"] = round(bd["collectives_ms"] / bd["iteration_ms"], 4)

    # e2e through the public API with host buffers: every step copies this
    # rank's rows of C from pinned host memory and reads f and g back
    e2e = None
    if not args.no_e2e:
        C_host = C.cpu().pin_memory()
        f_host = torch.empty(1, r1 - r0).pin_memory()
        g_host = torch.empty(1, n).pin_memory()

        def e2e_step():
            C.copy_(C_host, non_blocking=True)
            f, g, _, _ = solve()
            f_host.copy_(f, non_blocking=True)
            g_host.copy_(g, non_blocking=True)

        e2e_step()
        torch.cuda.synchronize()
        k_e2e = max(3, min(args.steps, 10))
        dist.barrier(device_ids=[local])
        torch.cuda.synchronize()
        e0.record()
        for _ in range(k_e2e):
            e2e_step()
        e1.record()
        torch.cuda.synchronize()
        dist.barrier(device_ids=[local])
        ms_e2e = max_over_ranks(e0.elapsed_time(e1))
        e2e = {"value": round((world if weak else 1) * k_e2e * iters / (ms_e2e / 1e3), 2),
               "unit": UNIT,
               "h2d_bytes_per_step": C_host.numel() * 4,
               "d2h_bytes_per_step": (f_host.numel() + g_host.numel()) * 4,
               "ms_per_step": round(ms_e2e / k_e2e, 3),
               "api": "sinkhorn_b200.distributed.sinkhorn_row_sharded (C ABI sk_solver_*)",
               "pipeline": "per rank: its rows of C host-to-device, the solve, f and g back "
                           "(serialised), max over ranks"}
    engine.close()
    dist.destroy_process_group()
    if rank != 0:
        return
    blocks = world if weak else 1  # 16384 x 16384 blocks per iteration of the whole problem
    value = blocks * args.steps * iters / (ms / 1e3)
    peak, _ = hbm_peak()
    read_gbs = args.steps * iters * 4.0 * n_global * n / (ms / 1e3) / 1e9
    print(json.dumps({
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": max(args.warmup, 3),
        "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
        "scaling": args.scaling, "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": dict(workload_config(args, world),
                       **(weak_rowshard_workload(n, world, iters) if weak else {}),
                       parallelism=f"row-sharded x{world}: {(r1 - r0)} rows per rank, "
                                   f"{_merge_text(args.merge)}"),
        "c_sweep_gbs": round(read_gbs, 1),
        "c_sweep_gbs_model": "bytes of C actually read per second, all ranks (one read of C "
                             "per iteration)",
        "hbm_frac_per_gpu": round(read_gbs / world / peak, 4),
        "per_iteration": bd,
        "clocks": clocks.summary(),
        "gpu_launches": args.steps * _rowshard_launches(args.merge, iters),
        "cpu_baseline": None,
        "cpu_baseline_note": "rank 0 at N=1 only (the single-GPU line)",
        "e2e": e2e,
    }))


def run_rowshard(args):
    """One N=M=n problem (default 65536: 16 GiB of C) split by rows over the
    ranks; per iteration each rank runs the single-read step on its rows
    (8-CTA clusters at M = 65536) and the chunk merge, and the ranks merge
    their column LSEs with NCCL (--merge). Strong scaling: value =
    iterations of the whole problem per second."""
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev,
                            **({} if world > 1 else {"init_method": "tcp://127.0.0.1:29519",
                                                      "rank": 0, "world_size": 1}))
    from sinkhorn_b200.distributed import CudaRowEngine, sinkhorn_row_sharded

    n = args.n if args.n != 16384 else 65536
    iters = ROWSHARD_ITERS
    r0, r1 = n * rank // world, n * (rank + 1) // world
    g = torch.Generator(device=dev).manual_seed(99)
    x = torch.rand(n, 8, device=dev, generator=g)
    y = torch.rand(n, 8, device=dev, generator=g)
    C = torch.empty(1, r1 - r0, n, device=dev)
    for s in range(r0, r1, 4096):
        e = min(r1, s + 4096)
        C[0, s - r0:e - r0] = torch.cdist(x[s:e], y).pow_(2)
    mx = C.max().reshape(1)
    dist.all_reduce(mx, op=dist.ReduceOp.MAX)
    C.div_(mx)
    del x, y
    torch.cuda.synchronize()

    a_rows = torch.full((1, r1 - r0), 1.0 / n, device=dev)
    engine = CudaRowEngine(C, a_rows, None, ROWSHARD_EPS, None, None, None, None, iters, 0.0,
                           10)

    def solve():
        engine.reset()
        return sinkhorn_row_sharded(C, a_rows, None, ROWSHARD_EPS, None, None, None, None,
                                    iters, 0.0, 10, n_global=n, engine=engine,
                                    merge=args.merge)

    for _ in range(max(args.warmup, 3)):
        _, _, n_it, _ = solve()
    assert n_it == iters
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    dist.barrier(device_ids=[local])
    torch.cuda.synchronize()
    uuid = None
    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:  # noqa: BLE001
        uuid = None
    with ClockSampler(local, uuid) as clocks:
        e0.record()
        for _ in range(args.steps):
            solve()
        e1.record()
        torch.cuda.synchronize()
    dist.barrier(device_ids=[local])
    t = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    engine.reset()
    bd = _rowshard_breakdown(engine, args.merge, world, dev)
    single_read = engine.single_read
    engine.close()
    dist.destroy_process_group()
    if rank != 0:
        return
    value = args.steps * iters / (ms / 1e3)
    peak, _ = hbm_peak()
    gbs = args.steps * iters * (4.0 if single_read else 8.0) * n * n / (ms / 1e3) / 1e9
    print(json.dumps({
        "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": max(args.warmup, 3),
        "ms_per_step": round(ms / args.steps, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"row-sharded balanced Sinkhorn B=1 N=M={n} fp32 "
                               f"(C {4 * n * n / 2**30:.0f} GiB split by rows), "
                               f"x,y~U[0,1]^8, C/max, eps={ROWSHARD_EPS}, {iters} iterations",
                   "parallelism": f"row-sharded x{world} ({_merge_text(args.merge)})"},
        "c_sweep_gbs": round(gbs, 1), "c_sweep_gbs_per_gpu": round(gbs / world, 1),
        "c_sweep_gbs_model": "bytes of C actually read per second (one read per iteration "
                             "on the single-read step)" if single_read else
                             "bytes of C actually read per second (two sweeps)",
        "hbm_frac_per_gpu": round(gbs / world / peak, 4),
        "per_iteration_rank0": bd,
        "clocks": clocks.summary(),
        "gpu_launches": args.steps * _rowshard_launches(args.merge, iters),
        "cpu_baseline": None, "e2e": None,
        "cpu_baseline_note": "not measured for this leg: C alone is 16 GiB of host memory and "
                             "the reference's CPU path adds a clone of C and log_K (>= 48 GiB); "
                             "the default workload's line carries the CPU baseline",
    }))


def cpu_sample(C_np, budget_s: float) -> dict:
    """The reference's CPU algorithm (oracle/ C restatement, fp32, OpenMP on
    every host core) on a bounded sample: a few full iterations of the same
    problem, scaled to iterations per second."""
    from oracle import oracle as O
    cores = O.ensure_threads(len(os.sched_getaffinity(0)))  # every host core
    t = time.perf_counter()
    O.forward(C_np, epsilon=EPS, max_iters=1, threshold=0.0, precision="f32")
    t1 = time.perf_counter() - t
    r = max(1, min(50, int(budget_s / max(t1, 1e-3))))
    t = time.perf_counter()
    O.forward(C_np, epsilon=EPS, max_iters=r, threshold=0.0, precision="f32")
    dt = time.perf_counter() - t
    n = C_np.shape[1]
    return {"value": round(r / dt, 4), "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"{r} full iterations of the N=M={n} problem (fp32 C restatement of "
                      f"sinkhorn_unbalanced, OpenMP) in {dt:.1f} s"}


def cpu_reference_torch(C_host, iters: int):
    """The reference's own CPU path (sinkhorn.pytorch.unbalanced, installed
    under baseline/_ref) on every host core: a few iterations of the same
    problem, beside the C restatement the reference arm times."""
    if iters <= 0:
        return None
    mod = _reference_module("sinkhorn.pytorch.unbalanced")
    if mod is None:
        return {"unavailable": "reference package not installed under baseline/_ref"}
    import torch
    cores = len(os.sched_getaffinity(0))
    prev = torch.get_num_threads()
    torch.set_num_threads(cores)
    try:
        Cc = C_host if C_host.device.type == "cpu" else C_host.cpu()
        mod.sinkhorn_unbalanced(Cc, None, None, EPS, None, None, None, None, 1, 0.0)
        t = time.perf_counter()
        mod.sinkhorn_unbalanced(Cc, None, None, EPS, None, None, None, None, iters, 0.0)
        dt = time.perf_counter() - t
    finally:
        torch.set_num_threads(prev)
    n = Cc.shape[1]
    return {"value": round(iters / dt, 4), "unit": UNIT, "cores": cores, "kind": "reference",
            "sample": f"{iters} iterations of the N=M={n} problem through the reference's "
                      f"sinkhorn_unbalanced (PyTorch CPU, fp32) in {dt:.1f} s"}


def run_reference(args):
    """Reference arm: the reference's CPU algorithm on the host cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import oracle as O
    cores = O.ensure_threads(len(os.sched_getaffinity(0)))  # every host core
    n, steps, warm = args.n, args.steps, max(args.warmup, 3)
    C_np = make_cost_cpu(n, seed=1234).numpy()
    # calibrate the per-step sample: ~1.5 s of CPU work, at least one iteration
    t = time.perf_counter()
    O.forward(C_np, epsilon=EPS, max_iters=1, threshold=0.0, precision="f32")
    t1 = time.perf_counter() - t
    r = max(1, int(round(1.5 / max(t1, 1e-3))))
    for _ in range(warm - 1):
        O.forward(C_np, epsilon=EPS, max_iters=r, threshold=0.0, precision="f32")
    t = time.perf_counter()
    for _ in range(steps):
        O.forward(C_np, epsilon=EPS, max_iters=r, threshold=0.0, precision="f32")
    dt = time.perf_counter() - t
    value = steps * r / dt
    sample = (f"{r} full iteration(s) per step of the N=M={n} problem (fp32 C restatement "
              "of sinkhorn_unbalanced, OpenMP, all host threads)")
    config = workload_config(args, 1)
    if args.gpus > 1 and args.scaling == "weak":
        # the GPU arm's problem at N GPUs is N blocks of n x n; the host cores
        # iterate every block alike, so its block-iterations per second are
        # those of the one block sampled here
        config = dict(config, **weak_rowshard_workload(n, args.gpus, args.iters),
                      parallelism=f"host cores (the GPU arm row-shards x{args.gpus})")
        sample += f"; value = {n} x {n} block-iterations per second, as the GPU arm's"
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": UNIT,
        "n_gpus": args.gpus, "steps": steps, "warmup": warm,
        "ms_per_step": round(dt / steps * 1e3, 3), "higher_is_better": True,
        "scaling": args.scaling, "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config,
        "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": cores,
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))


def main(argv=None):
    args = parse_args(argv)
    if args.profile > 0:
        run_profile_case(args)
    elif args.workload == "rowshard" and args.impl == "cuda":
        run_rowshard(args)
    elif args.dtype == "bf16" and args.impl == "cuda":
        run_bf16(args)
    elif args.workload == "sweep" and args.impl == "cuda":
        run_sweep(args)
    elif args.workload == "cfg3" and args.impl == "cuda":
        run_cfg3(args)
    elif args.workload == "cfg4" and args.impl == "cuda":
        run_cfg4(args)
    elif args.workload == "mid" and args.impl == "cuda":
        run_mid(args)
    elif args.workload == "implicit" and args.impl == "cuda":
        run_implicit(args)
    elif args.workload == "f1" and args.impl == "cuda":
        run_f1(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_cuda(args)


if __name__ == "__main__":
    main()
