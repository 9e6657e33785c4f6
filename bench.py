#!/usr/bin/env python
"""Benchmark: Sinkhorn iterations per second of SinkSLOT's sparse solve on B200.

Workload (one step = one Sinkhorn iteration = CSR row half-step + CSC column
half-step): N = M = 2^20 points in d = 3, x ~ N(0, I), y ~ N(0, I) + 1.5 drawn
from torch's CPU generator seeded with 1, uniform weights, eps = 0.01,
L = 64 slices (seed 0), alternating variant.  Synthetic data of the headline
configuration; the reference publishes no number for it.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

One process per GPU; for N > 1 launch under torch.distributed.run.  N > 1
solves one problem of N * 2^20 points per cloud whose rows and columns are
partitioned over the ranks (2^20 of each per rank: weak scaling), the potential
slices exchanged by peer stores after every half-step; the value counts
iterations of 2^20-point problems (N per iteration) over the slowest rank's
time.  ``--replicas`` instead runs one independent 2^20 problem per rank.
``--impl reference`` times the reference algorithm's CPU implementation (the
C port in oracle/, all host threads) on the same workload; rank 0 only.
Rank 0 prints one JSON line.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "Sinkhorn iter/s at N=M=2^20,d=3,L=64 fp32; achieved HBM GB/s as % of peak"
UNIT = "iter/s"
WORKLOAD = dict(n=1 << 20, m=1 << 20, d=3, L=64, eps=0.01, n_iters=500, data_seed=1, shift=1.5,
                proj_seed=0, variant="alternating")
WORKLOAD_NAME = ("sinkslot sparse Sinkhorn, N=M=2^20, d=3, L=64, eps=0.01, alternating, "
                 "x~N(0,I), y~N(0,I)+1.5 (seed 1), uniform weights")


def measured_peak_gbs():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def ncu_traffic():
    p = os.path.join(ROOT, "profiles", "half_step_traffic.json")
    try:
        with open(p) as f:
            return json.load(f)
    except Exception:
        return None


def make_inputs(rank: int, w=None):
    """x, y, a, b on the host for workload w: drawn in that order from torch's
    global CPU generator seeded with the workload's seed (+1000 per replica)."""
    w = WORKLOAD if w is None else w
    torch.manual_seed(w["data_seed"] + 1000 * rank)
    gen = w.get("gen", "gauss")
    n, m, d = w["n"], w["m"], w["d"]
    if gen == "gauss":
        x = torch.randn(n, d)
        y = torch.randn(m, d) + w["shift"]
    elif gen == "gmm_unit":
        x = gmm_unit_cloud(n, w["components"], d, w["std"])
        y = gmm_unit_cloud(m, w["components"], d, w["std"])
    elif gen == "gmm_shift":
        means = w["spread"] * torch.randn(w["components"], d)
        x = means[torch.randint(0, w["components"], (n,))] + torch.randn(n, d)
        y = means[torch.randint(0, w["components"], (m,))] + torch.randn(m, d) + w["shift"]
    else:
        raise ValueError(gen)
    if w.get("weights", "uniform") == "dirichlet":
        a = -torch.rand(n).clamp_min(1e-12).log()
        b = -torch.rand(m).clamp_min(1e-12).log()
        a, b = a / a.sum(), b / b.sum()
    else:
        a = torch.full((n,), 1.0 / n)
        b = torch.full((m,), 1.0 / m)
    return x, y, a, b


def gmm_unit_cloud(n: int, k: int, d: int, std: float) -> torch.Tensor:
    """n points of a k-component Gaussian mixture in [0, 1]^d: means uniform in
    the cube, isotropic std, clipped to the cube (a colour cloud's shape)."""
    means = torch.rand(k, d)
    comp = torch.randint(0, k, (n,))
    return (means[comp] + std * torch.randn(n, d)).clamp_(0.0, 1.0)


# The other workloads of the benchmark suite (one JSON line each, --config):
#   cfg3  colour-transfer shape: N = 2^21 source, M = 2^20 target RGB-like clouds,
#         16-component mixtures in [0,1]^3 (std 0.05, clipped), Dirichlet(1)
#         weights, eps = 0.005, L = 128, symmetric (alpha 0.5), marginal stop at
#         1e-6 checked every 5 iterations; then the plan and the barycentric map
#   cfg4  gradient flow: N = M = 2^18, d = 2, y ~ N(0, I) + 3 (seed 2), 200 outer
#         steps x -= 0.1 * slot_grad(x, y, eps=0.01, L=100, seed=0, n_iters=200),
#         the support rebuilt every step
#   cfg5  scale-out: N = M = 2^24, d = 3, a 4-component Gaussian mixture (means
#         2 * N(0, I), unit components; seed 3) against the same mixture shifted
#         by 1.5; eps = 0.01, L = 64, 300 alternating iterations; under
#         torch.distributed.run the fixed problem is partitioned over the ranks
#         (strong scaling)
CONFIGS = {
    "cfg1": dict(n=10000, m=10000, d=2, L=64, eps=0.05, n_iters=200, data_seed=0, shift=0.0,
                 proj_seed=0, variant="alternating"),
    "cfg2": WORKLOAD,
    "cfg3": dict(n=1 << 21, m=1 << 20, d=3, L=128, eps=0.005, n_iters=20000, data_seed=4,
                 gen="gmm_unit", components=16, std=0.05, weights="dirichlet", proj_seed=0,
                 variant="symmetric", alpha=0.5, stop_mode="marginal", stop_tol=1e-6,
                 stop_check_every=5),
    "cfg4": dict(n=1 << 18, m=1 << 18, d=2, L=100, eps=0.01, n_iters=200, data_seed=2,
                 shift=3.0, proj_seed=0, outer_steps=200, lr=0.1, variant="alternating"),
    "cfg5": dict(n=1 << 24, m=1 << 24, d=3, L=64, eps=0.01, n_iters=300, data_seed=3,
                 gen="gmm_shift", components=4, spread=2.0, shift=1.5, proj_seed=0,
                 variant="alternating"),
}
CONFIG_NAMES = {
    "cfg1": "sinkslot CPU-runnable configuration, N=M=10^4, d=2, x,y~N(0,I) (seed 0), uniform "
            "weights, eps=0.05, L=64, 200 alternating iterations; SamplesLoss cost, potentials, "
            "slot_grad",
    "cfg3": "sinkslot colour-transfer shape, N=2^21 x M=2^20, d=3, 16-component mixtures in "
            "[0,1]^3, Dirichlet weights, L=128, eps=0.005, symmetric, marginal stop 1e-6/5 "
            "(seed 4); then plan + barycentric map",
    "cfg4": "sinkslot gradient flow, N=M=2^18, d=2, y~N(0,I)+3 (seed 2), x -= 0.1*slot_grad("
            "eps=0.01, L=100, 200 iterations), support rebuilt every step",
    "cfg5": "sinkslot scale-out, N=M=2^24, d=3, 4-component mixture vs shifted mixture (seed 3), "
            "L=64, eps=0.01, 300 alternating iterations",
}


# --------------------------------------------------------------------------
# clocks sampled during the timed region
# --------------------------------------------------------------------------
_REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
            0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
            0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
            0x100: "display_clock_setting"}


class ClockSampler:
    def __init__(self, device_index: int):
        self.proc = None
        self.lines = []
        try:
            uuid = "GPU-" + str(torch.cuda.get_device_properties(device_index).uuid)
        except Exception:
            uuid = str(device_index)
        self.cmd = ["nvidia-smi", f"--id={uuid}",
                    "--query-gpu=clocks.sm,clocks.max.sm,clocks_event_reasons.active",
                    "--format=csv,noheader,nounits", "-lms", "50"]

    def start(self):
        try:
            self.proc = subprocess.Popen(self.cmd, stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        time.sleep(0.15)

    def stop(self):
        if self.proc is None:
            return self._summary([])
        time.sleep(0.06)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out, _ = self.proc.communicate()
        return self._summary(out.strip().splitlines())

    @staticmethod
    def _summary(lines):
        sm, mx, reasons = [], [], set()
        for ln in lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 3:
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
                bits = int(parts[2], 16)
            except ValueError:
                continue
            for bit, name in _REASONS.items():
                if bits & bit:
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# --------------------------------------------------------------------------
# distributed plumbing
# --------------------------------------------------------------------------
def dist_setup(gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    elif gpus > 1:
        raise SystemExit("--gpus > 1 needs torch.distributed.run (one process per GPU)")
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(v: float, world: int, dev) -> float:
    if world == 1:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# launches per half-step of each side kind: the exact kernel; the staged tiled
# pass + the exact pass over handed-back rows; the two-pass kind's exponent
# pass, sum pass and handed-back pass
SIDE_LAUNCHES = {"exact": 1, "staged": 2, "two_pass": 3}


def side_kind(layout, nseg: int, m_other: int, nnz: int) -> str:
    """How a side runs: "exact" (no tiled layout), "staged" or "two_pass"."""
    if layout is None:
        return "exact"
    from sinkslot_b200.sinkhorn_solvers import tiles_kind_of
    return tiles_kind_of(nseg, m_other, nnz)


# --------------------------------------------------------------------------
# the B200 arm
# --------------------------------------------------------------------------
def run_b200(args):
    import sinkslot_b200
    from sinkslot_b200 import sinkslot_solve
    from sinkslot_b200.sinkhorn_solvers import (build_tiles, seg_lse_online,
                                                sinkslot_alternating_b200, tiles_pay_off)
    from sinkslot_b200.solver import _to_csr, cost_and_lam, sot_plan_coo

    world, rank, local = dist_setup(args.gpus)
    if world > 1 and not args.replicas:
        return run_b200_sharded(args, world, rank, local)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    torch.backends.cuda.matmul.allow_tf32 = False
    sinkslot_b200.load_library()
    w = WORKLOAD
    x, y, a, b = make_inputs(rank)
    X, Y, A, B = (t.to(dev) for t in (x, y, a, b))

    # setup (untimed for the iteration metric; reported cold -- the first call,
    # with library and allocator start-up -- and warm, as each e2e step runs it)
    def setup():
        rows, cols, S = sot_plan_coo(X, Y, A, B, L=w["L"], seed=w["proj_seed"])
        lam, _ = cost_and_lam(X, Y, rows, cols, S, w["eps"])
        r_ptr, r_idx, r_lam, _ = _to_csr(rows, cols, lam, w["n"], want_perm=False)
        c_ptr, c_idx, c_lam, _ = _to_csr(cols, rows, lam, w["m"], want_perm=False)
        nnz0 = int(rows.numel())
        tiles = None if args.plain else (
            build_tiles(r_ptr, r_idx, r_lam, w["n"], w["m"])
            if tiles_pay_off(w["n"], w["m"], nnz0) else None,
            build_tiles(c_ptr, c_idx, c_lam, w["m"], w["n"])
            if tiles_pay_off(w["m"], w["n"], nnz0) else None)
        return rows, cols, lam, r_ptr, r_idx, r_lam, c_ptr, c_idx, c_lam, tiles

    setup_times = []
    for _ in range(2):
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        rows, cols, lam, r_ptr, r_idx, r_lam, c_ptr, c_idx, c_lam, tiles = setup()
        log_a, log_b = A.log(), B.log()
        torch.cuda.synchronize(dev)
        setup_times.append((time.perf_counter() - t0) * 1e3)
    setup_cold_ms, setup_ms = setup_times
    nnz = int(rows.numel())
    csr = (r_ptr, r_idx, r_lam, c_ptr, c_idx, c_lam, log_a, log_b, w["n"], w["m"])
    sides = {"row": side_kind(tiles[0] if tiles else None, w["n"], w["m"], nnz),
             "col": side_kind(tiles[1] if tiles else None, w["m"], w["n"], nnz)}

    # warm-up, then exactly K timed iterations in one fused-loop call
    sinkslot_alternating_b200(*csr, max(args.warmup, 0), tiles=tiles)
    torch.cuda.synchronize(dev)
    stream = torch.cuda.current_stream(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
    barrier(world)
    torch.cuda.synchronize(dev)
    ev0.record(stream)
    phi, psi, *_ = sinkslot_alternating_b200(*csr, args.steps, tiles=tiles)
    ev1.record(stream)
    torch.cuda.synchronize(dev)
    barrier(world)
    clocks = sampler.stop() if sampler else None
    ms = max_over_ranks(ev0.elapsed_time(ev1), world, dev)
    value = world * args.steps / (ms / 1e3) if ms > 0 else 0.0
    # the half-step as the loop runs it (tiled pass + exact pass over handed-back
    # rows, or the exact kernel alone with --plain), averaged over the timed region
    t_half = ms / 1e3 / (2 * args.steps)

    # the exact kernel alone, each launch timed with events on its stream
    reps = 20
    dur = {"row": [], "col": []}
    out_phi = torch.empty_like(log_a)
    out_psi = torch.empty_like(log_b)
    z_n, z_m = torch.zeros_like(log_a), torch.zeros_like(log_b)
    for _ in range(reps):
        for side in ("row", "col"):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            if side == "row":
                seg_lse_online(r_ptr, r_idx, r_lam, z_n, psi, w["n"], base=log_a, out=out_phi)
            else:
                seg_lse_online(c_ptr, c_idx, c_lam, z_m, phi, w["m"], base=log_b, out=out_psi)
            e1.record(stream)
            torch.cuda.synchronize(dev)
            dur[side].append(e0.elapsed_time(e1))
    s_idx = r_idx.element_size()
    bytes_row = nnz * (s_idx + 4) + 16 * w["n"]
    bytes_col = nnz * (c_idx.element_size() + 4) + 16 * w["m"]
    t_row = statistics.median(dur["row"]) / 1e3
    t_col = statistics.median(dur["col"]) / 1e3
    achieved = (bytes_row + bytes_col) / (2 * t_half) / 1e9
    peak, peak_kind = measured_peak_gbs()
    b_iter = bytes_row + bytes_col
    traffic = ncu_traffic()

    # end to end through the public API from pinned host buffers
    xh, yh, ah, bh = (t.pin_memory() for t in (x, y, a, b))
    phi_h = torch.empty(w["n"]).pin_memory()
    psi_h = torch.empty(w["m"]).pin_memory()

    def e2e_step():
        Xd = xh.to(dev, non_blocking=True)
        Yd = yh.to(dev, non_blocking=True)
        Ad = ah.to(dev, non_blocking=True)
        Bd = bh.to(dev, non_blocking=True)
        r = sinkslot_solve(Xd, Yd, Ad, Bd, w["eps"], w["L"], w["proj_seed"], w["n_iters"])
        phi_h.copy_(r.phi, non_blocking=True)
        psi_h.copy_(r.psi, non_blocking=True)

    e2e_step()
    torch.cuda.synchronize(dev)
    e2e_steps = 3
    barrier(world)
    torch.cuda.synchronize(dev)
    q0, q1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    q0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    q1.record(stream)
    torch.cuda.synchronize(dev)
    barrier(world)
    e2e_ms = max_over_ranks(q0.elapsed_time(q1), world, dev)
    e2e_value = world * e2e_steps * w["n_iters"] / (e2e_ms / 1e3)
    h2d = sum(t.numel() * t.element_size() for t in (x, y, a, b))
    d2h = (w["n"] + w["m"]) * 4

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline_from_support(rows, cols, lam, log_a, log_b, w)
    triton_ref = None
    if rank == 0 and world == 1 and not args.no_triton:
        del rows, cols, lam, csr, r_ptr, r_idx, r_lam, c_ptr, c_idx, c_lam, tiles
        torch.cuda.empty_cache()
        triton_ref = triton_reference_leg(X, Y, A, B, w, min(args.steps, 1000), value)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD_NAME, "n": w["n"], "m": w["m"], "d": w["d"],
                       "L": w["L"], "eps": w["eps"], "nnz": nnz,
                       "parallelism": f"independent problem per GPU x{world}" if world > 1
                       else "single GPU",
                       "l2": "inputs larger than L2: %.2f GB of CSR+CSC streamed per iteration"
                             % (2 * nnz * (s_idx + 4) / 1e9),
                       "setup_ms": round(setup_ms, 1), "setup_cold_ms": round(setup_cold_ms, 1),
                       "algorithmic_bytes_per_iter": b_iter,
                       "iteration_gbs": round(b_iter * value / world / 1e9, 1)},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "peak_source": peak_kind,
                         "traffic": traffic.get("bytes_per_launch") if traffic else None,
                         "kernel": ("half_step_kernel (exact)" if args.plain else
                                    "tiled half-step (staged: tiled_half_step_kernel; two-pass: "
                                    "block_gather_kernel + panel_sum_kernel) + exact pass over "
                                    "handed-back rows")
                                   + ", per half-step, averaged over the timed region",
                         "sides": sides,
                         "bytes_per_half_step": {"row": bytes_row, "col": bytes_col},
                         "half_step_us": round(t_half * 1e6, 2),
                         "exact_kernel_us": {"row": round(t_row * 1e6, 2),
                                             "col": round(t_col * 1e6, 2),
                                             "timing": "each launch alone, median of %d" % reps}},
            "cpu_baseline": cpu,
            "triton_reference": triton_ref,
            "e2e": {"value": round(e2e_value, 2), "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h,
                    "step": "sinkslot_solve(...) from pinned host x, y, a, b: support build + "
                            "%d iterations + potentials back" % w["n_iters"]},
            # per iteration the launches of each side's kind (the first iteration's
            # row half-step is one exact launch, its column side adds a max pass)
            "gpu_launches": args.steps * (SIDE_LAUNCHES[sides["row"]] +
                                          SIDE_LAUNCHES[sides["col"]]),
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def run_b200_sharded(args, world, rank, local):
    """N > 1: one problem of N * 2^20 points per cloud, rows and columns
    partitioned over the N ranks (2^20 of each per rank: weak scaling), the
    potentials exchanged by peer stores after every half-step."""
    import torch.distributed as dist
    import sinkslot_b200
    from sinkslot_b200.sharded import ShardedSolver, sinkslot_solve_sharded

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    torch.backends.cuda.matmul.allow_tf32 = False
    sinkslot_b200.load_library()
    w = dict(WORKLOAD)
    w["n"] *= world
    w["m"] *= world
    x, y, a, b = make_inputs(0, w)  # identical on every rank
    X, Y, A, B = (t.to(dev) for t in (x, y, a, b))
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    solver = ShardedSolver(X, Y, A, B, w["eps"], L=w["L"], seed=w["proj_seed"])
    torch.cuda.synchronize(dev)
    setup_ms = (time.perf_counter() - t0) * 1e3
    nnz = solver.nnz
    solver.solve(max(args.warmup, 0), copy_out=False)
    torch.cuda.synchronize(dev)
    stream = torch.cuda.current_stream(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
    barrier(world)
    torch.cuda.synchronize(dev)
    ev0.record(stream)
    solver.solve(args.steps, copy_out=False)
    ev1.record(stream)
    torch.cuda.synchronize(dev)
    barrier(world)
    clocks = sampler.stop() if sampler else None
    ms = max_over_ranks(ev0.elapsed_time(ev1), world, dev)
    # units: iterations of a 2^20-point problem (each iteration here is `world` of them)
    value = world * args.steps / (ms / 1e3) if ms > 0 else 0.0
    t_half = ms / 1e3 / (2 * args.steps)
    # this rank's bytes per half-step: its slice's entries and segments
    r_nnz, c_nnz = solver.row[3], solver.col[3]
    sides = {"row": side_kind(solver.r_tiles, solver.nr, w["m"], r_nnz),
             "col": side_kind(solver.c_tiles, solver.nc, w["n"], c_nnz)}
    bytes_row = r_nnz * (solver.row[1].element_size() + 4) + 16 * solver.nr
    bytes_col = c_nnz * (solver.col[1].element_size() + 4) + 16 * solver.nc
    achieved = max_over_ranks(-((bytes_row + bytes_col) / (2 * t_half) / 1e9), world, dev)
    achieved = -achieved  # the slowest rank's rate
    solver.close()
    del solver
    peak, peak_kind = measured_peak_gbs()

    # end to end through the public API from pinned host buffers (support build,
    # the partitioned solve, potentials back)
    xh, yh, ah, bh = (t.pin_memory() for t in (x, y, a, b))
    phi_h = torch.empty(w["n"]).pin_memory()
    psi_h = torch.empty(w["m"]).pin_memory()

    def e2e_step():
        r = sinkslot_solve_sharded(xh.to(dev, non_blocking=True), yh.to(dev, non_blocking=True),
                                   ah.to(dev, non_blocking=True), bh.to(dev, non_blocking=True),
                                   w["eps"], w["L"], w["proj_seed"], w["n_iters"])
        phi_h.copy_(r.phi, non_blocking=True)
        psi_h.copy_(r.psi, non_blocking=True)

    e2e_step()  # untimed: first-call set-up (IPC mappings, library state)
    torch.cuda.synchronize(dev)
    barrier(world)
    torch.cuda.synchronize(dev)
    q0, q1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    q0.record(stream)
    e2e_step()
    q1.record(stream)
    torch.cuda.synchronize(dev)
    barrier(world)
    e2e_ms = max_over_ranks(q0.elapsed_time(q1), world, dev)
    e2e_value = world * w["n_iters"] / (e2e_ms / 1e3)
    h2d = sum(t.numel() * t.element_size() for t in (x, y, a, b))
    d2h = (w["n"] + w["m"]) * 4
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD_NAME.replace(
                           "N=M=2^20", f"N=M={world}x2^20 partitioned over {world} GPUs"),
                       "n": w["n"], "m": w["m"], "d": w["d"], "L": w["L"], "eps": w["eps"],
                       "nnz": nnz,
                       "parallelism": f"rows and columns partitioned over {world} GPUs; "
                                      f"potential slices exchanged by peer stores after every "
                                      f"half-step",
                       "unit_note": f"one step = one iteration of the {world}x2^20 problem = "
                                    f"{world} iterations of the 2^20 problem",
                       "l2": "inputs larger than L2: %.2f GB of CSR+CSC streamed per rank "
                             "per iteration" % ((bytes_row + bytes_col) / 1e9),
                       "setup_ms": round(setup_ms, 1)},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "peak_source": peak_kind, "traffic": None,
                         "kernel": "per rank: the half-step kernel of each side (tiled "
                                   "half-step + exact pass over handed-back rows, or the "
                                   "exact kernel) + peer push + epoch wait, per half-step, "
                                   "averaged over the timed region",
                         "sides": sides,
                         "bytes_per_half_step_rank0": {"row": bytes_row, "col": bytes_col},
                         "half_step_us": round(t_half * 1e6, 2)},
            "cpu_baseline": None,
            "e2e": {"value": round(e2e_value, 2), "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h,
                    "step": "sinkslot_solve_sharded(...) from pinned host x, y, a, b: support "
                            "build + %d iterations + potentials back" % w["n_iters"]},
            # per half-step: the side's kernels + peer publish + epoch wait
            "gpu_launches": args.steps * (SIDE_LAUNCHES[sides["row"]] +
                                          SIDE_LAUNCHES[sides["col"]] + 4),
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    dist.destroy_process_group()


# --------------------------------------------------------------------------
# the other workloads (--config cfg3 | cfg4 | cfg5), one GPU unless noted
# --------------------------------------------------------------------------
def _timed(stream, fn):
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(stream)
    out = fn()
    e1.record(stream)
    torch.cuda.synchronize()
    return out, e0.elapsed_time(e1)


def _side_bytes(idx, nnz, nseg):
    return nnz * (idx.element_size() + 4) + 16 * nseg


def _base_line(cfg, w, value, unit, world, steps, warmup, ms_per_step, clocks, extra_config):
    config = {"workload": CONFIG_NAMES[cfg], "n": w["n"], "m": w["m"], "d": w["d"], "L": w["L"],
              "eps": w["eps"]}
    config.update(extra_config)
    return {"metric": METRICS[cfg], "value": round(value, 3), "unit": unit, "n_gpus": world,
            "steps": steps, "warmup": warmup, "ms_per_step": round(ms_per_step, 4),
            "higher_is_better": True, "scaling": "strong" if cfg == "cfg5" else "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": config,
            "clocks": clocks}


METRICS = {
    "cfg1": "Sinkhorn iter/s at N=M=10^4,d=2,L=64 fp32 (launch-bound small problem)",
    "cfg3": "colour-transfer-shaped solve: symmetric Sinkhorn iter/s at N=2^21,M=2^20,d=3,L=128 "
            "fp32 (marginal stop)",
    "cfg4": "gradient-flow outer steps/s at N=M=2^18,d=2,L=100 fp32 (support rebuilt per step)",
    "cfg5": "Sinkhorn iter/s at N=M=2^24,d=3,L=64 fp32, rows/cols partitioned over the GPUs",
}


def run_cfg1(args):
    """The small configuration the reference runs on CPU: a step is one
    iteration of the 200-iteration solve loop (launch-bound: ~8 MB of CSR/CSC,
    L2-resident); e2e is SamplesLoss (cost, backward) + the potentials from host
    tensors, per solve of 200 iterations."""
    import sinkslot_b200
    from sinkslot_b200 import SamplesLoss
    from sinkslot_b200.sinkhorn_solvers import sinkslot_alternating_b200
    from sinkslot_b200.solver import _to_csr, cost_and_lam, sot_plan_coo

    world, rank, local = dist_setup(1)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    torch.backends.cuda.matmul.allow_tf32 = False
    sinkslot_b200.load_library()
    w = CONFIGS["cfg1"]
    n, m = w["n"], w["m"]
    x, y, a, b = make_inputs(0, w)
    X, Y, A, B = (t.to(dev) for t in (x, y, a, b))
    stream = torch.cuda.current_stream(dev)

    def setup():
        rows, cols, S = sot_plan_coo(X, Y, A, B, L=w["L"], seed=w["proj_seed"])
        lam, _ = cost_and_lam(X, Y, rows, cols, S, w["eps"])
        r = _to_csr(rows, cols, lam, n, want_perm=False)
        c = _to_csr(cols, rows, lam, m, want_perm=False)
        return int(rows.numel()), (r[0], r[1], r[2], c[0], c[1], c[2], A.log(), B.log(), n, m)

    setup()
    (nnz, csr), setup_ms = _timed(stream, setup)
    sinkslot_alternating_b200(*csr, max(args.warmup, 3))
    K = max(1, min(args.steps, 2000))
    sampler = ClockSampler(local)
    sampler.start()
    _, ms = _timed(stream, lambda: sinkslot_alternating_b200(*csr, K))
    clocks = sampler.stop()
    value = K / (ms / 1e3)
    b_iter = _side_bytes(csr[1], nnz, n) + _side_bytes(csr[4], nnz, m)
    peak, peak_kind = measured_peak_gbs()
    loss_fn = SamplesLoss(eps=w["eps"], L=w["L"], seed=w["proj_seed"], n_iters=w["n_iters"])
    xh, yh = x.pin_memory(), y.pin_memory()
    gh = torch.empty_like(x).pin_memory()

    def e2e():
        Xd = xh.to(dev, non_blocking=True).requires_grad_(True)
        Yd = yh.to(dev, non_blocking=True)
        loss = loss_fn(Xd, Yd)
        (g,) = torch.autograd.grad(loss, [Xd])
        gh.copy_(g, non_blocking=True)

    e2e()
    reps = 20
    _, e2e_ms = _timed(stream, lambda: [e2e() for _ in range(reps)])
    tri = None if args.no_triton else triton_reference_leg(X, Y, A, B, w, K, value)
    line = _base_line("cfg1", w, value, UNIT, 1, K, max(args.warmup, 3), ms / K, clocks, {
        "nnz": nnz, "setup_ms": round(setup_ms, 2), "idx_bytes": csr[1].element_size(),
        "l2": "L2-resident: %.1f MB of CSR+CSC per iteration" % (b_iter / 1e6),
        "solve_us_per_iteration": round(ms / K * 1e3, 2)})
    line["roofline"] = {"bound": "hbm", "achieved": round(b_iter * value / 1e9, 1), "peak": peak,
                        "unit": "GB/s", "frac": round(b_iter * value / 1e9 / peak, 4),
                        "peak_source": peak_kind, "traffic": None,
                        "kernel": "exact half-step kernel (below the tiled pass's threshold); "
                                  "launch-bound, data L2-resident"}
    line["cpu_baseline"] = None
    line["triton_reference"] = tri
    line["e2e"] = {"value": round(reps * w["n_iters"] / (e2e_ms / 1e3), 2), "unit": UNIT,
                   "h2d_bytes_per_step": (x.numel() + y.numel()) * 4,
                   "d2h_bytes_per_step": x.numel() * 4,
                   "step": "SamplesLoss forward (support build + 200 iterations + cost) and "
                           "backward from pinned host x, y; the gradient back",
                   "ms_per_solve": round(e2e_ms / reps, 3)}
    line["gpu_launches"] = 2 * K
    print(json.dumps(line), flush=True)


def run_cfg3(args):
    """The colour-transfer shape: build, symmetric solve to the marginal stop,
    plan export and barycentric map.  A step is one whole solve from zero
    potentials; the value counts Sinkhorn iterations per second over the
    timed solves (each check adds the reference's two check half-steps)."""
    from types import SimpleNamespace
    import sinkslot_b200
    from sinkslot_b200 import sparse_barycentric_map, sparse_transport_plan
    from sinkslot_b200.sinkhorn_solvers import build_tiles, sinkslot_symmetric_b200, tiles_pay_off
    from sinkslot_b200.solver import _to_csr, cost_and_lam, sot_plan_coo

    world, rank, local = dist_setup(1)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    torch.backends.cuda.matmul.allow_tf32 = False
    sinkslot_b200.load_library()
    w = CONFIGS["cfg3"]
    n, m = w["n"], w["m"]
    x, y, a, b = make_inputs(0, w)
    X, Y, A, B = (t.to(dev) for t in (x, y, a, b))
    stream = torch.cuda.current_stream(dev)

    def setup():
        rows, cols, S = sot_plan_coo(X, Y, A, B, L=w["L"], seed=w["proj_seed"])
        lam, _ = cost_and_lam(X, Y, rows, cols, S, w["eps"])
        r = _to_csr(rows, cols, lam, n, want_perm=False)
        c = _to_csr(cols, rows, lam, m, want_perm=False)
        nnz = int(rows.numel())
        tiles = (build_tiles(r[0], r[1], r[2], n, m) if tiles_pay_off(n, m, nnz) else None,
                 build_tiles(c[0], c[1], c[2], m, n) if tiles_pay_off(m, n, nnz) else None)
        return nnz, (r[0], r[1], r[2], c[0], c[1], c[2], A.log(), B.log(), n, m), tiles

    (nnz, csr, tiles), setup_cold = _timed(stream, setup)
    del nnz, csr, tiles
    (nnz, csr, tiles), setup_ms = _timed(stream, setup)
    stop = SimpleNamespace(mode=w["stop_mode"], max_iter=w["n_iters"], tol=w["stop_tol"],
                           check_every=w["stop_check_every"])

    def solve(st=stop):
        return sinkslot_symmetric_b200(*csr, 0, st, eps=w["eps"], alpha=w["alpha"],
                                       tiles=tiles)

    # warm-up: a short solve (the full one runs to max_iter: tiny Dirichlet
    # weights leave empty rows whose +inf potentials make every marginal check
    # NaN, in the reference as here)
    solve(SimpleNamespace(mode=stop.mode, max_iter=max(args.warmup, 3) * 5, tol=stop.tol,
                          check_every=stop.check_every))
    K = 1
    sampler = ClockSampler(local)
    sampler.start()
    res, ms = _timed(stream, lambda: [solve() for _ in range(K)])
    clocks = sampler.stop()
    iters = sum(r[2] for r in res)
    it, conv, viol = res[-1][2], res[-1][3], res[-1][4]
    value = iters / (ms / 1e3)
    checks = iters // w["stop_check_every"]
    half_steps = 2 * iters + 2 * checks  # each check: both check-only half-steps
    b_row, b_col = _side_bytes(csr[1], nnz, n), _side_bytes(csr[4], nnz, m)
    achieved = (iters + checks) * (b_row + b_col) / (ms / 1e3) / 1e9
    peak, peak_kind = measured_peak_gbs()

    # end to end: sparse_transport_plan + sparse_barycentric_map from pinned host
    # inputs, the barycentric images back to the host
    xh, yh, ah, bh = (t.pin_memory() for t in (x, y, a, b))
    txh = torch.empty(n, 3).pin_memory()

    def e2e():
        Xd, Yd = xh.to(dev, non_blocking=True), yh.to(dev, non_blocking=True)
        Ad, Bd = ah.to(dev, non_blocking=True), bh.to(dev, non_blocking=True)
        P = sparse_transport_plan(Xd, Yd, Ad, Bd, eps=w["eps"], L=w["L"], seed=w["proj_seed"],
                                  stop_mode=w["stop_mode"], stop_max_iter=w["n_iters"],
                                  stop_tol=w["stop_tol"],
                                  stop_check_every=w["stop_check_every"], variant="symmetric",
                                  alpha=w["alpha"])
        Tx, _ = sparse_barycentric_map(P, Xd, Yd)
        txh.copy_(Tx, non_blocking=True)

    _, e2e_ms = _timed(stream, e2e)  # the solve above warmed the kernels and the allocator
    line = _base_line("cfg3", w, value, UNIT, 1, K, 1, ms / K, clocks, {
        "nnz": nnz, "iters_per_solve": it, "converged": bool(conv),
        "final_viol": None if viol != viol else viol,
        "setup_ms": round(setup_ms, 1), "setup_cold_ms": round(setup_cold, 1),
        "step": "one symmetric solve from zero potentials to the marginal stop",
        "sides": {"row": "tiled" if tiles[0] is not None else "exact",
                  "col": "tiled" if tiles[1] is not None else "exact"},
        "l2": "inputs larger than L2: %.2f GB of CSR+CSC streamed per iteration"
              % ((b_row + b_col) / 1e9)})
    line["roofline"] = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                        "unit": "GB/s", "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                        "traffic": None, "half_steps_per_solve": half_steps // K if K else None,
                        "kernel": "all half-steps of the timed solves (tiled + exact passes), "
                                  "algorithmic bytes of each over the solve time"}
    line["cpu_baseline"] = None
    line["e2e"] = {"value": round(it / (e2e_ms / 1e3), 3), "unit": UNIT,
                   "h2d_bytes_per_step": sum(t.numel() * t.element_size() for t in (x, y, a, b)),
                   "d2h_bytes_per_step": n * 3 * 4,
                   "step": "sparse_transport_plan(symmetric, marginal stop) + "
                           "sparse_barycentric_map from pinned host inputs, Tx back",
                   "ms": round(e2e_ms, 1)}
    line["gpu_launches"] = None
    print(json.dumps(line), flush=True)


def run_cfg4(args):
    """Gradient flow: x -= lr * slot_grad(x, y, ...) with the support rebuilt
    every step.  A step is one outer step; K = min(--steps, 200) steps timed."""
    import sinkslot_b200
    from sinkslot_b200 import slot_grad

    world, rank, local = dist_setup(1)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    torch.backends.cuda.matmul.allow_tf32 = False
    sinkslot_b200.load_library()
    w = CONFIGS["cfg4"]
    x, y, a, b = make_inputs(0, w)
    X0, Y, A, B = (t.to(dev) for t in (x, y, a, b))
    stream = torch.cuda.current_stream(dev)

    def step(X):
        g = slot_grad(X, Y, A, B, w["eps"], w["L"], w["proj_seed"], w["n_iters"])
        X.sub_(w["lr"] * g)

    Xw = X0.clone()
    for _ in range(max(args.warmup, 3)):
        step(Xw)
    K = max(1, min(args.steps, w["outer_steps"]))
    X = X0.clone()
    sampler = ClockSampler(local)
    sampler.start()
    _, ms = _timed(stream, lambda: [step(X) for _ in range(K)])
    clocks = sampler.stop()
    value = K / (ms / 1e3)
    # one instrumented step: set-up, solve loop and export separately
    parts = cfg4_breakdown(X0, Y, A, B, w, stream)
    # end to end: every step copies x from pinned host memory and x back
    xh = x.clone().pin_memory()
    Yh, Ah, Bh = (t.pin_memory() for t in (y, a, b))
    Yd, Ad, Bd = Yh.to(dev), Ah.to(dev), Bh.to(dev)

    def e2e():
        for _ in range(K):
            Xd = xh.to(dev, non_blocking=True)
            g = slot_grad(Xd, Yd, Ad, Bd, w["eps"], w["L"], w["proj_seed"], w["n_iters"])
            Xd.sub_(w["lr"] * g)
            xh.copy_(Xd, non_blocking=True)

    _, e2e_ms = _timed(stream, e2e)
    line = _base_line("cfg4", w, value, "steps/s", 1, K, max(args.warmup, 3), ms / K, clocks,
                      {"outer_steps_timed": K, "lr": w["lr"], "n_iters": w["n_iters"],
                       "per_step_ms": parts,
                       "step": "slot_grad (support build + 200 alternating iterations + "
                               "barycentric gradient) and the update x -= 0.1 grad"})
    line["roofline"] = parts.pop("roofline")
    line["cpu_baseline"] = None
    line["e2e"] = {"value": round(K / (e2e_ms / 1e3), 3), "unit": "steps/s",
                   "h2d_bytes_per_step": x.numel() * 4, "d2h_bytes_per_step": x.numel() * 4,
                   "step": "x from pinned host, slot_grad, update, x back"}
    line["gpu_launches"] = None
    print(json.dumps(line), flush=True)


def cfg4_breakdown(X, Y, A, B, w, stream):
    """Milliseconds of one gradient-flow step's parts, and the roofline of its
    solve loop (algorithmic bytes per iteration over the loop's time)."""
    from sinkslot_b200.gradient import grad_from_plan
    from sinkslot_b200.sinkhorn_solvers import (build_tiles, plan_values,
                                                sinkslot_alternating_b200, tiles_pay_off)
    from sinkslot_b200.solver import _to_csr, cost_and_lam, sot_plan_coo
    n, m = w["n"], w["m"]
    (rows, cols, S), t_sup = _timed(stream, lambda: sot_plan_coo(X, Y, A, B, L=w["L"],
                                                                  seed=w["proj_seed"]))

    def prep():
        lam, _ = cost_and_lam(X, Y, rows, cols, S, w["eps"])
        r = _to_csr(rows, cols, lam, n, want_perm=False)
        c = _to_csr(cols, rows, lam, m, want_perm=False)
        nnz = rows.numel()
        tl = (build_tiles(r[0], r[1], r[2], n, m) if tiles_pay_off(n, m, nnz) else None,
              build_tiles(c[0], c[1], c[2], m, n) if tiles_pay_off(m, n, nnz) else None)
        return r, c, tl

    (r, c, tl), t_prep = _timed(stream, prep)
    csr = (r[0], r[1], r[2], c[0], c[1], c[2], A.log(), B.log(), n, m)
    (phi, psi, *_), t_loop = _timed(stream, lambda: sinkslot_alternating_b200(
        *csr, w["n_iters"], tiles=tl))
    _, t_exp = _timed(stream, lambda: grad_from_plan(plan_values(
        phi, psi, rows, cols, S, X, Y, w["eps"], grad_form=True), rows, cols, X, Y, A))
    nnz = int(rows.numel())
    b_iter = _side_bytes(r[1], nnz, n) + _side_bytes(c[1], nnz, m)
    achieved = b_iter * w["n_iters"] / (t_loop / 1e3) / 1e9
    peak, peak_kind = measured_peak_gbs()
    return {"support": round(t_sup, 3), "cost_csr_tiles": round(t_prep, 3),
            "solve_loop": round(t_loop, 3), "plan_and_gradient": round(t_exp, 3), "nnz": nnz,
            "sides": {"row": "tiled" if tl[0] is not None else "exact",
                      "col": "tiled" if tl[1] is not None else "exact"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "peak_source": peak_kind, "traffic": None,
                         "kernel": "the solve loop of one outer step (200 iterations)"}}


def run_cfg5(args):
    """N = M = 2^24.  One GPU: the whole solve.  Under torch.distributed.run the
    same fixed problem is partitioned over the ranks (strong scaling).  Fixed
    iterations; K = min(--steps, 300) timed after the warm-up."""
    import sinkslot_b200
    from sinkslot_b200.sinkhorn_solvers import build_tiles, sinkslot_alternating_b200, tiles_pay_off
    from sinkslot_b200.solver import _to_csr, cost_and_lam, sot_plan_coo

    world, rank, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    torch.backends.cuda.matmul.allow_tf32 = False
    sinkslot_b200.load_library()
    w = CONFIGS["cfg5"]
    n, m = w["n"], w["m"]
    x, y, a, b = make_inputs(0, w)
    X, Y, A, B = (t.to(dev) for t in (x, y, a, b))
    stream = torch.cuda.current_stream(dev)
    K = max(1, min(args.steps, w["n_iters"]))
    peak, peak_kind = measured_peak_gbs()
    if world == 1:
        def setup():
            rows, cols, S = sot_plan_coo(X, Y, A, B, L=w["L"], seed=w["proj_seed"], chunk=8)
            lam, _ = cost_and_lam(X, Y, rows, cols, S, w["eps"])
            del S
            nnz = int(rows.numel())
            r = _to_csr(rows, cols, lam, n, want_perm=False)
            c = _to_csr(cols, rows, lam, m, want_perm=False)
            del rows, cols, lam
            tl = (build_tiles(r[0], r[1], r[2], n, m) if tiles_pay_off(n, m, nnz) else None,
                  build_tiles(c[0], c[1], c[2], m, n) if tiles_pay_off(m, n, nnz) else None)
            return nnz, (r[0], r[1], r[2], c[0], c[1], c[2], A.log(), B.log(), n, m), tl

        (nnz, csr, tl), setup_cold_ms = _timed(stream, setup)
        del csr, tl
        torch.cuda.empty_cache()
        (nnz, csr, tl), setup_ms = _timed(stream, setup)
        sinkslot_alternating_b200(*csr, max(args.warmup, 3), tiles=tl)
        sampler = ClockSampler(local)
        sampler.start()
        _, ms = _timed(stream, lambda: sinkslot_alternating_b200(*csr, K, tiles=tl))
        clocks = sampler.stop()
        b_iter = _side_bytes(csr[1], nnz, n) + _side_bytes(csr[4], nnz, m)
        sides = {"row": side_kind(tl[0], n, m, nnz), "col": side_kind(tl[1], m, n, nnz)}
        achieved = b_iter * K / (ms / 1e3) / 1e9
        launches = K * (SIDE_LAUNCHES[sides["row"]] + SIDE_LAUNCHES[sides["col"]])
        del csr, tl
        torch.cuda.empty_cache()
    else:
        from sinkslot_b200.sharded import ShardedSolver

        def make_solver():
            return ShardedSolver(X, Y, A, B, w["eps"], L=w["L"], seed=w["proj_seed"], chunk=8)

        # the first construction pays the communicators and IPC mappings
        (solver), setup_cold_ms = _timed(stream, make_solver)
        setup_cold_ms = max_over_ranks(setup_cold_ms, world, dev)
        solver.close()
        del solver
        torch.cuda.empty_cache()
        barrier(world)
        (solver), setup_ms = _timed(stream, make_solver)
        setup_ms = max_over_ranks(setup_ms, world, dev)
        nnz = solver.nnz
        solver.solve(max(args.warmup, 3), copy_out=False)
        sampler = ClockSampler(local) if rank == 0 else None
        if sampler:
            sampler.start()
        barrier(world)
        _, ms = _timed(stream, lambda: solver.solve(K, copy_out=False))
        barrier(world)
        clocks = sampler.stop() if sampler else None
        ms = max_over_ranks(ms, world, dev)
        b_iter = (_side_bytes(solver.row[1], solver.row[3], solver.nr) +
                  _side_bytes(solver.col[1], solver.col[3], solver.nc))
        sides = {"row": side_kind(solver.r_tiles, solver.nr, m, solver.row[3]),
                 "col": side_kind(solver.c_tiles, solver.nc, n, solver.col[3])}
        achieved = -max_over_ranks(-(b_iter * K / (ms / 1e3) / 1e9), world, dev)
        # per half-step: the side's kernels over the rank's slice, the publish, the epoch wait
        launches = K * (SIDE_LAUNCHES[sides["row"]] + SIDE_LAUNCHES[sides["col"]] + 4)
        solver.close()
        del solver
        torch.cuda.empty_cache()
    value = K / (ms / 1e3)

    # end to end through the public API from pinned host buffers: support build,
    # the whole solve (its iteration count), potentials back
    from sinkslot_b200 import sinkslot_solve
    from sinkslot_b200.sharded import sinkslot_solve_sharded
    xh, yh, ah, bh = (t.pin_memory() for t in (x, y, a, b))
    phi_h = torch.empty(n).pin_memory()
    psi_h = torch.empty(m).pin_memory()

    def e2e_step():
        args_d = (xh.to(dev, non_blocking=True), yh.to(dev, non_blocking=True),
                  ah.to(dev, non_blocking=True), bh.to(dev, non_blocking=True),
                  w["eps"], w["L"], w["proj_seed"], w["n_iters"])
        r = sinkslot_solve(*args_d, chunk=8) if world == 1 else \
            sinkslot_solve_sharded(*args_d, chunk=8)
        phi_h.copy_(r.phi, non_blocking=True)
        psi_h.copy_(r.psi, non_blocking=True)
        del r

    barrier(world)
    _, e2e_ms = _timed(stream, e2e_step)
    barrier(world)
    e2e_ms = max_over_ranks(e2e_ms, world, dev)
    e2e = {"value": round(w["n_iters"] / (e2e_ms / 1e3), 2), "unit": UNIT,
           "h2d_bytes_per_step": sum(t.numel() * t.element_size() for t in (x, y, a, b)),
           "d2h_bytes_per_step": (n + m) * 4,
           "step": ("sinkslot_solve" if world == 1 else "sinkslot_solve_sharded") +
                   "(...) from pinned host x, y, a, b: support build + %d iterations + "
                   "potentials back" % w["n_iters"]}
    if rank == 0:
        line = _base_line("cfg5", w, value, UNIT, world, K, max(args.warmup, 3), ms / K, clocks, {
            "nnz": nnz, "setup_ms": round(setup_ms, 1), "setup_cold_ms": round(setup_cold_ms, 1),
            "sides": sides,
            "parallelism": "single GPU" if world == 1 else
            f"rows and columns partitioned over {world} GPUs; potential slices exchanged by "
            f"peer stores after every half-step",
            "l2": "inputs larger than L2: %.2f GB of CSR+CSC streamed per rank per iteration"
                  % (b_iter / 1e9)})
        line["roofline"] = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                            "unit": "GB/s", "frac": round(achieved / peak, 4),
                            "peak_source": peak_kind, "traffic": None,
                            "kernel": "per rank: both half-steps per iteration, algorithmic "
                                      "bytes of the rank's slices over the loop time"}
        line["cpu_baseline"] = None
        line["e2e"] = e2e
        line["gpu_launches"] = launches
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def import_reference():
    """The reference package (cai4cai/SinkSLOT's ``sinkslot``) from the unmodified
    install in baseline/_ref, or None when it is not there."""
    path = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(path, "sinkslot")):
        return None
    if path not in sys.path:
        sys.path.insert(0, path)
    try:
        import sinkslot
        from sinkslot import sinkhorn_solvers  # noqa: F401
    except Exception:
        return None
    return sinkslot


def triton_reference_leg(X, Y, A, B, w, steps: int, ours: float):
    """The reference's own GPU kernel on this device: its Triton segmented LSE
    (sinkslot/sinkhorn_solvers.py:45-94) driven by its alternating loop
    (:195-289) over its own CSR/CSC, built by its CUDA pipeline (the
    "sinkslotcuda" method of its benchmark harness: CUDA builder, Triton cost,
    narrow keys).  `steps` iterations timed with CUDA events after warm-up.
    None when the reference package is not importable or Triton fails."""
    ref = import_reference()
    if ref is None:
        return None
    try:
        from sinkslot import sinkhorn_solvers as rss
        from sinkslot import solver as rs
        n, m = w["n"], w["m"]
        dev = X.device
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        rows, cols, S = rs.sot_plan_coo(X, Y, A, B, L=w["L"], seed=w["proj_seed"],
                                        ot1d=rs._ot_1d_coo_batched_cuda)
        cost = rs.sparse_sqeuclidean_cost(X, Y, rows, cols, use_triton=True)
        lam = S.clamp_min(torch.finfo(S.dtype).tiny).log() - cost / w["eps"]
        R = rs.to_csr(rows, cols, lam, n, narrow_key=True)
        C = rs.to_csr(cols, rows, lam, m, narrow_key=True)
        torch.cuda.synchronize(dev)
        setup_ms = (time.perf_counter() - t0) * 1e3
        nnz = int(rows.numel())
        del rows, cols, S, cost, lam
        la, lb = A.log(), B.log()
        args = (R[0], R[1], R[2], C[0], C[1], C[2], la, lb, n, m)
        rss.sinkslot_alternating_triton(*args, 5)  # JIT compile + warm-up
        stream = torch.cuda.current_stream(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(dev)
        e0.record(stream)
        rss.sinkslot_alternating_triton(*args, steps)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        ms = e0.elapsed_time(e1)
        v = steps / (ms / 1e3)
        b_iter = nnz * (R[1].element_size() + 4) + nnz * (C[1].element_size() + 4) + 16 * (n + m)
        return {"value": round(v, 2), "unit": UNIT, "steps": steps,
                "gbs": round(b_iter * v / 1e9, 1), "nnz": nnz, "setup_ms": round(setup_ms, 1),
                "speedup_of_this_build": round(ours / v, 3) if v > 0 else None,
                "kind": "the reference's Triton kernel _seg_lse_online_kernel in its "
                        "sinkslot_alternating_triton loop, on this B200, over its own "
                        "CSR/CSC (unmodified install in baseline/_ref)"}
    except Exception as exc:  # the comparison is reported, never required
        return {"unavailable": f"{type(exc).__name__}: {exc}"[:300]}


def cpu_baseline_from_support(rows, cols, lam, log_a, log_b, w, budget_s: float = 15.0):
    """The oracle's torch-backend iteration (C, OpenMP, all host threads) on the
    same support, a bounded number of iterations."""
    from oracle import oracle as O
    O.build()
    it = O.IterationTimer(rows.cpu().numpy(), cols.cpu().numpy(), lam.cpu().numpy(),
                          log_a.cpu().numpy(), log_b.cpu().numpy(), w["n"], w["m"])
    t0 = time.perf_counter()
    it.run(1)
    t1 = time.perf_counter() - t0
    k = int(max(1, min(50, budget_s / max(t1, 1e-6))))
    t0 = time.perf_counter()
    it.run(k)
    dt = time.perf_counter() - t0
    it.close()
    return {"value": round(k / dt, 4), "unit": UNIT, "cores": O.num_threads(), "kind": "port",
            "sample": f"{k} alternating iterations of the full workload (nnz={rows.numel()}) "
                      f"after 1 untimed; support built once, untimed"}


# --------------------------------------------------------------------------
# the reference arm: the reference algorithm's CPU implementation (oracle port)
# --------------------------------------------------------------------------
def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    from oracle import oracle as O
    O.build()
    w = WORKLOAD
    x, y, a, b = make_inputs(0)
    t0 = time.perf_counter()
    rows, cols, S = O.sot_plan_coo(x.numpy(), y.numpy(), a.numpy(), b.numpy(), w["L"],
                                   w["proj_seed"], builder="cuda_on_cpu")
    cost = O.sqeuclid_cost(x.numpy(), y.numpy(), rows, cols)
    lam = O.lam_values(S, cost, w["eps"])
    setup_s = time.perf_counter() - t0
    la = np.log(a.numpy()).astype(np.float32)
    lb = np.log(b.numpy()).astype(np.float32)
    it = O.IterationTimer(rows, cols, lam, la, lb, w["n"], w["m"])
    it.run(1)  # warm-up (bounded: one iteration)
    t0 = time.perf_counter()
    it.run(1)
    t1 = time.perf_counter() - t0
    k = int(max(1, min(args.steps, 120.0 / max(t1, 1e-6))))
    t0 = time.perf_counter()
    it.run(k)
    dt = time.perf_counter() - t0
    it.close()
    value = k / dt
    cores = O.num_threads()
    sample = (f"{k} of the requested {args.steps} alternating iterations of the full workload "
              f"(nnz={rows.size}), after 2 untimed; support built once on the CPU "
              f"({setup_s:.1f} s, untimed)")
    line = {
        "metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": world,
        "steps": k, "warmup": args.warmup, "ms_per_step": round(dt / k * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "impl": "reference",
        "config": {"workload": WORKLOAD_NAME, "n": w["n"], "m": w["m"], "d": w["d"],
                   "L": w["L"], "eps": w["eps"], "nnz": int(rows.size),
                   "parallelism": f"host CPU, {cores} threads"},
        "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawTextHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--config", choices=["cfg1", "cfg2", "cfg3", "cfg4", "cfg5"], default="cfg2",
                    help="workload: cfg2 the headline (default); cfg1 N=M=10^4 (small, "
                         "launch-bound); cfg3 colour-transfer shape; cfg4 gradient flow; cfg5 "
                         "N=M=2^24 (strong scaling under torchrun)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-triton", action="store_true",
                    help="skip timing the reference's Triton kernel on the same device")
    ap.add_argument("--plain", action="store_true",
                    help="time the exact half-step kernel alone (no shared-memory tiles)")
    ap.add_argument("--replicas", action="store_true",
                    help="N > 1: one independent 2^20 problem per GPU instead of one "
                         "partitioned problem")
    ap.add_argument("--log2n", type=int, default=20,
                    help="points per cloud = 2^log2n (20: the headline problem; smaller sizes "
                         "are for profiling captures)")
    ap.add_argument("--tiles-kind", choices=["auto", "staged", "two_pass"], default="auto",
                    help="how sides with a tiled layout run (auto: by the cost of staging)")
    args = ap.parse_args()
    if args.impl == "b200" and args.tiles_kind != "auto":
        from sinkslot_b200.sinkhorn_solvers import set_tiles_kind
        set_tiles_kind(args.tiles_kind)
    if args.log2n != 20:
        global WORKLOAD_NAME
        WORKLOAD["n"] = WORKLOAD["m"] = 1 << args.log2n
        WORKLOAD_NAME = WORKLOAD_NAME.replace("N=M=2^20", f"N=M=2^{args.log2n}")
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.config == "cfg1":
        run_cfg1(args)
    elif args.config == "cfg3":
        run_cfg3(args)
    elif args.config == "cfg4":
        run_cfg4(args)
    elif args.config == "cfg5":
        run_cfg5(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
