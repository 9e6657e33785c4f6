"""Generate the golden fixtures in this directory from the reference package.

Run once, on a machine where the reference source tree is available:

    python tests/golden/make_golden.py /path/to/SinkSLOT

It imports the reference (``<path>/torch-ext/sinkslot``) and records its CPU
outputs (``backend="torch"``) for a few seeded problems.  The fixtures are the
reference's own numbers; the tests compare the CPU oracle (and, on a GPU, the
sm_100a kernels) against them.

Tie order: torch's CPU argsort is not stable, while the reference's CUDA run
sorts with CUB's stable radix sort.  For problems whose projections contain
exact ties the two reference runs pair tied points differently.  Those fixtures
are generated with ``torch.argsort`` wrapped to ``stable=True`` -- the CUDA tie
order, reproduced on CPU -- and say so in their ``meta`` entry; the raw
(unwrapped) CPU support size is recorded next to it.
"""

from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(np.asarray(a)).tobytes()).hexdigest()


def problem_nonuniform(n, m, d, seed, shift=1.0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(n, d, generator=g)
    y = torch.randn(m, d, generator=g) + shift
    a = torch.rand(n, generator=g) + 0.1
    b = torch.rand(m, generator=g) + 0.1
    return x, y, a / a.sum(), b / b.sum()


def main(ref_root: str) -> None:
    sys.path.insert(0, os.path.join(ref_root, "torch-ext"))
    import sinkslot.solver as RS
    from sinkslot import sinkslot_solve, slot_grad, sparse_transport_plan, sparse_barycentric_map
    from sinkslot import SamplesLoss
    from sinkslot.solver import (sot_plan_coo, sparse_sqeuclidean_cost, _ot_1d_coo_batched,
                                 _ot_1d_coo_batched_cuda, get_random_projections)

    torch.set_num_threads(1)
    orig_argsort = torch.argsort

    def stable_argsort(t, dim=-1, descending=False, stable=False, **kw):
        return orig_argsort(t, dim=dim, descending=descending, stable=True)

    def run_case(name, x, y, a, b, eps, L, n_iters, stable_patch, full=True, modes=True):
        out = {}
        meta = {"name": name, "n": x.shape[0], "m": y.shape[0], "d": x.shape[1], "eps": eps,
                "L": L, "n_iters": n_iters, "stable_argsort_patch": stable_patch}
        if stable_patch:
            r0, _, _ = sot_plan_coo(x, y, a, b, L=L, seed=0, ot1d=_ot_1d_coo_batched_cuda)
            meta["nnz_unpatched_cpu"] = int(r0.numel())
            RS.torch.argsort = stable_argsort
        try:
            for tag, ot in (("cudabuilder", _ot_1d_coo_batched_cuda), ("naive", _ot_1d_coo_batched)):
                r, c, S = sot_plan_coo(x, y, a, b, L=L, seed=0, ot1d=ot)
                meta[f"nnz_{tag}"] = int(r.numel())
                meta[f"sha_rows_{tag}"] = sha(r.numpy())
                meta[f"sha_cols_{tag}"] = sha(c.numpy())
                meta[f"sha_S_{tag}"] = sha(S.numpy())
                if full:
                    out[f"rows_{tag}"] = r.numpy()
                    out[f"cols_{tag}"] = c.numpy()
                    out[f"S_{tag}"] = S.numpy()
            res = sinkslot_solve(x, y, a, b, eps, L, seed=0, n_iters=n_iters, backend="torch")
            out["phi_alt"] = res.phi.numpy()
            out["psi_alt"] = res.psi.numpy()
            cost = sparse_sqeuclidean_cost(x, y, res.rows, res.cols, use_triton=False)
            meta["sha_cost"] = sha(cost.numpy())
            if full:
                out["cost"] = cost.numpy()
            res_s = sinkslot_solve(x, y, a, b, eps, L, seed=0, n_iters=n_iters, backend="torch",
                                   variant="symmetric")
            out["phi_sym"] = res_s.phi.numpy()
            out["psi_sym"] = res_s.psi.numpy()
            g = slot_grad(x, y, a, b, eps, L, 0, n_iters, backend="torch")
            out["grad"] = g.numpy()
            loss = SamplesLoss(eps=eps, L=L, n_iters=n_iters, backend="torch")(x, y, a, b)
            meta["loss"] = float(loss)
            if full:
                P = sparse_transport_plan(x, y, a, b, eps=eps, L=L, seed=0, n_iters=n_iters,
                                          backend="torch")
                out["plan_vals"] = P.values().numpy()
                Tx, Ty = sparse_barycentric_map(P, x, y)
                out["Tx"] = Tx.numpy()
                out["Ty"] = Ty.numpy()
            if modes:
                for variant in ("alternating", "symmetric"):
                    for mode, tol in (("marginal", 1e-6), ("potential", 1e-4)):
                        rr = sinkslot_solve(x, y, a, b, eps, L, seed=0, n_iters=20000,
                                            stop_mode=mode, stop_max_iter=20000, stop_tol=tol,
                                            backend="torch", variant=variant)
                        key = f"{variant}_{mode}"
                        meta[f"iters_{key}"] = int(rr.iters_run)
                        meta[f"conv_{key}"] = bool(rr.converged)
                        meta[f"viol_{key}"] = float(rr.final_viol)
                        out[f"phi_{key}"] = rr.phi.numpy()
                        out[f"psi_{key}"] = rr.psi.numpy()
        finally:
            RS.torch.argsort = orig_argsort
        out["x"] = x.numpy()
        out["y"] = y.numpy()
        out["a"] = a.numpy()
        out["b"] = b.numpy()
        out["theta"] = get_random_projections(x.shape[1], L, 0).numpy()
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), meta=json.dumps(meta), **out)
        print(name, meta.get("nnz_cudabuilder"), "saved")

    # 1. the reference tests' small non-uniform problem (test_torch_fallback.py:40-46)
    x, y, a, b = problem_nonuniform(300, 250, 3, 0)
    run_case("small_nonuniform", x, y, a, b, eps=0.05, L=40, n_iters=200, stable_patch=False)

    # 2. the reference bench-test shape (test_sinkslot_bench.py:32-38), d=4
    x, y, a, b = problem_nonuniform(512, 384, 4, 0, shift=1.5)
    run_case("bench_shape", x, y, a, b, eps=0.05, L=32, n_iters=100, stable_patch=False,
             modes=False)

    # 3. the CPU-runnable configuration: N=M=10000, d=2, seed 0, uniform weights,
    #    eps=0.05, L=64, 200 iterations (has exact projection ties)
    torch.manual_seed(0)
    x = torch.randn(10000, 2)
    y = torch.randn(10000, 2)
    a = torch.full((10000,), 1.0 / 10000)
    b = torch.full((10000,), 1.0 / 10000)
    run_case("cfg1", x, y, a, b, eps=0.05, L=64, n_iters=200, stable_patch=True, full=False,
             modes=False)

    # 4. n != m non-uniform with a tie (slice 22 of y)
    x, y, a, b = problem_nonuniform(2000, 3000, 3, 1)
    run_case("unequal_ties", x, y, a, b, eps=0.05, L=50, n_iters=100, stable_patch=True,
             full=False, modes=False)

    # 5. zero weights: a few source and target points carry no mass
    x, y, a, b = problem_nonuniform(200, 180, 2, 3)
    a[::17] = 0.0
    b[::23] = 0.0
    a, b = a / a.sum(), b / b.sum()
    run_case("zero_weights", x, y, a, b, eps=0.1, L=16, n_iters=50, stable_patch=False,
             modes=False)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("SINKSLOT_REF", ""))
