"""The row/column-partitioned solve on two or more GPUs of one node against the
single-GPU solve of the same problem (one process per GPU, NCCL for set-up
and stop checks, peer stores for the potentials).  The support, built across
the ranks (each builds a range of the slices; entries meet at their row and
column owners), equals the single build bit for bit.

Tolerance: rtol 1e-4 / atol scaled like the tiled-vs-exact comparison (the
ranks' tiled layouts cut the rows into different panels, so the exact pass
takes back different rows; both are fp32 with exact fixed-point row sums).
Skipped with fewer than two GPUs.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(n, m, seed, dev):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(n, 3, generator=g)
    y = torch.randn(m, 3, generator=g) + 1.0
    a = -torch.log(torch.rand(n, generator=g).clamp_min(1e-12))
    b = -torch.log(torch.rand(m, generator=g).clamp_min(1e-12))
    return x.to(dev), y.to(dev), (a / a.sum()).to(dev), (b / b.sum()).to(dev)


CASES = [
    # n, m, variant, stop_mode, eps, L
    (200000, 150000, "alternating", "fixed", 0.01, 32),
    (60000, 70000, "symmetric", "fixed", 0.05, 16),
    (40000, 40000, "alternating", "marginal", 0.05, 16),
    (30000, 25000, "symmetric", "potential", 0.05, 16),
    (1001, 999, "alternating", "fixed", 0.05, 8),  # slices not multiples of the panel size
]


def _rank(rank, world, port, q, kind="auto"):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    import datetime
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120), device_id=dev)
    try:
        torch.backends.cuda.matmul.allow_tf32 = False
        import sinkslot_b200
        from sinkslot_b200 import sinkslot_solve
        from sinkslot_b200.sharded import sinkslot_solve_sharded
        sinkslot_b200.load_library()
        from sinkslot_b200.sinkhorn_solvers import set_tiles_kind
        set_tiles_kind(kind)  # every rank and the single-GPU solve alike
        out = []
        for n, m, variant, mode, eps, L in CASES:
            x, y, a, b = _inputs(n, m, 5, dev)
            kw = dict(eps=eps, L=L, seed=0, n_iters=60, stop_mode=mode, stop_max_iter=3000,
                      stop_tol=1e-5, stop_check_every=5, variant=variant)
            rs = sinkslot_solve_sharded(x, y, a, b, **kw)
            r1 = sinkslot_solve(x, y, a, b, **kw) if rank == 0 else None
            sup = (rs.rows.cpu(), rs.cols.cpu(), rs.S.cpu())
            if r1 is not None:
                # the support built across the ranks is the single build, bit for bit
                assert torch.equal(rs.rows, r1.rows) and torch.equal(rs.cols, r1.cols)
                assert torch.equal(rs.S, r1.S)
            out.append((rs.phi.cpu(), rs.psi.cpu(), rs.iters_run, rs.converged, rs.final_viol,
                        None if r1 is None else (r1.phi.cpu(), r1.psi.cpu(), r1.iters_run,
                                                 r1.converged, r1.final_viol), sup))
        q.put((rank, out, None))
    except Exception as e:  # reported by the parent
        q.put((rank, None, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("kind", ["auto", "two_pass"])
@pytest.mark.parametrize("world", [2, 4])
def test_sharded_solve_matches_single_gpu(world, kind):
    """kind "two_pass": the tiled sides (the first case's slices) run the
    two-pass half-step, whose sum pass stores into the peers' buffers."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q, kind)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        rank, out, err = q.get(timeout=600)
        assert err is None, f"rank {rank}: {err}"
        res[rank] = out
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for ci, (n, m, variant, mode, eps, L) in enumerate(CASES):
        single = res[0][ci][5]
        for rank in range(world):
            phi, psi, it, conv, viol, _, sup = res[rank][ci]
            assert all(torch.equal(u, v) for u, v in zip(sup, res[0][ci][6]))
            sphi, spsi, sit, sconv, sviol = single
            if mode == "fixed":
                assert it == sit
            else:
                # same stop semantics; the check value may cross the threshold
                # one interval apart because the two solves differ in rounding
                assert conv == sconv and abs(it - sit) <= 5
            atol_p = 1e-5 + 2e-7 * float(sphi.abs().max())
            atol_q = 1e-5 + 2e-7 * float(spsi.abs().max())
            if mode == "fixed":
                torch.testing.assert_close(phi, sphi, rtol=1e-4, atol=atol_p)
                torch.testing.assert_close(psi, spsi, rtol=1e-4, atol=atol_q)
            else:
                # points whose weight vanishes in the fp32 cumulative sums have
                # empty rows and potential +inf in both solves; the (+c, -c)
                # shift is taken over the finite entries
                fin = torch.isfinite(phi) & torch.isfinite(sphi)
                c = float((phi[fin] - sphi[fin]).double().mean()) if fin.any() else 0.0
                torch.testing.assert_close(phi - c, sphi, rtol=0, atol=5e-3)
                torch.testing.assert_close(psi + c, spsi, rtol=0, atol=5e-3)
        # every rank holds the same full potentials
        for rank in range(1, world):
            assert torch.equal(res[rank][ci][0], res[0][ci][0])
            assert torch.equal(res[rank][ci][1], res[0][ci][1])
