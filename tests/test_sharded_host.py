"""Host logic of the row/column-partitioned solve, on CPU.

The partition and CSR slicing are checked directly.  The chunked stop logic
(``plan_chunks`` + ``drive``) is checked against the single-process loop of
the oracle (the reference's loop semantics, sinkslot/sinkhorn_solvers.py:
443-588) by running two and three gloo ranks, each computing only its own row
and column slices with the oracle's segmented LSE and exchanging slices with an
all-gather after every half-step -- the data flow the GPU ranks implement with
peer stores.  Same support, same iteration counts and convergence flags,
potentials to fp32 rounding.
"""

from __future__ import annotations

import math
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from sinkslot_b200.sharded import drive, plan_chunks, shard_bounds, slice_csr


@pytest.mark.parametrize("n", [1, 3, 4, 5, 17, 100, 1001])
@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_shard_bounds_partition(n, world):
    covered = []
    for r in range(world):
        s, c = shard_bounds(n, world, r)
        assert s % 4 == 0 and c >= 0 and s + c <= n
        covered.extend(range(s, s + c))
    assert covered == list(range(n))


def test_slice_csr_reassembles():
    g = torch.Generator().manual_seed(0)
    counts = torch.randint(0, 6, (37,), generator=g)
    ptr = torch.zeros(38, dtype=torch.int32)
    ptr[1:] = torch.cumsum(counts, 0)
    nnz = int(ptr[-1])
    idx = torch.randint(0, 50, (nnz,), generator=g).to(torch.int16)
    vals = torch.randn(nnz, generator=g)
    parts = [slice_csr(ptr, idx, vals, *shard_bounds(37, 3, r)) for r in range(3)]
    assert all(p[0].dtype == torch.int32 and int(p[0][0]) == 0 for p in parts)
    assert torch.equal(torch.cat([p[1] for p in parts]), idx)
    assert torch.equal(torch.cat([p[2] for p in parts]), vals)
    assert sum(p[3] for p in parts) == nnz
    lens = torch.cat([p[0][1:] - p[0][:-1] for p in parts])
    assert torch.equal(lens, counts.to(torch.int32))


def _single_loop_checks(mode, max_iter, every):
    """Iteration counts after which the single-GPU loop checks."""
    out = []
    for it in range(max_iter):
        chk = (it + 1) % every == 0 or (mode == "marginal" and it + 1 == max_iter)
        if chk:
            out.append(it + 1)
    return out


@pytest.mark.parametrize("mode", ["potential", "marginal"])
@pytest.mark.parametrize("max_iter,every", [(20, 5), (23, 5), (3, 5), (7, 1), (12, 7)])
def test_plan_chunks_checks_where_the_single_loop_checks(mode, max_iter, every):
    it, ends = 0, []
    while it < max_iter:
        k, check = plan_chunks(mode, it, 0, max_iter, every)
        assert k >= 1
        it += k
        if check:
            ends.append(it)
    assert it == max_iter
    assert ends == _single_loop_checks(mode, max_iter, every)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _problem():
    from oracle import oracle
    rng = np.random.default_rng(3)
    n, m = 61, 47
    x = rng.standard_normal((n, 2)).astype(np.float32)
    y = (rng.standard_normal((m, 2)) + 0.5).astype(np.float32)
    a = rng.random(n).astype(np.float32) + 0.2
    b = rng.random(m).astype(np.float32) + 0.2
    a /= a.sum()
    b /= b.sum()
    rows, cols, S = oracle.sot_plan_coo(x, y, a, b, L=8, seed=0, builder="cpu")
    eps = 0.1
    lam = oracle.lam_values(S, oracle.sqeuclid_cost(x, y, rows, cols), eps)
    return n, m, rows, cols, lam, np.log(a), np.log(b), eps


def _rank_main(rank, world, port, variant, mode, q):
    from oracle import oracle
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        n, m, rows, cols, lam, la, lb, eps = _problem()
        alpha, tol, every, max_iter, n_iters = 0.5, 1e-5, 3, 400, 25
        w_old, w_new = np.float32(1 - alpha), np.float32(alpha)
        r0, nr = shard_bounds(n, world, rank)
        c0, nc = shard_bounds(m, world, rank)
        rm = (rows >= r0) & (rows < r0 + nr)
        cm = (cols >= c0) & (cols < c0 + nc)
        st = {"phi": [np.zeros(n, np.float32), np.zeros(n, np.float32)],
              "psi": [np.zeros(m, np.float32), np.zeros(m, np.float32)], "cur": 0,
              "prev": {True: np.zeros(nr, np.float32), False: np.zeros(nc, np.float32)}}

        def gather(local, total, bounds):
            size = max(bounds(r)[1] for r in range(world))
            t = torch.zeros(size)
            t[:local.size] = torch.from_numpy(local)
            parts = [torch.zeros(size) for _ in range(world)]
            dist.all_gather(parts, t)
            full = np.zeros(total, np.float32)
            for r in range(world):
                s, c = bounds(r)
                full[s:s + c] = parts[r][:c].numpy()
            return full

        def half(row, out_buf, chk, write):
            c = st["cur"]
            if row:
                self_old = st["phi"][c][r0:r0 + nr]
                other = st["psi"][c]
                cand = oracle.seg_lse_coo(rows[rm] - r0, cols[rm], lam[rm], other, la[r0:r0 + nr],
                                          nr)
                base = la[r0:r0 + nr]
            else:
                self_old = st["psi"][c][c0:c0 + nc]
                other = st["phi"][c]
                cand = oracle.seg_lse_coo(cols[cm] - c0, rows[cm], lam[cm], other, lb[c0:c0 + nc],
                                          nc)
                base = lb[c0:c0 + nc]
            nv = cand if variant == "alternating" else (w_old * self_old + w_new * cand).astype(
                np.float32)
            val = 0.0
            if chk == 1:  # potential
                d = np.abs(nv - st["prev"][row])
                val = float(d.max()) if d.size else 0.0
                st["prev"][row] = nv.copy()
            elif chk == 2:  # marginal
                ea = np.exp(base)
                d = np.abs(ea * np.exp(self_old - cand) - ea)
                val = (math.nan if np.isnan(d).any() else float(d.max())) if d.size else 0.0
            if write:
                key = "phi" if row else "psi"
                bounds = (lambda r: shard_bounds(n, world, r)) if row else (
                    lambda r: shard_bounds(m, world, r))
                st[key][out_buf] = gather(nv, n if row else m, bounds)
            return val

        def run_chunk(it0, k, check):
            c0v = c1v = 0.0
            for j in range(k):
                last = j == k - 1
                chk = check if last else 0
                c = st["cur"]
                if variant == "alternating":
                    c0v = half(True, c, chk, True)
                    c1v = half(False, c, chk, True)
                else:
                    c0v = half(True, 1 - c, 1 if chk == 1 else 0, True)
                    c1v = half(False, 1 - c, 1 if chk == 1 else 0, True)
                    st["cur"] = 1 - c
                    if chk == 2:
                        c0v = half(True, None, 2, False)
                        c1v = half(False, None, 2, False)
            return c0v, c1v

        def reduce_max(a0, a1):
            nan = [math.isnan(a0), math.isnan(a1)]
            t = torch.tensor([0.0 if nan[0] else a0, 0.0 if nan[1] else a1, float(nan[0]),
                              float(nan[1])], dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            v = t.tolist()
            return (math.nan if v[2] else v[0]), (math.nan if v[3] else v[1])

        it, conv, viol = drive(run_chunk, reduce_max, mode, n_iters, max_iter, every, tol, eps,
                               alpha, variant)
        q.put((rank, st["phi"][st["cur"]], st["psi"][st["cur"]], it, conv, viol))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,variant,mode", [
    (2, "alternating", "fixed"), (2, "alternating", "marginal"), (2, "symmetric", "potential"),
    (2, "symmetric", "marginal"), (3, "alternating", "potential"), (3, "symmetric", "fixed")])
def test_sharded_loop_matches_single_loop(world, variant, mode):
    from oracle import oracle
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, variant, mode, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    n, m, rows, cols, lam, la, lb, eps = _problem()
    phi, psi, it, conv, viol = oracle.solve_loops(
        rows, cols, lam, la, lb, n, m, 25, variant=variant, stop_mode=mode, stop_max_iter=400,
        stop_tol=1e-5, stop_check_every=3, eps=eps, alpha=0.5)
    for rank, rphi, rpsi, rit, rconv, rviol in results:
        assert rit == it and rconv == conv, (rank, rit, it, rconv, conv)
        np.testing.assert_allclose(rphi, phi, rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(rpsi, psi, rtol=1e-5, atol=1e-5)
        if mode != "fixed":
            assert rviol == pytest.approx(viol, rel=1e-3, abs=1e-9)


def _dying_rank_main(rank, world, port, q):
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=10))
    try:
        def run_chunk(it0, k, check):
            if rank == 1 and it0 > 0:
                raise RuntimeError("rank 1 stops between chunks")
            return 0.5, 0.5

        def reduce_max(a0, a1):
            t = torch.tensor([a0, a1], dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return tuple(t.tolist())

        drive(run_chunk, reduce_max, "marginal", 0, 100, 5, 1e-9, 0.05, 0.5, "alternating")
        q.put((rank, "finished"))
    except Exception as e:  # the surviving rank must see an error, not hang
        q.put((rank, f"error {type(e).__name__}"))
    finally:
        dist.destroy_process_group()


def test_a_rank_that_leaves_between_chunks_is_an_error_on_the_others():
    """A rank leaves between chunks (no kernel in flight): the next stop check's
    reduction fails on the surviving rank with an error instead of waiting."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dying_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=90) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    assert got[1].startswith("error RuntimeError")
    assert got[0].startswith("error"), got[0]


class _OracleOps:
    """The device steps of build_partitioned_support, done by the oracle on CPU."""

    def project_t(self, X, theta):
        from oracle import oracle
        return torch.from_numpy(oracle.project(X.numpy(), theta.numpy()))

    def ot1d(self, PXt, PYt, a, b, scan_rows):
        from oracle import oracle
        R, C, M = oracle.ot1d(PXt.numpy(), PYt.numpy(), a.numpy(), b.numpy(), builder="cuda",
                              scan_rows=scan_rows)
        return torch.from_numpy(R), torch.from_numpy(C), torch.from_numpy(M)

    def partition(self, seg, other, vals, bounds):
        s = seg.numpy()
        part = np.searchsorted(np.asarray(bounds[1:-1]), s, side="right")
        order = np.argsort(part, kind="stable")
        counts = np.bincount(part, minlength=len(bounds) - 1).tolist()
        return seg[order], other[order], vals[order], counts

    def coalesce(self, R, C, M, n, m, L):
        from oracle import oracle
        r, c, S = oracle.coalesce(R.numpy(), C.numpy(), M.numpy(), m, L, builder="cuda")
        return torch.from_numpy(r), torch.from_numpy(c), torch.from_numpy(S)

    def cost_lam(self, X, Y, rows, cols, S, eps):
        from oracle import oracle
        cost = oracle.sqeuclid_cost(X.numpy(), Y.numpy(), rows.numpy(), cols.numpy())
        return torch.from_numpy(oracle.lam_values(S.numpy(), cost, eps))


def _support_problem():
    rng = np.random.default_rng(5)
    n, m = 130, 97
    x = rng.standard_normal((n, 3)).astype(np.float32)
    y = (rng.standard_normal((m, 3)) + 0.7).astype(np.float32)
    a = (rng.random(n) + 0.1).astype(np.float32)
    b = (rng.random(m) + 0.1).astype(np.float32)
    return x, y, a / a.sum(), b / b.sum(), 12, 0.05


def _support_rank_main(rank, world, port, chunk, q):
    from sinkslot_b200.sharded import build_partitioned_support
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x, y, a, b, L, eps = _support_problem()
        t = [torch.from_numpy(v) for v in (x, y, a, b)]
        (rows, cols, S, lam), (cc, cr, cl) = build_partitioned_support(
            *t, eps, L, 0, chunk, None, ops=_OracleOps())
        q.put((rank, rows.numpy(), cols.numpy(), S.numpy(), lam.numpy(), cc.numpy(),
               cr.numpy(), cl.numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,chunk", [(2, None), (3, 2), (4, 1), (3, 5), (2, 7)])
def test_partitioned_support_equals_the_single_build(world, chunk):
    """Slices built on different ranks, entries routed to their row owners
    (all-to-all), coalesced there, then routed to their column owners: every
    rank's rows equal the single build's rows (rows, cols and S bit-exact, in
    key order), and its columns' entries arrive in the CSC order of the single
    build."""
    from oracle import oracle
    from sinkslot_b200.sharded import owner_bounds
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_support_rank_main, args=(r, world, port, chunk, q))
             for r in range(world)]
    for p in procs:
        p.start()
    got = dict((r[0], r[1:]) for r in (q.get(timeout=120) for _ in range(world)))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    x, y, a, b, L, eps = _support_problem()
    rows, cols, S = oracle.sot_plan_coo(x, y, a, b, L, 0, chunk=chunk, builder="cuda")
    lam = oracle.lam_values(S, oracle.sqeuclid_cost(x, y, rows, cols), eps)
    rb, cb = owner_bounds(len(x), world), owner_bounds(len(y), world)
    order = np.argsort(cols, kind="stable")  # CSC order of the single build
    for g in range(world):
        r, c, s, lm, cc, cr, cl = got[g]
        mine = (rows >= rb[g]) & (rows < rb[g + 1])
        np.testing.assert_array_equal(r, rows[mine])
        np.testing.assert_array_equal(c, cols[mine])
        np.testing.assert_array_equal(s, S[mine])
        np.testing.assert_array_equal(lm, lam[mine])
        colmine = order[(cols[order] >= cb[g]) & (cols[order] < cb[g + 1])]
        o = np.argsort(cc, kind="stable")
        np.testing.assert_array_equal(cc[o], cols[colmine])
        np.testing.assert_array_equal(cr[o], rows[colmine])
        np.testing.assert_array_equal(cl[o], lam[colmine])
