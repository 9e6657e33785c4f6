"""Row/column-partitioned SinkSLOT solve across the GPUs of one node.

One process per GPU (``torch.distributed`` initialised by the caller, e.g.
under ``torchrun``).  Every rank builds the same sliced support (the build is
deterministic for identical inputs), keeps the CSR rows and CSC columns of its
slice, and runs the Sinkhorn loop of ``sinkslot_solve`` on them in
libsinkslot_b200.so (``sinkslot_solve_shard``): after every half-step the rank
stores its potential slice straight into each peer's potential buffer (peer
stores over NVLink through CUDA IPC mappings) and publishes a barrier epoch;
the next half-step waits, bounded, until every peer's epoch has arrived.
``torch.distributed`` carries only the set-up (IPC handles) and the stop
checks (a max-reduction of two floats per check), so every rank takes the same
stop decision at the same iteration, with the semantics of the single-GPU loop
(reference: sinkslot/sinkhorn_solvers.py:195-419).

The partition, the check schedule and the stop decisions are plain host code
(``shard_bounds``, ``slice_csr``, ``plan_chunks``, ``drive``), exercised on CPU
with gloo ranks by the tests.
"""

from __future__ import annotations

import ctypes
import math
from types import SimpleNamespace
from typing import Callable

import torch
import torch.distributed as dist

from . import _lib
from ._lib import call, ptr, stream_of
from .sinkhorn_solvers import (SinkslotSolveResult, _idx_bytes, _resolve_stop_mode, _validate,
                               build_tiles, tiles_pay_off)
from .solver import _to_csr, cost_and_lam, sot_plan_coo

MAX_RANKS = 8
_CHECK_CODE = {"fixed": 0, "potential": 1, "marginal": 2}


def shard_bounds(n: int, world: int, rank: int) -> tuple[int, int]:
    """(start, count) of rank's slice of n items: equal slices of
    ceil(n / world) rounded up to a multiple of 4 (16-byte aligned starts); the
    last slices may be short or empty."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    size = -(-n // world)
    size = (size + 3) // 4 * 4
    if rank * size >= n:
        return n // 4 * 4, 0  # an empty slice (start kept 4-aligned)
    start = rank * size
    return start, min(size, n - start)


def slice_csr(ptr_: torch.Tensor, idx: torch.Tensor, vals: torch.Tensor, start: int,
              count: int):
    """Segments [start, start+count) of a CSR: (ptr rebased to 0 as int32, idx,
    vals, nnz)."""
    lo = int(ptr_[start])
    hi = int(ptr_[start + count])
    p = (ptr_[start:start + count + 1].to(torch.int64) - lo).to(torch.int32).contiguous()
    return p, idx[lo:hi].contiguous(), vals[lo:hi].contiguous(), hi - lo


def plan_chunks(mode: str, it: int, n_iters: int, max_iter: int, every: int) -> tuple[int, int]:
    """(iterations, check) of the next chunk from iteration `it`: the chunk
    ends at the next iteration that checks (check 1 potential / 2 marginal) or
    at the end of the run (check 0).  The checking iterations are those of the
    single-GPU loop: potential mode after iteration it+1 when (it+1) % every
    == 0; marginal mode also at it+1 == max_iter; fixed mode never."""
    if mode == "fixed":
        return max(0, n_iters - it), 0
    k = every - (it % every)
    if it + k <= max_iter:
        return k, _CHECK_CODE[mode]
    left = max_iter - it
    return left, (_CHECK_CODE[mode] if mode == "marginal" else 0)


def _py_max(a: float, b: float) -> float:
    return b if b > a else a  # Python's max(a, b)


def drive(run_chunk: Callable[[int, int, int], tuple[float, float]],
          reduce_max: Callable[[float, float], tuple[float, float]], mode: str, n_iters: int,
          max_iter: int, every: int, tol: float, eps: float, alpha: float, variant: str):
    """The stop logic of the single-GPU loop over chunks.  ``run_chunk(it0, k,
    check)`` runs k iterations and returns this rank's two check maxima;
    ``reduce_max`` makes them global.  Returns (iters_run, converged,
    final_viol) as the reference loops do."""
    if mode == "fixed":
        if n_iters > 0:
            run_chunk(0, n_iters, 0)
        return int(n_iters), None, None
    it = 0
    value = math.inf
    thr = tol if variant == "alternating" else alpha * tol
    while it < max_iter:
        k, check = plan_chunks(mode, it, n_iters, max_iter, every)
        c0, c1 = run_chunk(it, k, check)
        it += k
        if check:
            c0, c1 = reduce_max(c0, c1)
            if mode == "potential":
                value = eps * _py_max(c0, c1)
                if value < thr:
                    return it, True, value
            else:
                value = math.nan if (math.isnan(c0) or math.isnan(c1)) else max(c0, c1)
                if value <= tol:
                    return it, True, value
    return it, False, value


# --------------------------------------------------------------------------
# the support built across the ranks
# --------------------------------------------------------------------------
def slice_range(L: int, world: int, rank: int) -> tuple[int, int]:
    """Slices [l0, l1) of the L slices that rank builds: contiguous ranges in
    rank order, so the ranks' entries, taken in rank order, are in slice order."""
    return rank * L // world, (rank + 1) * L // world


def owner_bounds(n: int, world: int) -> list[int]:
    """world + 1 non-decreasing bounds: rank g owns segments [b[g], b[g+1]),
    the slices of shard_bounds."""
    b = []
    for g in range(world):
        start, count = shard_bounds(n, world, g)
        b.append(start if count > 0 else n)
    return b + [n]


def exchange(arrays, counts, group):
    """All-to-all of equally partitioned arrays: arrays[i] holds, part by part,
    counts[g] entries for rank g; returns the arrays this rank receives, the
    parts of ranks 0, 1, ... in that order, and the received counts."""
    world = dist.get_world_size(group)
    dev = arrays[0].device
    send = torch.tensor([int(c) for c in counts], dtype=torch.int64, device=dev)
    recv = torch.empty(world, dtype=torch.int64, device=dev)
    dist.all_to_all_single(recv, send, group=group)
    rc = [int(v) for v in recv.tolist()]
    out = []
    for a in arrays:
        o = torch.empty(sum(rc), dtype=a.dtype, device=dev)
        dist.all_to_all_single(o, a.contiguous(), rc, [int(c) for c in counts], group=group)
        out.append(o)
    return out, rc


class DeviceOps:
    """The device steps of the partitioned support build, in libsinkslot_b200.so."""

    def __init__(self, device):
        self.dev = device

    def _ws(self, nbytes):
        return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=self.dev)

    def project_t(self, X, theta):
        """(C, n) slice-major projections of X onto theta's rows: the FMA chain
        for d <= 4, cuBLAS's product otherwise (as sot_plan_coo)."""
        from .solver import OWN_PROJECTION_MAX_D, project
        if X.shape[1] <= OWN_PROJECTION_MAX_D:
            return project(X, theta)
        return (X @ theta.T).T.contiguous()

    def ot1d(self, PXt, PYt, a, b, scan_rows):
        from .solver import _ot_1d_coo_batched_cuda
        return _ot_1d_coo_batched_cuda(PXt.T, PYt.T, a, b, scan_rows=scan_rows)

    def partition(self, seg, other, vals, bounds):
        nnz = seg.numel()
        nb = _lib.out_i64()
        call("sinkslot_partition_workspace_bytes", nnz, ctypes.byref(nb))
        ws = self._ws(nb.value)
        so, oo, vo = torch.empty_like(seg), torch.empty_like(other), torch.empty_like(vals)
        parts = len(bounds) - 1
        bh = (ctypes.c_int64 * (parts + 1))(*bounds)
        counts = (ctypes.c_int64 * parts)()
        with torch.cuda.device(self.dev):
            call("sinkslot_partition_coo", ptr(seg), ptr(other), ptr(vals), nnz, bh, parts,
                 ptr(ws), ws.numel(), ptr(so), ptr(oo), ptr(vo), counts, stream_of(self.dev))
        return so, oo, vo, list(counts)

    def coalesce(self, R, Cc, M, n, m, L):
        nraw = R.numel()
        nb = _lib.out_i64()
        call("sinkslot_coalesce_workspace_bytes", nraw, ctypes.byref(nb))
        ws = self._ws(nb.value)
        rows = torch.empty(max(nraw, 1), dtype=torch.int64, device=self.dev)
        cols = torch.empty_like(rows)
        S = torch.empty(max(nraw, 1), dtype=torch.float32, device=self.dev)
        k = _lib.out_i64()
        with torch.cuda.device(self.dev):
            call("sinkslot_coalesce_coo", ptr(R), ptr(Cc), ptr(M), nraw, n, m, L, ptr(ws),
                 ws.numel(), ptr(rows), ptr(cols), ptr(S), ctypes.byref(k), stream_of(self.dev))
        return rows[:k.value], cols[:k.value], S[:k.value]

    def cost_lam(self, X, Y, rows, cols, S, eps):
        return cost_and_lam(X, Y, rows, cols, S, eps)[0]


def build_partitioned_support(X, Y, a, b, eps, L: int, seed: int, chunk, group, ops=None):
    """This rank's part of the sliced support, built across the ranks of `group`
    (every rank holds the same X, Y, a, b):

    1. rank g builds the raw entries of slices slice_range(L, world, g)
       (reference: _ot_1d_coo_batched_cuda, solver.py:107-150), each slice
       with the cumsum association of the batch (`chunk` slices, or all L) that
       holds it in the single-device build;
    2. the entries go to their row's owner (stable partition + all-to-all),
       where they arrive in slice order;
    3. each owner coalesces its rows (solver.py:194-232: duplicates summed in
       slice order, / L) -- the same bits as the single-device build -- and
       computes lam = log S - cost / eps for them;
    4. the coalesced entries go to their column's owner, arriving in row order.

    Returns (rows, cols, S, lam) of the rows this rank owns, sorted by
    rows * m + cols, and (cols, rows, lam) of the columns it owns, in row
    order within each column's run of the concatenation."""
    from .solver import get_random_projections
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    ops = ops if ops is not None else DeviceOps(X.device)
    n, d = X.shape
    m = Y.shape[0]
    theta = get_random_projections(d, L, seed).to(X.dtype).to(X.device)
    l0, l1 = slice_range(L, world, rank)
    step = L if chunk is None else max(1, min(L, int(chunk)))
    parts = []
    for b0 in range(0, L, step):  # the single-device build's batches
        b1 = min(L, b0 + step)
        s0, s1 = max(b0, l0), min(b1, l1)
        if s0 >= s1:
            continue
        t = theta[s0:s1].contiguous()
        parts.append(ops.ot1d(ops.project_t(X, t), ops.project_t(Y, t), a, b, b1 - b0))
    if parts:
        R = torch.cat([p[0] for p in parts])
        Cc = torch.cat([p[1] for p in parts])
        M = torch.cat([p[2] for p in parts])
    else:
        R = torch.zeros(0, dtype=torch.int64, device=X.device)
        Cc = torch.zeros(0, dtype=torch.int64, device=X.device)
        M = torch.zeros(0, dtype=torch.float32, device=X.device)
    del parts
    R, Cc, M, counts = ops.partition(R, Cc, M, owner_bounds(n, world))
    (R, Cc, M), _ = exchange([R, Cc, M], counts, group)
    rows, cols, S = ops.coalesce(R, Cc, M, n, m, L)
    del R, Cc, M
    lam = ops.cost_lam(X, Y, rows, cols, S, eps)
    c_cols, c_rows, c_lam, counts = ops.partition(cols, rows, lam, owner_bounds(m, world))
    (c_cols, c_rows, c_lam), _ = exchange([c_cols, c_rows, c_lam], counts, group)
    return (rows, cols, S, lam), (c_cols, c_rows, c_lam)


def _reduce_max_dist(group, device):
    def reduce_max(c0: float, c1: float) -> tuple[float, float]:
        nan = [math.isnan(c0), math.isnan(c1)]
        t = torch.tensor([0.0 if nan[0] else c0, 0.0 if nan[1] else c1,
                          float(nan[0]), float(nan[1])], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
        v = t.tolist()
        return (math.nan if v[2] else v[0]), (math.nan if v[3] else v[1])
    return reduce_max


class _SharedState:
    """This rank's peer-writable buffer (phi[k] | psi[k] | flags) and the
    mapped buffers of every peer."""

    def __init__(self, n: int, m: int, nbuf: int, group, device):
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.n4 = (n + 3) // 4 * 4
        self.m4 = (m + 3) // 4 * 4
        self.nbuf = nbuf
        self.floats = 2 * (self.n4 + self.m4) + 64  # flags: `world` words in the last 64
        self.buf = torch.zeros(self.floats, dtype=torch.float32, device=device)
        self.imported = []
        handle = (ctypes.c_uint8 * 64)()
        off = ctypes.c_int64(0)
        with torch.cuda.device(device):
            call("sinkslot_ipc_export", ptr(self.buf), handle, ctypes.byref(off))
        mine = (bytes(handle), off.value)
        every = [None] * self.world
        dist.all_gather_object(every, mine, group=group)
        self.bases = []
        for g, (h, o) in enumerate(every):
            if g == self.rank:
                self.bases.append(self.buf.data_ptr())
                continue
            p = ctypes.c_void_p(0)
            hb = (ctypes.c_uint8 * 64).from_buffer_copy(h)
            with torch.cuda.device(device):
                call("sinkslot_ipc_import", hb, o, ctypes.byref(p))
            self.imported.append((p.value, o))
            self.bases.append(p.value)

    def pointers(self):
        """(phi[2*world], psi[2*world], flags[world]) pointer arrays."""
        W = self.world
        phi = (ctypes.c_void_p * (2 * W))()
        psi = (ctypes.c_void_p * (2 * W))()
        flags = (ctypes.c_void_p * W)()
        for g, b in enumerate(self.bases):
            for k in range(2):
                phi[2 * g + k] = b + 4 * k * self.n4 if k < self.nbuf else None
                psi[2 * g + k] = b + 4 * (2 * self.n4 + k * self.m4) if k < self.nbuf else None
            flags[g] = b + 4 * (2 * (self.n4 + self.m4))
        return phi, psi, flags

    def phi(self, k: int, n: int) -> torch.Tensor:
        return self.buf[k * self.n4:k * self.n4 + n]

    def psi(self, k: int, m: int) -> torch.Tensor:
        o = 2 * self.n4 + k * self.m4
        return self.buf[o:o + m]

    def close(self):
        for p, o in self.imported:
            call("sinkslot_ipc_close", p, o)
        self.imported = []


class ShardedSolver:
    """One rank's share of a partitioned solve, prepared once: the support (built
    on every rank), this rank's CSR rows / CSC columns and their tiled layouts,
    and the peer-mapped potential buffers.  ``solve`` runs a Sinkhorn loop from
    zero potentials; ``close`` unmaps the peers' buffers (collective)."""

    def __init__(self, X, Y, a, b, eps, L=64, seed=0, chunk=None, variant="alternating",
                 alpha=0.5, group=None, tiled: bool = True, support: str = "partitioned"):
        if not dist.is_initialized():
            raise RuntimeError("sharded solves need torch.distributed initialised")
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > MAX_RANKS:
            raise ValueError(f"at most {MAX_RANKS} ranks (one node), got {self.world}")
        dev = X.device
        self.dev = dev
        n, m = X.shape[0], Y.shape[0]
        self.n, self.m = n, m
        self.eps, self.alpha, self.variant = eps, alpha, variant
        self.log_a, self.log_b = a.log().contiguous(), b.log().contiguous()
        self.r0, self.nr = shard_bounds(n, self.world, self.rank)
        self.c0, self.nc = shard_bounds(m, self.world, self.rank)
        sizes = [None] * self.world
        dist.all_gather_object(sizes, (n, m, X.shape[1], L, seed), group=group)
        if any(s != sizes[0] for s in sizes):
            raise ValueError(f"ranks were given different problems {sizes}")
        if support == "partitioned":
            # each rank builds a range of the slices; the entries meet at their
            # row and column owners (build_partitioned_support)
            (rows, cols, S, lam), (c_cols, c_rows, c_lam) = build_partitioned_support(
                X, Y, a, b, eps, L, seed, chunk, group)
            # this rank's rows of the support (sorted by rows * m + cols)
            self.rows, self.cols, self.S = rows, cols, S
            p, i, v, _ = _to_csr(rows - self.r0, cols, lam, self.nr, want_perm=False)
            self.row = (p, i, v, int(i.numel()))
            p, i, v, _ = _to_csr(c_cols - self.c0, c_rows, c_lam, self.nc, want_perm=False)
            self.col = (p, i, v, int(i.numel()))
            del rows, cols, S, lam, c_cols, c_rows, c_lam
        elif support == "replicated":
            # every rank builds the whole support and keeps its slices
            self.rows, self.cols, self.S = sot_plan_coo(X, Y, a, b, L=L, seed=seed, chunk=chunk)
            lam, _ = cost_and_lam(X, Y, self.rows, self.cols, self.S, eps)
            r_ptr, r_idx, r_lam, _ = _to_csr(self.rows, self.cols, lam, n, want_perm=False)
            c_ptr, c_idx, c_lam, _ = _to_csr(self.cols, self.rows, lam, m, want_perm=False)
            self.row = slice_csr(r_ptr, r_idx, r_lam, self.r0, self.nr)
            self.col = slice_csr(c_ptr, c_idx, c_lam, self.c0, self.nc)
            del r_ptr, r_idx, r_lam, c_ptr, c_idx, c_lam, lam
        else:
            raise ValueError(f"support must be 'partitioned' or 'replicated', got {support!r}")
        self.support = support
        t = torch.tensor([self.row[3]], dtype=torch.int64, device=dev)
        dist.all_reduce(t, group=group)
        self.nnz = int(t.item())  # entries of the whole support
        self.r_tiles = build_tiles(self.row[0], self.row[1], self.row[2], self.nr, m) \
            if tiled and tiles_pay_off(self.nr, m, self.row[3]) else None
        self.c_tiles = build_tiles(self.col[0], self.col[1], self.col[2], self.nc, n) \
            if tiled and tiles_pay_off(self.nc, n, self.col[3]) else None
        self.vcode = 0 if variant == "alternating" else 1
        self.state = _SharedState(n, m, 1 + self.vcode, group, dev)
        self.ptrs = self.state.pointers()
        wf = _lib.out_i64()
        call("sinkslot_shard_work_floats", self.nr, self.nc, ctypes.byref(wf))
        self.work = torch.empty(wf.value, dtype=torch.float32, device=dev)
        self.epoch = ctypes.c_uint32(0)
        dist.barrier(group=group)  # every rank's buffer is zeroed and mapped

    def _run_chunk(self, cur: ctypes.c_int, it0: int, k: int, check: int):
        ch0, ch1 = ctypes.c_double(0.0), ctypes.c_double(0.0)
        if k <= 0:
            return 0.0, 0.0
        (lr_ptr, lr_idx, lr_lam, r_nnz), (lc_ptr, lc_idx, lc_lam, c_nnz) = self.row, self.col
        phi_p, psi_p, flag_p = self.ptrs
        with torch.cuda.device(self.dev):
            call("sinkslot_solve_shard", ptr(lr_ptr), ptr(lr_idx), _idx_bytes(lr_idx),
                 ptr(lr_lam), r_nnz, self.r0, self.nr, ptr(self.r_tiles),
                 self.r_tiles.numel() if self.r_tiles is not None else 0,
                 ptr(lc_ptr), ptr(lc_idx), _idx_bytes(lc_idx), ptr(lc_lam), c_nnz, self.c0,
                 self.nc, ptr(self.c_tiles),
                 self.c_tiles.numel() if self.c_tiles is not None else 0,
                 ptr(self.log_a), ptr(self.log_b), self.n, self.m, self.vcode,
                 float(self.alpha), self.rank, self.world, phi_p, psi_p, flag_p, it0, k, check,
                 ctypes.byref(cur), ctypes.byref(self.epoch), ptr(self.work), self.work.numel(),
                 ctypes.byref(ch0), ctypes.byref(ch1), stream_of(self.dev))
        return ch0.value, ch1.value

    def solve(self, n_iters=200, stop_mode="fixed", stop_max_iter=20000, stop_tol=1e-6,
              stop_check_every=5, copy_out: bool = True):
        """(phi, psi, iters_run, converged, final_viol) from zero potentials,
        with the stop semantics of the single-GPU loop.  All ranks call it."""
        mode = _resolve_stop_mode(None if stop_mode == "fixed" else SimpleNamespace(
            mode=stop_mode))
        if mode == "potential" and self.eps is None:
            raise ValueError("eps is required for stop.mode == 'potential'")
        for k in range(1 + self.vcode):
            self.state.phi(k, self.n).zero_()
            self.state.psi(k, self.m).zero_()
        cur = ctypes.c_int(0)
        # peers may write this rank's buffers only after every rank has reset its own
        dist.barrier(group=self.group)
        it, converged, viol = drive(
            lambda it0, k, check: self._run_chunk(cur, it0, k, check),
            _reduce_max_dist(self.group, self.dev), mode, int(n_iters), int(stop_max_iter),
            int(stop_check_every), float(stop_tol),
            float(self.eps) if self.eps is not None else 0.0, float(self.alpha), self.variant)
        phi = self.state.phi(cur.value, self.n)
        psi = self.state.psi(cur.value, self.m)
        if copy_out:
            phi, psi = phi.clone(), psi.clone()
        return phi, psi, it, converged, viol

    def close(self):
        # no rank may unmap or free a buffer a peer still writes
        torch.cuda.synchronize(self.dev)
        dist.barrier(group=self.group)
        self.state.close()
        dist.barrier(group=self.group)


def sinkslot_solve_sharded(X, Y, a=None, b=None, eps=0.05, L=64, seed=0, n_iters=200,
                           stop_mode="fixed", stop_max_iter=20000, stop_tol=1e-6,
                           stop_check_every=5, chunk=None, backend="auto",
                           variant="alternating", alpha=0.5, group=None,
                           tiled: bool = True, support: str = "partitioned",
                           gather_support: bool = True) -> SinkslotSolveResult:
    """``sinkslot_solve`` with the support build and the Sinkhorn loop
    partitioned over the ranks of ``group`` (default: the world), one GPU
    each.  Same arguments and result as ``sinkslot_solve``: every rank returns
    the full phi, psi and -- with ``gather_support`` (default) -- the full
    support; without it, the rows of the support it owns.  X, Y, a, b must be
    identical on every rank.  ``support="replicated"`` has every rank build the
    whole support instead of its share."""
    if not dist.is_initialized():
        raise RuntimeError("sinkslot_solve_sharded needs torch.distributed initialised")
    if a is None:
        a = torch.full((X.shape[0],), 1.0 / X.shape[0], device=X.device, dtype=X.dtype)
    if b is None:
        b = torch.full((Y.shape[0],), 1.0 / Y.shape[0], device=Y.device, dtype=Y.dtype)
    _validate(X, Y, a, b, backend, variant)
    stop = None if stop_mode == "fixed" else SimpleNamespace(
        mode=stop_mode, max_iter=stop_max_iter, tol=stop_tol, check_every=stop_check_every)
    mode = _resolve_stop_mode(stop)
    if mode == "potential" and eps is None:
        raise ValueError("eps is required for stop.mode == 'potential'")
    solver = ShardedSolver(X, Y, a, b, eps, L=L, seed=seed, chunk=chunk, variant=variant,
                           alpha=alpha, group=group, tiled=tiled, support=support)
    try:
        phi, psi, it, converged, viol = solver.solve(n_iters, mode, stop_max_iter, stop_tol,
                                                     stop_check_every)
    finally:
        solver.close()
    rows, cols, S = solver.rows, solver.cols, solver.S
    if gather_support and solver.support == "partitioned":
        rows, cols, S = (_gather_parts(t, group) for t in (rows, cols, S))
    return SinkslotSolveResult(phi, psi, rows, cols, S, it, converged, viol)


def _gather_parts(t: torch.Tensor, group) -> torch.Tensor:
    """The ranks' pieces of a 1-D tensor, concatenated in rank order, on every rank."""
    world = dist.get_world_size(group)
    n = torch.tensor([t.numel()], dtype=torch.int64, device=t.device)
    sizes = torch.empty(world, dtype=torch.int64, device=t.device)
    dist.all_gather_into_tensor(sizes, n, group=group)
    sizes = [int(v) for v in sizes.tolist()]
    cap = max(sizes) if sizes else 0
    buf = torch.zeros(cap, dtype=t.dtype, device=t.device)
    buf[:t.numel()] = t
    out = torch.empty(world * cap, dtype=t.dtype, device=t.device)
    dist.all_gather_into_tensor(out, buf, group=group)
    return torch.cat([out[g * cap:g * cap + sizes[g]] for g in range(world)])
