"""The shared-memory-staged (tiled) half-step against the exact kernel.

The tiled pass stabilises each row's log-sum-exp by its previous value and sums
in fixed point (2^-32 units, exact); rows outside the safe window go to the exact
kernel.
Checks: the layout holds exactly the CSR's entries, tile by tile; tiled and
exact solves agree to the parity bar on several problems (uniform and
Dirichlet weights, n != m, tiny and large eps so rows are handed back); tiled
solves are bit-reproducible.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-4, 1e-5


@pytest.fixture(scope="module")
def cuda():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import sinkslot_b200
    sinkslot_b200.load_library()
    return torch.device("cuda:0")


def _problem(n, m, d, seed, kind, cuda, L=32, eps=0.05, shift=1.0):
    from sinkslot_b200.solver import cost_and_lam, sot_plan_coo, to_csr
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(n, d, generator=g).to(cuda)
    y = (torch.randn(m, d, generator=g) + shift).to(cuda)
    if kind == "uniform":
        a = torch.full((n,), 1.0 / n, device=cuda)
        b = torch.full((m,), 1.0 / m, device=cuda)
    else:
        a = -torch.log(torch.rand(n, generator=g).clamp_min(1e-12))
        b = -torch.log(torch.rand(m, generator=g).clamp_min(1e-12))
        a, b = (a / a.sum()).to(cuda), (b / b.sum()).to(cuda)
    rows, cols, S = sot_plan_coo(x, y, a, b, L=L, seed=0)
    lam, _ = cost_and_lam(x, y, rows, cols, S, eps)
    r = to_csr(rows, cols, lam, n)
    c = to_csr(cols, rows, lam, m)
    return (r[0], r[1], r[2], c[0], c[1], c[2], a.log(), b.log(), n, m)


def _geometry(nseg, m_o, nnz):
    from sinkslot_b200 import _lib
    geom = (ctypes.c_int * 5)()
    _lib.call("sinkslot_tiles_geometry", nseg, m_o, nnz, geom)
    return list(geom)


def _align(x, a=256):
    return (x + a - 1) // a * a


def _column_bank_positions(p, tile, rb, cls, tile_len, place_max=9216):
    """Sorted positions after the column-bank placement inside each row-bank run.

    p: position of each entry in its tile's row-bank order; tile, rb, cls: its
    tile, row bank and column class (column mod 32), all in that order.  In a run
    [S, S + c), the k-th entry of class t (in run order) goes to relative position
    ((t - S) mod 32) + 32 k when below c; the others fill the free positions by
    class, then rank.  Tiles of more than place_max entries keep their order.
    """
    n = p.size
    if n == 0:
        return p
    run = tile.astype(np.int64) * 32 + rb
    start = np.r_[True, run[1:] != run[:-1]]
    run_id = np.cumsum(start) - 1
    S = p[start][run_id]
    nrun = int(run_id[-1]) + 1
    # rank of each entry among its run's entries of the same class, in run order
    o2 = np.lexsort((p, cls, run_id))
    g = run_id[o2] * 32 + cls[o2]
    gstart = np.r_[True, g[1:] != g[:-1]]
    first = np.maximum.accumulate(np.where(gstart, np.arange(n), 0))
    k = np.empty(n, dtype=np.int64)
    k[o2] = np.arange(n) - first
    e_all = np.bincount(run_id * 32 + cls, minlength=nrun * 32).reshape(nrun, 32)
    S_run = p[start]
    c_run = np.bincount(run_id)
    off_all = (np.arange(32)[None, :] - S_run[:, None]) % 32
    p_all = np.where(c_run[:, None] > off_all, (c_run[:, None] - 1 - off_all) // 32 + 1, 0)
    m_all = np.minimum(e_all, p_all)
    h_all, o_all = p_all - m_all, e_all - m_all
    pre_h = np.concatenate([np.zeros((nrun, 1), np.int64), np.cumsum(h_all, 1)], 1)
    pre_o = np.concatenate([np.zeros((nrun, 1), np.int64), np.cumsum(o_all, 1)], 1)
    off = (cls - S) % 32
    pc = p_all[run_id, cls]
    jn = off + 32 * k
    left = np.nonzero(k >= pc)[0]
    if left.size:
        rl = run_id[left]
        L = pre_o[rl, cls[left]] + (k[left] - pc[left])
        u = (pre_h[rl, 1:32] <= L[:, None]).sum(1)  # the largest class u with pre_h[u] <= L
        kk = e_all[rl, u] + (L - pre_h[rl, u])
        jn[left] = (u - S[left]) % 32 + 32 * kk
    out = S + jn
    keep = tile_len > place_max
    out[keep] = p[keep]
    return out


@pytest.mark.parametrize("n,m,L", [(3000, 2000, 16), (70000, 50000, 8), (300, 250, 40),
                                   (2000, 6_500_000, 2),   # 397 blocks: the sort-based builder
                                   (14800, 10000, 64)])    # tiles of ~12800: row-bank order kept
def test_layout_holds_the_csr_tile_by_tile(cuda, n, m, L):
    from sinkslot_b200.sinkhorn_solvers import build_tiles
    csr = _problem(n, m, 3, 1, "dirichlet", cuda, L=L)
    ptr, idx, lam = csr[0], csr[1], csr[2]
    nnz = idx.numel()
    layout = build_tiles(ptr, idx, lam, n, m).cpu().numpy()
    P, R, B, logW, smem = _geometry(n, m, nnz)
    assert smem <= 227 * 1024 and R < 16384 and logW <= 14 and P * R >= n and B << logW >= m
    T = P * B
    cap = nnz + 63 * T
    off = _align(64)
    tstart = layout[off:off + 8 * (T + 1)].view(np.int64)
    off = _align(off + 8 * (T + 1))
    ent = layout[off:off + 8 * cap].view(np.uint32).reshape(cap, 2)
    meta = ent[:, 0]
    tlam = ent[:, 1].copy().view(np.float32)
    ptr_h = ptr.cpu().numpy().astype(np.int64)
    idx_h = idx.cpu().numpy().astype(np.int64)
    lam_h = lam.cpu().numpy()
    row_of = np.repeat(np.arange(n), np.diff(ptr_h))
    tile_of = (row_of // R) * B + (idx_h >> logW)
    # inside a tile: stably by the bank of the row state, (row within panel) mod 32
    rb_all = (row_of % R) % 32
    order = np.lexsort((np.arange(nnz), rb_all, tile_of))
    counts = np.bincount(tile_of, minlength=T)
    slabs = (counts + 31) // 32
    slabs += (slabs > 0) & (slabs % 2 == 0)  # an odd number of slabs
    padded = slabs * 32
    np.testing.assert_array_equal(tstart, np.concatenate([[0], np.cumsum(padded)]))
    # meta = (row within panel) * 4 << 16 | (column within block) * 4 (byte
    # offsets into the kernel's shared-memory arrays); padding: the dummy row R,
    # column 0, lam = -inf
    want_meta = np.full(cap, R << 18, dtype=np.uint64)
    want_lam = np.full(cap, -np.inf, dtype=np.float32)
    ustart = np.concatenate([[0], np.cumsum(counts)])
    t_o = tile_of[order]
    p = np.arange(nnz) - ustart[t_o]
    p = _column_bank_positions(p, t_o, rb_all[order], idx_h[order] & 31, padded[t_o])
    ns = padded[t_o] // 32
    # sorted position p of a tile with N slabs: slab p mod N, lane p // N
    pos = tstart[t_o] + 32 * (p % ns) + p // ns
    want_meta[pos] = ((row_of[order] % R) << 18) | ((idx_h[order] & ((1 << logW) - 1)) << 2)
    want_lam[pos] = lam_h[order]
    np.testing.assert_array_equal(meta, want_meta.astype(np.uint32))
    np.testing.assert_array_equal(tlam, want_lam)


CASES = [
    (4000, 4000, 3, "uniform", 0.05, 64),
    (5000, 3000, 3, "dirichlet", 0.05, 32),
    (60000, 60000, 3, "uniform", 0.01, 64),
    (20000, 30000, 2, "dirichlet", 0.002, 48),   # small eps: rows handed back
    (3000, 3000, 4, "dirichlet", 2.0, 16),       # large eps
    (100, 50000, 2, "dirichlet", 0.05, 16),      # rows of > 4096 entries: handed back whole
]


@pytest.mark.parametrize("n,m,d,kind,eps,L", CASES)
@pytest.mark.parametrize("variant", ["alternating", "symmetric"])
def test_tiled_matches_exact_fixed(cuda, n, m, d, kind, eps, L, variant):
    from sinkslot_b200.sinkhorn_solvers import (build_tiles, sinkslot_alternating_b200,
                                                sinkslot_symmetric_b200)
    csr = _problem(n, m, d, 7, kind, cuda, L=L, eps=eps)
    tiles = (build_tiles(csr[0], csr[1], csr[2], n, m), build_tiles(csr[3], csr[4], csr[5], m, n))
    fn = sinkslot_alternating_b200 if variant == "alternating" else sinkslot_symmetric_b200
    pe, qe, *_ = fn(*csr, 150)
    pt, qt, *_ = fn(*csr, 150, tiles=tiles)
    pt2, qt2, *_ = fn(*csr, 150, tiles=tiles)
    assert torch.equal(pt, pt2) and torch.equal(qt, qt2), "tiled solve is not reproducible"
    # Both are fp32 with different summation orders; after 150 iterations their
    # difference near zero is the fp32 resolution of the potentials' scale
    # (|phi| reaches ~10^3 at eps = 0.01), so atol is scaled by max|phi|.
    atol_p = ATOL + 2e-7 * float(pe.abs().max())
    atol_q = ATOL + 2e-7 * float(qe.abs().max())
    torch.testing.assert_close(pt, pe, rtol=RTOL, atol=atol_p)
    torch.testing.assert_close(qt, qe, rtol=RTOL, atol=atol_q)


@pytest.mark.parametrize("mode,tol", [("marginal", 1e-6), ("potential", 1e-5)])
@pytest.mark.parametrize("variant", ["alternating", "symmetric"])
def test_tiled_matches_exact_stop_modes(cuda, mode, tol, variant):
    from types import SimpleNamespace
    from sinkslot_b200.sinkhorn_solvers import (build_tiles, sinkslot_alternating_b200,
                                                sinkslot_symmetric_b200)
    n, m = 3000, 2500
    csr = _problem(n, m, 3, 9, "dirichlet", cuda, L=40)
    tiles = (build_tiles(csr[0], csr[1], csr[2], n, m), build_tiles(csr[3], csr[4], csr[5], m, n))
    stop = SimpleNamespace(mode=mode, max_iter=20000, tol=tol, check_every=5)
    fn = sinkslot_alternating_b200 if variant == "alternating" else sinkslot_symmetric_b200
    pe, qe, ie, ce, ve = fn(*csr, 0, stop, eps=0.05)
    pt, qt, it, ct, vt = fn(*csr, 0, stop, eps=0.05, tiles=tiles)
    assert ce and ct and abs(ie - it) <= 5
    c = float((pt - pe).double().mean())
    torch.testing.assert_close(pt - c, pe, rtol=0, atol=5e-3)
    torch.testing.assert_close(qt + c, qe, rtol=0, atol=5e-3)


@pytest.mark.parametrize("sides", ["row", "col"])
@pytest.mark.parametrize("variant", ["alternating", "symmetric"])
def test_one_side_tiled_matches_exact(cuda, sides, variant):
    """One side tiled, the other exact (the choice large gathered axes make):
    the handed-back row counters of the tiled side are reset every half-step."""
    from sinkslot_b200.sinkhorn_solvers import (build_tiles, sinkslot_alternating_b200,
                                                sinkslot_symmetric_b200)
    n, m = 20000, 30000
    csr = _problem(n, m, 2, 7, "dirichlet", cuda, L=48, eps=0.002)  # rows are handed back
    rt = build_tiles(csr[0], csr[1], csr[2], n, m) if sides == "row" else None
    ct = build_tiles(csr[3], csr[4], csr[5], m, n) if sides == "col" else None
    fn = sinkslot_alternating_b200 if variant == "alternating" else sinkslot_symmetric_b200
    pe, qe, *_ = fn(*csr, 150)
    pt, qt, *_ = fn(*csr, 150, tiles=(rt, ct))
    atol_p = ATOL + 2e-7 * float(pe.abs().max())
    atol_q = ATOL + 2e-7 * float(qe.abs().max())
    torch.testing.assert_close(pt, pe, rtol=RTOL, atol=atol_p)
    torch.testing.assert_close(qt, qe, rtol=RTOL, atol=atol_q)


@pytest.mark.parametrize("iters", [1, 2, 3])
@pytest.mark.parametrize("variant", ["alternating", "symmetric"])
@pytest.mark.parametrize("kind,eps", [("uniform", 0.01), ("dirichlet", 0.002)])
def test_first_iterations_tiled_match_exact(cuda, iters, variant, kind, eps):
    """The first iteration has no previous log-sum-exp to stabilise by: its row
    half-step (both half-steps, symmetric) gathers the zero start potential and
    runs the exact kernel without the gather -- the same bits as gathering
    zeros --, and the alternating first column half-step takes its stabilisers
    from a tiled max pass.  Both paths are fp32 with different summation
    orders, so near zero the bar's atol is scaled by max|phi| as in the other
    tiled-vs-exact comparisons."""
    from sinkslot_b200.sinkhorn_solvers import (build_tiles, sinkslot_alternating_b200,
                                                sinkslot_symmetric_b200)
    n, m = 60000, 50000
    csr = _problem(n, m, 3, 11, kind, cuda, L=64, eps=eps)
    tiles = (build_tiles(csr[0], csr[1], csr[2], n, m), build_tiles(csr[3], csr[4], csr[5], m, n))
    fn = sinkslot_alternating_b200 if variant == "alternating" else sinkslot_symmetric_b200
    pe, qe, *_ = fn(*csr, iters)
    pt, qt, *_ = fn(*csr, iters, tiles=tiles)
    if iters == 1:
        # exact kernel on both paths, with and without the gather of zeros
        assert torch.equal(pt, pe)
        if variant == "symmetric":
            assert torch.equal(qt, qe)
    torch.testing.assert_close(pt, pe, rtol=RTOL, atol=ATOL + 2e-7 * float(pe.abs().max()))
    torch.testing.assert_close(qt, qe, rtol=RTOL, atol=ATOL + 2e-7 * float(qe.abs().max()))
