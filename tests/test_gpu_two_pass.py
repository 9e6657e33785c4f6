"""The two-pass kind of the tiled half-step against the staged kind.

The two-pass kind computes every term's exponent lam + potential in a first pass
(one CTA per column block, the block staged once) and sums each panel's terms in
a second pass with the staged kind's fixed-point arithmetic, cap and hand-back
rule.  The exponent is rounded the same way in both kinds (fp32 add, then the
stabiliser subtracted), and the fixed-point sums do not depend on order, so a
two-pass solve must give the staged solve's potentials bit for bit.
Checks: the layout (the staged layout, its geometry for the two-pass panels,
plus each slot's row offset, column offset and lam), bit equality with the staged kind in every variant
and stop mode and in the first iterations, the automatic choice on a large
gathered axis against the exact kernel, and a layout used under the other kind
fails with an error status.
"""

from __future__ import annotations

import ctypes
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from test_gpu_tiled import ATOL, RTOL, _align, _problem

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cuda():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import sinkslot_b200
    sinkslot_b200.load_library()
    return torch.device("cuda:0")


@pytest.fixture
def kinds(cuda):
    """Sets the process-wide tiled kind for a block of code; restores auto."""
    from sinkslot_b200.sinkhorn_solvers import set_tiles_kind
    yield set_tiles_kind
    set_tiles_kind("auto")


def _tiles(csr, n, m):
    from sinkslot_b200.sinkhorn_solvers import build_tiles
    return (build_tiles(csr[0], csr[1], csr[2], n, m), build_tiles(csr[3], csr[4], csr[5], m, n))


def _solve(csr, variant, iters, tiles, stop=None, eps=None):
    from sinkslot_b200.sinkhorn_solvers import sinkslot_alternating_b200, sinkslot_symmetric_b200
    fn = sinkslot_alternating_b200 if variant == "alternating" else sinkslot_symmetric_b200
    return fn(*csr, iters, stop, eps=eps, tiles=tiles)


def _both_kinds(kinds, csr, n, m, variant, iters, stop=None, eps=None):
    out = {}
    for kind in ("staged", "two_pass"):
        kinds(kind)
        tiles = _tiles(csr, n, m)
        out[kind] = _solve(csr, variant, iters, tiles, stop, eps)
        del tiles
    kinds("auto")
    return out["staged"], out["two_pass"]


@pytest.mark.parametrize("n,m,L", [(3000, 2000, 16), (70000, 50000, 8),
                                   (14800, 10000, 64), (300, 250, 40)])
def test_two_pass_layout(cuda, kinds, n, m, L):
    from sinkslot_b200 import _lib
    from sinkslot_b200.sinkhorn_solvers import build_tiles, tiles_kind_of
    csr = _problem(n, m, 3, 1, "dirichlet", cuda, L=L)
    ptr, idx, lam = csr[0], csr[1], csr[2]
    nnz = idx.numel()
    kinds("staged")
    staged = build_tiles(ptr, idx, lam, n, m).cpu().numpy()
    gs = (ctypes.c_int * 5)()
    _lib.call("sinkslot_tiles_geometry", n, m, nnz, gs)
    kinds("two_pass")
    assert tiles_kind_of(n, m, nnz) == "two_pass"
    layout = build_tiles(ptr, idx, lam, n, m).cpu().numpy()
    g2 = (ctypes.c_int * 5)()
    _lib.call("sinkslot_tiles_geometry", n, m, nnz, g2)
    P, R, B, logW, smem = list(g2)
    # panels of up to 16383 rows (no potential ring beside the row state)
    assert R < 16384 and R >= gs[1] and P * R >= n and (B, logW) == (gs[2], gs[3])
    assert smem <= 227 * 1024
    T = P * B
    cap = nnz + 63 * T
    header = layout[:64].view(np.int64)
    lens = np.diff(ptr.cpu().numpy())
    assert list(header[1:4]) == [2, P, B] and header[0] == lens[lens <= 4096].max()
    assert list(staged[:64].view(np.int64)[1:4]) == [1, gs[0], gs[2]]
    off = _align(64)
    tstart = layout[off:off + 8 * (T + 1)].view(np.int64)
    off = _align(off + 8 * (T + 1))
    ent = layout[off:off + 8 * cap].view(np.uint32).reshape(cap, 2)
    off = _align(off + 8 * cap)
    rowoff = layout[off:off + 2 * cap].view(np.uint16)
    off = _align(_align(off + 2 * cap) + 4 * cap)  # past the exponents
    coloff = layout[off:off + 2 * cap].view(np.uint16)
    off = _align(off + 2 * cap)
    lamv = layout[off:off + 4 * cap].view(np.uint32)
    # every slot split into what each pass reads, padding (the dummy row R,
    # column 0, lam = -inf) included
    np.testing.assert_array_equal(rowoff, (ent[:, 0] >> 16).astype(np.uint16))
    np.testing.assert_array_equal(coloff, (ent[:, 0] & 0xFFFF).astype(np.uint16))
    np.testing.assert_array_equal(lamv, ent[:, 1])
    # the same entries as the CSR, each in the tile of its (panel, block)
    ptr_h = ptr.cpu().numpy().astype(np.int64)
    idx_h = idx.cpu().numpy().astype(np.int64)
    row_of = np.repeat(np.arange(n), np.diff(ptr_h))
    tile_of = (row_of // R) * B + (idx_h >> logW)
    counts = np.bincount(tile_of, minlength=T)
    slabs = (counts + 31) // 32
    slabs += (slabs > 0) & (slabs % 2 == 0)
    np.testing.assert_array_equal(tstart, np.concatenate([[0], np.cumsum(slabs * 32)]))
    t_slot = np.repeat(np.arange(T), np.diff(tstart))
    real = ent[:tstart[-1], 0] >> 18 < R
    got_rows = (t_slot[real] // B) * R + (ent[:tstart[-1], 0][real] >> 18)
    got_cols = (t_slot[real] % B << logW) + ((ent[:tstart[-1], 0][real] & 0xFFFF) >> 2)
    got = np.lexsort((got_cols, got_rows))
    np.testing.assert_array_equal(got_rows[got], row_of)
    np.testing.assert_array_equal(got_cols[got], idx_h)
    np.testing.assert_array_equal(ent[:tstart[-1], 1][real][got].view(np.float32),
                                  lam.cpu().numpy())


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
def test_two_pass_equals_staged_fixed(cuda, kinds, n, m, d, kind, eps, L, variant):
    csr = _problem(n, m, d, 7, kind, cuda, L=L, eps=eps)
    (ps, qs, *_), (pt, qt, *_) = _both_kinds(kinds, csr, n, m, variant, 150)
    assert torch.equal(pt, ps) and torch.equal(qt, qs), \
        f"max |dphi| {float((pt - ps).abs().max())}, max |dpsi| {float((qt - qs).abs().max())}"


@pytest.mark.parametrize("iters", [1, 2, 3])
@pytest.mark.parametrize("variant", ["alternating", "symmetric"])
def test_two_pass_first_iterations(cuda, kinds, iters, variant):
    """The alternating first column half-step takes its stabilisers from a max
    pass; in the two-pass kind the sum pass reuses the max pass's exponents."""
    n, m = 60000, 50000
    csr = _problem(n, m, 3, 11, "dirichlet", cuda, L=64, eps=0.002)
    (ps, qs, *_), (pt, qt, *_) = _both_kinds(kinds, csr, n, m, variant, iters)
    assert torch.equal(pt, ps) and torch.equal(qt, qs)


@pytest.mark.parametrize("mode,tol", [("marginal", 1e-6), ("potential", 1e-5)])
@pytest.mark.parametrize("variant", ["alternating", "symmetric"])
def test_two_pass_equals_staged_stop_modes(cuda, kinds, mode, tol, variant):
    n, m = 3000, 2500
    csr = _problem(n, m, 3, 9, "dirichlet", cuda, L=40)
    stop = SimpleNamespace(mode=mode, max_iter=20000, tol=tol, check_every=5)
    s, t = _both_kinds(kinds, csr, n, m, variant, 0, stop, eps=0.05)
    assert torch.equal(t[0], s[0]) and torch.equal(t[1], s[1])
    assert t[2:] == s[2:]  # iterations run, converged, final violation


def test_two_pass_chosen_for_a_long_gathered_axis(cuda, kinds):
    """Auto policy: 2^16 rows gathering from 2^21 columns (L = 8) stage 148 x 8 MB
    per half-step, more than 4x the row side's entry stream -- the row side runs
    two passes, the column side (gathering 2^16) the staged kind; the solve
    agrees with the exact kernel to the tiled-vs-exact bar and with the staged
    kind bit for bit."""
    from sinkslot_b200.sinkhorn_solvers import tiles_kind_of
    n, m = 1 << 16, 1 << 21
    csr = _problem(n, m, 3, 5, "uniform", cuda, L=8, eps=0.05)
    nnz = csr[1].numel()
    kinds("auto")
    assert tiles_kind_of(n, m, nnz) == "two_pass"
    assert tiles_kind_of(m, n, nnz) == "staged"
    pa, qa, *_ = _solve(csr, "alternating", 100, _tiles(csr, n, m))
    pe, qe, *_ = _solve(csr, "alternating", 100, (None, None))
    torch.testing.assert_close(pa, pe, rtol=RTOL, atol=ATOL + 2e-7 * float(pe.abs().max()))
    torch.testing.assert_close(qa, qe, rtol=RTOL, atol=ATOL + 2e-7 * float(qe.abs().max()))
    kinds("staged")
    ps, qs, *_ = _solve(csr, "alternating", 100, _tiles(csr, n, m))
    assert torch.equal(pa, ps) and torch.equal(qa, qs)


def test_layout_of_the_other_kind_is_rejected(cuda, kinds):
    """A two-pass layout (the larger buffer) passed to a solve under the staged
    setting: every kernel reads the kind in the layout's header, does nothing
    and the call fails; a staged layout under the two-pass setting is too small
    and is refused before any launch.  The same context then solves normally."""
    from sinkslot_b200._lib import SinkslotError
    n, m = 4000, 4000
    csr = _problem(n, m, 3, 3, "uniform", cuda, L=32)
    kinds("two_pass")
    t2 = _tiles(csr, n, m)
    kinds("staged")
    with pytest.raises(SinkslotError, match="another kind"):
        _solve(csr, "alternating", 20, t2)
    t1 = _tiles(csr, n, m)
    kinds("two_pass")
    with pytest.raises(ValueError, match="too small"):
        _solve(csr, "alternating", 20, t1)
    kinds("staged")
    p1, q1, *_ = _solve(csr, "alternating", 20, t1)
    pe, qe, *_ = _solve(csr, "alternating", 20, (None, None))
    torch.testing.assert_close(p1, pe, rtol=RTOL, atol=ATOL + 2e-7 * float(pe.abs().max()))
