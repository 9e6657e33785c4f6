"""sinkslot_solve_csr_static (the solve loop on the library's static device
scratch) against sinkslot_solve_csr with a caller work buffer.

Each case runs the caller-buffer solve once and the static-scratch solve twice
in a row (the second call reuses the scratch the first left behind), through
the C ABI, and compares potentials at the parity bar (rtol 1e-4, atol 1e-5).
The file sorts last so the static scratch is also exercised after every other
test has used the device.
"""

from __future__ import annotations

import ctypes
from types import SimpleNamespace

import pytest
import torch

RTOL, ATOL = 1e-4, 1e-5
STATIC_FLOATS = 1 << 20  # SINKSLOT_STATIC_SOLVE_FLOATS in include/sinkslot_b200.h

_MODES = {"fixed": 0, "potential": 1, "marginal": 2}


def _problem(n, m, seed, cuda, L=32, eps=0.05):
    from sinkslot_b200.solver import cost_and_lam, sot_plan_coo, to_csr
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(n, 3, generator=g).to(cuda)
    y = (torch.randn(m, 3, generator=g) + 1.0).to(cuda)
    a = -torch.log(torch.rand(n, generator=g).clamp_min(1e-12))
    b = -torch.log(torch.rand(m, generator=g).clamp_min(1e-12))
    a, b = (a / a.sum()).to(cuda), (b / b.sum()).to(cuda)
    rows, cols, S = sot_plan_coo(x, y, a, b, L=L, seed=0)
    lam, _ = cost_and_lam(x, y, rows, cols, S, eps)
    r = to_csr(rows, cols, lam, n)
    c = to_csr(cols, rows, lam, m)
    return (r[0], r[1], r[2], c[0], c[1], c[2], a.log().contiguous(), b.log().contiguous(), n, m)


def _static_solve(csr, variant, mode, n_iters, max_iter, every, tol, eps, tiles):
    from sinkslot_b200 import _lib
    from sinkslot_b200._lib import ptr, stream_of
    r_ptr, r_idx, r_lam, c_ptr, c_idx, c_lam, la, lb, n, m = csr
    dev = la.device
    phi = torch.empty(n, dtype=torch.float32, device=dev)
    psi = torch.empty(m, dtype=torch.float32, device=dev)
    it, conv, viol = ctypes.c_int64(0), ctypes.c_int(0), ctypes.c_double(0.0)
    rt, ct = tiles if tiles is not None else (None, None)
    with torch.cuda.device(dev):
        _lib.call("sinkslot_solve_csr_static", ptr(r_ptr), ptr(r_idx), r_idx.element_size(),
                  ptr(r_lam), ptr(c_ptr), ptr(c_idx), c_idx.element_size(), ptr(c_lam),
                  r_idx.numel(), ptr(la), ptr(lb), n, m, variant, _MODES[mode], n_iters, max_iter,
                  every, tol, eps, 0.5, ptr(rt), rt.numel() if rt is not None else 0,
                  ptr(ct), ct.numel() if ct is not None else 0, ptr(phi), ptr(psi),
                  ctypes.byref(it), ctypes.byref(conv), ctypes.byref(viol), stream_of(dev))
    return phi, psi, int(it.value), int(conv.value)


CASES = [
    # n, m, variant, mode, tiled
    (3000, 2500, 0, "fixed", False),
    (3000, 2500, 1, "fixed", True),
    (4000, 3500, 0, "marginal", True),
    (2000, 2000, 1, "potential", False),
    (170000, 170000, 0, "fixed", True),  # scratch near its capacity
]


@pytest.mark.gpu
@pytest.mark.parametrize("n,m,variant,mode,tiled", CASES)
def test_static_scratch_solve_matches_work_buffer_solve(n, m, variant, mode, tiled):
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import sinkslot_b200
    from sinkslot_b200.sinkhorn_solvers import (build_tiles, sinkslot_alternating_b200,
                                                sinkslot_symmetric_b200)
    sinkslot_b200.load_library()
    cuda = torch.device("cuda:0")
    csr = _problem(n, m, 11, cuda)
    tiles = None
    if tiled:
        tiles = (build_tiles(csr[0], csr[1], csr[2], n, m), build_tiles(csr[3], csr[4], csr[5], m, n))
    n_iters, max_iter, every, tol, eps = 60, 4000, 5, 1e-6 if mode == "marginal" else 1e-5, 0.05
    stop = None if mode == "fixed" else SimpleNamespace(mode=mode, max_iter=max_iter, tol=tol,
                                                        check_every=every)
    fn = sinkslot_alternating_b200 if variant == 0 else sinkslot_symmetric_b200
    pw, qw, iw, cw, _ = fn(*csr, n_iters, stop, eps=eps, tiles=tiles)
    for call in range(2):
        ps, qs, it, conv = _static_solve(csr, variant, mode, n_iters, max_iter, every, tol, eps,
                                         tiles)
        torch.testing.assert_close(ps, pw, rtol=RTOL, atol=ATOL, msg=f"phi, static call {call}")
        torch.testing.assert_close(qs, qw, rtol=RTOL, atol=ATOL, msg=f"psi, static call {call}")
        if mode != "fixed":
            assert it == iw and bool(conv) == cw


def test_static_scratch_rejects_oversize_problem():
    """A problem whose scratch exceeds the static array is refused before any
    device work (status 1 -> ValueError naming the limit)."""
    from sinkslot_b200 import _lib
    from sinkslot_b200 import build
    build.build()
    wf = ctypes.c_int64(0)
    n = m = 1 << 20
    _lib.call("sinkslot_solve_work_floats", n, m, ctypes.byref(wf))
    assert wf.value > STATIC_FLOATS
    it, conv, viol = ctypes.c_int64(0), ctypes.c_int(0), ctypes.c_double(0.0)
    with pytest.raises(ValueError, match=f"at most {STATIC_FLOATS}"):
        _lib.call("sinkslot_solve_csr_static", None, None, 4, None, None, None, 4, None, 0, None,
                  None, n, m, 0, 0, 10, 0, 1, 0.0, 0.05, 0.5, None, 0, None, 0, None, None,
                  ctypes.byref(it), ctypes.byref(conv), ctypes.byref(viol), None)
