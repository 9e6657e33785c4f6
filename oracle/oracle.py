"""CPU parity oracle for the SinkSLOT sparse-Sinkhorn path -- TEST INFRASTRUCTURE.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference arm may import this module, and only as the checker or as the timed
CPU reference.  The product (``sinkslot_b200``) never calls it.

It wraps ``liboracle.so`` (``sinkslot_oracle.c``, a plain-C restatement of the
reference algorithm) with numpy arrays and mirrors the reference's functions:

=====================================  ========================================
oracle function                        reference (cai4cai/SinkSLOT, torch-ext/)
=====================================  ========================================
``get_random_projections``             ``sinkslot/solver.py:31-52``
``project``                            ``sinkslot/solver.py:221``
``ot1d``                               ``sinkslot/solver.py:55-150``
``sot_plan_coo``                       ``sinkslot/solver.py:153-232``
``to_csr``                             ``sinkslot/solver.py:235-276``
``sqeuclid_cost``                      ``sinkslot/solver.py:346``
``seg_lse_coo``                        ``sinkslot/sinkhorn_solvers.py:427-440``
``solve_loops``                        ``sinkslot/sinkhorn_solvers.py:443-588``
``sinkslot_solve``                     ``sinkslot/sinkhorn_solvers.py:591-722``
``plan_values``                        ``sinkslot/sinkhorn_solvers.py:755-758``
``barycentric_map`` / ``slot_grad``    ``sinkslot/gradient.py:25-99``
``samples_loss_value``                 ``sinkslot/samples_loss.py:69-74``
=====================================  ========================================

Support semantics (``builder``):

* ``"cuda"`` (default) -- the reference's CUDA builder on a CUDA device
  (``_ot_1d_coo_batched_cuda``, solver.py:107-150): stable sort with
  -0.0 == +0.0 (CUB radix sort), torch's CUDA innermost-dim scan order for the
  cumsum, slice-major emission, and ``S * (1/L)`` (torch divides a CUDA tensor
  by a CPU scalar through its reciprocal).
* ``"cuda_on_cpu"`` -- the same builder executed by torch's CPU ops:
  double-accumulated cumsum, slice-major emission, ``S / L``.
* ``"cpu"`` -- the naive builder ``_ot_1d_coo_batched`` (solver.py:55-104) on
  CPU tensors: double-accumulated cumsum, position-major emission, ``S / L``.

Torch's CPU argsort is not stable, so on exact ties in a projection the two
CPU presets can pair tied points differently from the reference's CPU run;
the stable order is the one the reference's CUDA run produces.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from typing import NamedTuple, Optional

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

_f32p = ctypes.POINTER(ctypes.c_float)
_i64p = ctypes.POINTER(ctypes.c_int64)
_i32p = ctypes.POINTER(ctypes.c_int32)


def build(force: bool = False) -> str:
    """Compile liboracle.so with the committed Makefile (gcc, OpenMP)."""
    if force or not os.path.exists(_LIB_PATH) or (
            os.path.getmtime(_LIB_PATH) < os.path.getmtime(os.path.join(_HERE, "sinkslot_oracle.c"))):
        subprocess.run(["make", "-s", "-C", _HERE, "liboracle.so"], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        L.orc_project.argtypes = [_f32p, ctypes.c_int64, ctypes.c_int, _f32p, ctypes.c_int, _f32p]
        L.orc_stable_argsort_f32.argtypes = [_f32p, ctypes.c_int64, _i32p]
        L.orc_cumsum.argtypes = [_f32p, ctypes.c_int64, ctypes.c_int, ctypes.c_int, _f32p]
        L.orc_torch_inner_scan_log_tx.argtypes = [ctypes.c_uint32, ctypes.c_uint32]
        L.orc_torch_inner_scan_log_tx.restype = ctypes.c_uint32
        L.orc_ot1d.argtypes = [_f32p, _f32p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int,
                               _f32p, _f32p, ctypes.c_int, ctypes.c_int, _i64p, _i64p, _f32p,
                               ctypes.c_int]
        L.orc_ot1d.restype = ctypes.c_int64
        L.orc_coalesce.argtypes = [_i64p, _i64p, _f32p, ctypes.c_int64, ctypes.c_int64,
                                   ctypes.c_int, ctypes.c_int, _i64p, _i64p, _f32p]
        L.orc_coalesce.restype = ctypes.c_int64
        L.orc_sqeuclid_cost.argtypes = [_f32p, _f32p, ctypes.c_int, _i64p, _i64p,
                                        ctypes.c_int64, _f32p]
        L.orc_lam.argtypes = [_f32p, _f32p, ctypes.c_int64, ctypes.c_double, _f32p]
        L.orc_seg_lse_coo.argtypes = [_i64p, _i64p, _f32p, ctypes.c_int64, _f32p, _f32p,
                                      ctypes.c_int64, _f32p]
        L.orc_solve.argtypes = [_i64p, _i64p, _f32p, ctypes.c_int64, _f32p, _f32p,
                                ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                                ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_double,
                                ctypes.c_double, ctypes.c_double, _f32p, _f32p,
                                ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_double)]
        L.orc_solve.restype = ctypes.c_int64
        L.orc_plan_values.argtypes = [_f32p, _f32p, _i64p, _i64p, _f32p, _f32p, ctypes.c_int64,
                                      ctypes.c_double, ctypes.c_int, _f32p]
        L.orc_barycentric.argtypes = [_f32p, _i64p, _i64p, ctypes.c_int64, _f32p, _f32p,
                                      ctypes.c_int64, ctypes.c_int64, ctypes.c_int, _f32p,
                                      _f32p, _f32p]
        L.orc_barycentric_cols.argtypes = [_f32p, _i64p, _i64p, ctypes.c_int64, _f32p,
                                           ctypes.c_int64, ctypes.c_int, _f32p]
        L.orc_num_threads.restype = ctypes.c_int
        L.orc_layout_new.argtypes = [_i64p, _i64p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64]
        L.orc_layout_new.restype = ctypes.c_void_p
        L.orc_layout_free.argtypes = [ctypes.c_void_p]
        L.orc_iterate_alternating.argtypes = [ctypes.c_void_p, _i64p, _i64p, _f32p, _f32p, _f32p,
                                              ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                              _f32p, _f32p]
        _lib = L
    return _lib


def _p(a: np.ndarray, ctype):
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data_as(ctypes.POINTER(ctype))


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def _i64(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.int64))


def num_threads() -> int:
    return int(lib().orc_num_threads())


# --------------------------------------------------------------------------
# support construction
# --------------------------------------------------------------------------

def get_random_projections(d: int, L: int, seed: int) -> np.ndarray:
    """solver.py:31-52.  The directions are defined by torch's CPU generator
    (``manual_seed(seed)``, ``randn((L, d), float64)``, row-normalised with
    ``clamp_min(1e-300)``); the same torch CPU ops are called here."""
    import torch
    gen = torch.Generator(device="cpu").manual_seed(seed)
    th = torch.randn((L, d), generator=gen, dtype=torch.float64)
    th = th / th.norm(dim=1, keepdim=True).clamp_min(1e-300)
    return th.numpy()


def project(X, theta) -> np.ndarray:
    """(L, n) projections, solver.py:221 transposed to the slice-major layout."""
    X = _f32(X)
    theta = _f32(theta)
    n, d = X.shape
    L = theta.shape[0]
    out = np.empty((L, n), dtype=np.float32)
    lib().orc_project(_p(X, ctypes.c_float), n, d, _p(theta, ctypes.c_float), L,
                      _p(out, ctypes.c_float))
    return out


def stable_argsort(v) -> np.ndarray:
    v = _f32(v)
    out = np.empty(v.shape[0], dtype=np.int32)
    lib().orc_stable_argsort_f32(_p(v, ctypes.c_float), v.shape[0], _p(out, ctypes.c_int32))
    return out


def cumsum(w, C: int, mode: str = "cuda") -> np.ndarray:
    """One slice's cumsum in torch's association order; ``C`` is the number of
    slices the reference scans in the same call (it sets torch's block shape)."""
    w = _f32(w)
    out = np.empty_like(w)
    lib().orc_cumsum(_p(w, ctypes.c_float), w.shape[0], C, 0 if mode == "cuda" else 1,
                     _p(out, ctypes.c_float))
    return out


# builder -> (cumsum order: 0 torch CUDA / 1 torch CPU, emission: 0 slice-major /
# 1 position-major, final division: 1 reciprocal multiply / 0 true division)
_BUILDERS = {"cuda": (0, 0, 1), "cuda_on_cpu": (1, 0, 0), "cpu": (1, 1, 0)}


def ot1d(PXt, PYt, a, b, builder: str = "cuda", scan_rows: int = 0):
    """Kept (R, C, mass) triples of C slices (solver.py:55-150).  PXt (C, n),
    PYt (C, m) slice-major projections.  scan_rows (0: C): the cumsum
    association of a batch of that many slices."""
    PXt, PYt, a, b = _f32(PXt), _f32(PYt), _f32(a), _f32(b)
    C, n = PXt.shape
    m = PYt.shape[1]
    cap = C * (n + m)
    R = np.empty(cap, dtype=np.int64)
    Cc = np.empty(cap, dtype=np.int64)
    M = np.empty(cap, dtype=np.float32)
    cum_mode, emit, _ = _BUILDERS[builder]
    cnt = lib().orc_ot1d(_p(PXt, ctypes.c_float), _p(PYt, ctypes.c_float), n, m, C,
                         _p(a, ctypes.c_float), _p(b, ctypes.c_float), cum_mode, emit,
                         _p(R, ctypes.c_int64), _p(Cc, ctypes.c_int64), _p(M, ctypes.c_float),
                         int(scan_rows))
    return R[:cnt], Cc[:cnt], M[:cnt]


def coalesce(R, Cc, v, m: int, L: int, builder: str = "cuda"):
    R, Cc, v = _i64(R), _i64(Cc), _f32(v)
    nraw = R.shape[0]
    rows = np.empty(max(nraw, 1), dtype=np.int64)
    cols = np.empty(max(nraw, 1), dtype=np.int64)
    S = np.empty(max(nraw, 1), dtype=np.float32)
    nu = lib().orc_coalesce(_p(R, ctypes.c_int64), _p(Cc, ctypes.c_int64), _p(v, ctypes.c_float),
                            nraw, m, L, _BUILDERS[builder][2], _p(rows, ctypes.c_int64),
                            _p(cols, ctypes.c_int64), _p(S, ctypes.c_float))
    return rows[:nu].copy(), cols[:nu].copy(), S[:nu].copy()


def sot_plan_coo(X, Y, a, b, L: int, seed: int, chunk: Optional[int] = None,
                 builder: str = "cuda", theta: Optional[np.ndarray] = None):
    """solver.py:153-232: (rows int64, cols int64, S float32), sorted by r*m+c."""
    X, Y, a, b = _f32(X), _f32(Y), _f32(a), _f32(b)
    n, d = X.shape
    m = Y.shape[0]
    if theta is None:
        theta = get_random_projections(d, L, seed)
    th = _f32(theta)
    chunk = L if chunk is None else chunk
    Rs, Cs, Vs = [], [], []
    for start in range(0, L, chunk):
        t = th[start:start + chunk]
        PXt, PYt = project(X, t), project(Y, t)
        r, c, v = ot1d(PXt, PYt, a, b, builder=builder)
        Rs.append(r); Cs.append(c); Vs.append(v)
    R = np.concatenate(Rs) if Rs else np.zeros(0, np.int64)
    Cc = np.concatenate(Cs) if Cs else np.zeros(0, np.int64)
    V = np.concatenate(Vs) if Vs else np.zeros(0, np.float32)
    return coalesce(R, Cc, V, m, L, builder=builder)


def to_csr(rows, cols, vals, n: int):
    """solver.py:235-276 (stable sort by ``rows``): (indptr int32, idx, vals, perm).
    ``idx`` is int16 when its maximum is below 2**15, else int32."""
    rows = _i64(rows)
    cols = _i64(cols)
    vals = np.asarray(vals)
    if rows.size == 0 or np.all(rows[1:] >= rows[:-1]):
        perm = None
        r = rows
    else:
        perm = np.argsort(rows, kind="stable")
        r = rows[perm]
    counts = np.bincount(r, minlength=n)
    indptr = np.zeros(n + 1, dtype=np.int32)
    indptr[1:] = np.cumsum(counts)
    idx = cols if perm is None else cols[perm]
    mx = int(idx.max()) if idx.size else 0
    idx = idx.astype(np.int16 if mx < 2 ** 15 else np.int32)
    return indptr, idx, (vals if perm is None else vals[perm]), perm


# --------------------------------------------------------------------------
# cost, lam, Sinkhorn
# --------------------------------------------------------------------------

def sqeuclid_cost(x, y, rows, cols) -> np.ndarray:
    x, y, rows, cols = _f32(x), _f32(y), _i64(rows), _i64(cols)
    out = np.empty(rows.shape[0], dtype=np.float32)
    lib().orc_sqeuclid_cost(_p(x, ctypes.c_float), _p(y, ctypes.c_float), x.shape[1],
                            _p(rows, ctypes.c_int64), _p(cols, ctypes.c_int64), rows.shape[0],
                            _p(out, ctypes.c_float))
    return out


def lam_values(S, cost, eps: float) -> np.ndarray:
    S, cost = _f32(S), _f32(cost)
    out = np.empty_like(S)
    lib().orc_lam(_p(S, ctypes.c_float), _p(cost, ctypes.c_float), S.shape[0], float(eps),
                  _p(out, ctypes.c_float))
    return out


def seg_lse_coo(idx_self, idx_other, lam, other, base, nseg: int) -> np.ndarray:
    """out[s] = base[s] - LSE_{k: idx_self[k]==s}(lam[k] + other[idx_other[k]])."""
    idx_self, idx_other = _i64(idx_self), _i64(idx_other)
    lam, other, base = _f32(lam), _f32(other), _f32(base)
    out = np.empty(nseg, dtype=np.float32)
    lib().orc_seg_lse_coo(_p(idx_self, ctypes.c_int64), _p(idx_other, ctypes.c_int64),
                          _p(lam, ctypes.c_float), lam.shape[0], _p(other, ctypes.c_float),
                          _p(base, ctypes.c_float), nseg, _p(out, ctypes.c_float))
    return out


_MODES = {"fixed": 0, "potential": 1, "marginal": 2}


def solve_loops(rows, cols, lam, log_a, log_b, n: int, m: int, n_iters: int,
                variant: str = "alternating", stop_mode: str = "fixed",
                stop_max_iter: int = 20000, stop_tol: float = 1e-6,
                stop_check_every: int = 5, eps: Optional[float] = None, alpha: float = 0.5):
    """sinkhorn_solvers.py:443-588: (phi, psi, iters_run, converged, final_viol)."""
    if stop_mode not in _MODES:
        raise ValueError(f"unknown stop.mode {stop_mode!r}; expected one of "
                         f"'fixed', 'marginal', 'potential'")
    if stop_mode == "potential" and eps is None:
        raise ValueError("eps is required for stop.mode == 'potential'")
    rows, cols, lam = _i64(rows), _i64(cols), _f32(lam)
    log_a, log_b = _f32(log_a), _f32(log_b)
    phi = np.empty(n, dtype=np.float32)
    psi = np.empty(m, dtype=np.float32)
    conv = ctypes.c_int(0)
    viol = ctypes.c_double(0.0)
    it = lib().orc_solve(_p(rows, ctypes.c_int64), _p(cols, ctypes.c_int64),
                         _p(lam, ctypes.c_float), rows.shape[0], _p(log_a, ctypes.c_float),
                         _p(log_b, ctypes.c_float), n, m, 0 if variant == "alternating" else 1,
                         _MODES[stop_mode], n_iters, stop_max_iter, stop_check_every,
                         float(stop_tol), float(eps if eps is not None else 0.0), float(alpha),
                         _p(phi, ctypes.c_float), _p(psi, ctypes.c_float), ctypes.byref(conv),
                         ctypes.byref(viol))
    if stop_mode == "fixed":
        return phi, psi, int(it), None, None
    return phi, psi, int(it), bool(conv.value), float(viol.value)


class IterationTimer:
    """Alternating fixed-mode iterations over a prebuilt layout (the CPU
    baseline's timed unit: one iteration = row + column half-step)."""

    def __init__(self, rows, cols, lam, log_a, log_b, n: int, m: int):
        self.rows, self.cols = _i64(rows), _i64(cols)
        self.lam = _f32(lam)
        self.log_a, self.log_b = _f32(log_a), _f32(log_b)
        self.n, self.m = n, m
        self.phi = np.zeros(n, dtype=np.float32)
        self.psi = np.zeros(m, dtype=np.float32)
        self.h = lib().orc_layout_new(_p(self.rows, ctypes.c_int64), _p(self.cols, ctypes.c_int64),
                                      self.rows.shape[0], n, m)

    def run(self, iters: int):
        lib().orc_iterate_alternating(self.h, _p(self.rows, ctypes.c_int64),
                                      _p(self.cols, ctypes.c_int64), _p(self.lam, ctypes.c_float),
                                      _p(self.log_a, ctypes.c_float), _p(self.log_b, ctypes.c_float),
                                      self.n, self.m, iters, _p(self.phi, ctypes.c_float),
                                      _p(self.psi, ctypes.c_float))

    def close(self):
        if self.h:
            lib().orc_layout_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class OracleSolveResult(NamedTuple):
    phi: np.ndarray
    psi: np.ndarray
    rows: np.ndarray
    cols: np.ndarray
    S: np.ndarray
    iters_run: Optional[int]
    converged: Optional[bool]
    final_viol: Optional[float]


def sinkslot_solve(X, Y, a=None, b=None, eps=0.05, L=64, seed=0, n_iters=200,
                   stop_mode="fixed", stop_max_iter=20000, stop_tol=1e-6, stop_check_every=5,
                   chunk=None, variant="alternating", alpha=0.5, builder="cuda"):
    """sinkhorn_solvers.py:591-722 with backend='torch' semantics."""
    X, Y = _f32(X), _f32(Y)
    n, m = X.shape[0], Y.shape[0]
    a = np.full(n, np.float32(1.0 / n), np.float32) if a is None else _f32(a)
    b = np.full(m, np.float32(1.0 / m), np.float32) if b is None else _f32(b)
    rows, cols, S = sot_plan_coo(X, Y, a, b, L, seed, chunk=chunk, builder=builder)
    cost = sqeuclid_cost(X, Y, rows, cols)
    lam = lam_values(S, cost, eps)
    log_a = np.log(a).astype(np.float32)
    log_b = np.log(b).astype(np.float32)
    phi, psi, it, conv, viol = solve_loops(rows, cols, lam, log_a, log_b, n, m, n_iters, variant,
                                           stop_mode, stop_max_iter, stop_tol, stop_check_every,
                                           eps, alpha)
    return OracleSolveResult(phi, psi, rows, cols, S, it, conv, viol)


def plan_values(phi, psi, rows, cols, S, cost, eps: float, grad_form: bool = False):
    phi, psi, S, cost = _f32(phi), _f32(psi), _f32(S), _f32(cost)
    rows, cols = _i64(rows), _i64(cols)
    out = np.empty(rows.shape[0], dtype=np.float32)
    lib().orc_plan_values(_p(phi, ctypes.c_float), _p(psi, ctypes.c_float),
                          _p(rows, ctypes.c_int64), _p(cols, ctypes.c_int64),
                          _p(S, ctypes.c_float), _p(cost, ctypes.c_float), rows.shape[0],
                          float(eps), 1 if grad_form else 0, _p(out, ctypes.c_float))
    return out


def barycentric_map(T, rows, cols, x, y):
    """gradient.py:25-61: (Tx, Ty)."""
    T, x, y = _f32(T), _f32(x), _f32(y)
    rows, cols = _i64(rows), _i64(cols)
    n, d = x.shape
    m = y.shape[0]
    Tx = np.empty((n, d), dtype=np.float32)
    Ty = np.empty((m, d), dtype=np.float32)
    dummy = np.zeros(n, dtype=np.float32)
    lib().orc_barycentric(_p(T, ctypes.c_float), _p(rows, ctypes.c_int64),
                          _p(cols, ctypes.c_int64), rows.shape[0], _p(x, ctypes.c_float),
                          _p(y, ctypes.c_float), n, m, d, _p(dummy, ctypes.c_float),
                          _p(Tx, ctypes.c_float), None)
    lib().orc_barycentric_cols(_p(T, ctypes.c_float), _p(rows, ctypes.c_int64),
                               _p(cols, ctypes.c_int64), rows.shape[0], _p(x, ctypes.c_float),
                               m, d, _p(Ty, ctypes.c_float))
    return Tx, Ty


def grad_from_plan(T, rows, cols, x, y, a):
    """gradient.py:97-99 / samples_loss.py:81-82: 2 * a * (x - Tx)."""
    T, x, y, a = _f32(T), _f32(x), _f32(y), _f32(a)
    rows, cols = _i64(rows), _i64(cols)
    n, d = x.shape
    Tx = np.empty((n, d), dtype=np.float32)
    g = np.empty((n, d), dtype=np.float32)
    lib().orc_barycentric(_p(T, ctypes.c_float), _p(rows, ctypes.c_int64),
                          _p(cols, ctypes.c_int64), rows.shape[0], _p(x, ctypes.c_float),
                          _p(y, ctypes.c_float), n, y.shape[0], d, _p(a, ctypes.c_float),
                          _p(Tx, ctypes.c_float), _p(g, ctypes.c_float))
    return g


def slot_grad(X, Y, a, b, eps, L, seed, n_iters, builder="cuda"):
    """gradient.py:65-99."""
    res = sinkslot_solve(X, Y, a, b, eps, L, seed, n_iters, builder=builder)
    cost = sqeuclid_cost(X, Y, res.rows, res.cols)
    T = plan_values(res.phi, res.psi, res.rows, res.cols, res.S, cost, eps, grad_form=True)
    return grad_from_plan(T, res.rows, res.cols, X, Y, a)


def samples_loss_value(phi, psi, a, b, eps: float) -> float:
    """samples_loss.py:74: eps * ((phi * a).sum() + (psi * b).sum()), fp32 sums."""
    pa = (_f32(phi) * _f32(a)).astype(np.float32)
    pb = (_f32(psi) * _f32(b)).astype(np.float32)
    return float(np.float32(eps) * np.float32(pa.sum(dtype=np.float64) + pb.sum(dtype=np.float64)))


def minres(matvec, b, tol: float = 1e-11, max_iter: int = 8000):
    """MINRES (Paige & Saunders, 1975) for a symmetric operator, float64: the
    recurrence the device solver restates (Lanczos vectors, Givens rotations of
    the tridiagonal, direction vectors; |eta| is the residual norm).  Returns
    (x, iterations, relative residual).  Stops when |eta| <= tol * ||b||."""
    b = np.asarray(b, dtype=np.float64)
    beta1 = float(np.linalg.norm(b))
    x = np.zeros_like(b)
    if beta1 == 0.0:
        return x, 0, 0.0
    v_prev = np.zeros_like(b)
    v = b / beta1
    w1 = np.zeros_like(b)  # w_{k-1}
    w2 = np.zeros_like(b)  # w_{k-2}
    beta, c1, s1, c2, s2, eta = beta1, 1.0, 0.0, 1.0, 0.0, beta1
    k = 0
    while k < max_iter:
        k += 1
        p = matvec(v) - beta * v_prev
        alpha = float(v @ p)
        p = p - alpha * v
        beta_next = float(np.linalg.norm(p))
        eps_k = s2 * beta
        dbar = c2 * beta
        delta = c1 * dbar + s1 * alpha
        gbar = -s1 * dbar + c1 * alpha
        gamma = float(np.hypot(gbar, beta_next))
        if gamma == 0.0:
            break
        c, s = gbar / gamma, beta_next / gamma
        w = (v - eps_k * w2 - delta * w1) / gamma
        x = x + c * eta * w
        eta = -s * eta
        w2, w1 = w1, w
        c2, s2, c1, s1 = c1, s1, c, s
        if beta_next == 0.0 or abs(eta) <= tol * beta1:
            break
        v_prev, v, beta = v, p / beta_next, beta_next
    return x, k, abs(eta) / beta1


def hvp_system(X, Y, a, v, rows, cols, T, eps: float, tau2: float = 3e-7):
    """The linear system of hvp.py:84-104 (float64): (M dense, rhs, dlam)."""
    X = np.asarray(X, np.float64); Y = np.asarray(Y, np.float64)
    a = np.asarray(a, np.float64); v = np.asarray(v, np.float64)
    T = np.asarray(T, np.float64); rows = _i64(rows); cols = _i64(cols)
    n, m = X.shape[0], Y.shape[0]
    dlam = -(2.0 / eps) * ((X[rows] - Y[cols]) * v[rows]).sum(1)
    rhs = np.zeros(n + m)
    np.add.at(rhs, rows, -(T * dlam))
    np.add.at(rhs, n + cols, -(T * dlam))
    M = np.zeros((n + m, n + m))
    M[np.arange(n), np.arange(n)] = a + tau2
    M[n + np.arange(m), n + np.arange(m)] = a[:m] + tau2  # the reference: a for both blocks
    np.add.at(M, (rows, n + cols), T)
    np.add.at(M, (n + cols, rows), T)
    return M, rhs, dlam


def hvp_x_sqeuclid_from_potentials(X, Y, a, v, rows, cols, T, eps: float, tau2: float = 3e-7,
                                   solver: str = "dense"):
    """hvp.py:34-113 in float64 with the linear system solved exactly
    (``solver="dense"``: the point MINRES converges to) or by :func:`minres`.
    Small problems only (dense (n+m)^2 matrix)."""
    M, rhs, dlam = hvp_system(X, Y, a, v, rows, cols, T, eps, tau2)
    if solver == "dense":
        sol = np.linalg.solve(M, rhs)
    else:
        sol, _, _ = minres(lambda z: M @ z, rhs)
    X = np.asarray(X, np.float64); Y = np.asarray(Y, np.float64)
    a = np.asarray(a, np.float64); v = np.asarray(v, np.float64)
    rows = _i64(rows); cols = _i64(cols)
    n = X.shape[0]
    u, w = sol[:n], sol[n:]
    weight = np.asarray(T, np.float64) * (u[rows] + w[cols] + dlam)
    dT = np.zeros_like(X)
    np.add.at(dT, rows, weight[:, None] * Y[cols])
    return 2.0 * a[:, None] * v - 2.0 * dT
