"""Hessian-vector product by implicit differentiation of the Sinkhorn fixed point.

Mirrors ``sinkslot/hvp.py`` of the reference (``hvp_x_sqeuclid``,
``hvp_x_sqeuclid_from_potentials``): the same arguments, defaults and result.
The reference solves its (n+m) x (n+m) sparse system with torchsparsegradutils'
MINRES; here the whole computation -- the right-hand side, MINRES on the
device over the plan's CSR and CSC, and the final contraction -- runs in
libsinkslot_b200.so (``sinkslot_hvp``).
"""

from __future__ import annotations

import ctypes
from typing import NamedTuple

import torch
from beartype import beartype
from jaxtyping import Float, jaxtyped

from . import _lib
from ._lib import call, ptr, stream_of
from .sinkhorn_solvers import _idx_bytes, _validate, plan_values, sinkslot_solve
from .solver import _to_csr


class HvpInfo(NamedTuple):
    """How the linear solve ended: MINRES iterations run and the final
    residual relative to the right-hand side's norm."""
    iters: int
    rel_residual: float


def hvp_x_sqeuclid_from_potentials(X, Y, a, v, rows, cols, T_vals, eps, *, tau2=3e-7,
                                   solve_tol=1e-11, max_cg_iter=8000,
                                   return_info: bool = False):
    """H(X) @ v given a solved sparse plan (rows, cols, T_vals) on a frozen
    support (reference: hvp.py:34-113).

    Solves [[diag(a + tau2), P], [P^T, diag(a + tau2)]] [u; w] = rhs by MINRES
    (at most ``max_cg_iter`` iterations, stopping once the residual is below
    ``solve_tol`` times the right-hand side's norm), then returns
    2 a v - 2 sum_j T_ij (u_i + w_j + dlam_ij) y_j.  As in the reference, ``a``
    weights both blocks, so X and Y must have the same number of points.
    With ``return_info`` also returns an :class:`HvpInfo`.
    """
    n, d = X.shape
    m = Y.shape[0]
    if m != n:
        raise ValueError(f"hvp_x_sqeuclid uses a as both marginals: X and Y must have the same "
                         f"number of points, got {n} and {m}")
    for name, t in (("X", X), ("Y", Y), ("a", a), ("v", v), ("T_vals", T_vals)):
        if not t.is_cuda or t.dtype != torch.float32:
            raise ValueError(f"hvp: {name} must be a float32 CUDA tensor (got {t.dtype} on "
                             f"{t.device}); sinkslot_b200 has no CPU path")
    out, info = torch.ops.sinkslot_b200.hvp_from_potentials(
        X, Y, a, v, rows, cols, T_vals, float(eps), float(tau2), float(solve_tol),
        int(max_cg_iter))
    if return_info:
        it, res = info.tolist()
        return out, HvpInfo(int(it), float(res))
    return out


def _hvp_impl(X, Y, a, v, rows, cols, T_vals, eps, tau2, solve_tol, max_cg_iter):
    """The body of the ``sinkslot_b200::hvp_from_potentials`` operator:
    (H v, iterations, relative residual)."""
    n, d = X.shape
    m = Y.shape[0]
    dev = X.device
    X, Y, a, v = X.contiguous(), Y.contiguous(), a.contiguous(), v.contiguous()
    rows = rows.to(torch.int64).contiguous()
    cols = cols.to(torch.int64).contiguous()
    r_ptr, r_idx, r_T, _ = _to_csr(rows, cols, T_vals.contiguous(), n, want_perm=False)
    c_ptr, c_idx, c_T, _ = _to_csr(cols, rows, T_vals.contiguous(), m, want_perm=False)
    if r_idx.dtype != c_idx.dtype:  # one index width for both sides
        r_idx, c_idx = r_idx.to(torch.int32), c_idx.to(torch.int32)
    wb = _lib.out_i64()
    call("sinkslot_hvp_workspace_bytes", n, m, ctypes.byref(wb))
    ws = torch.empty(max(wb.value, 1), dtype=torch.uint8, device=dev)
    out = torch.empty((n, d), dtype=torch.float32, device=dev)
    iters = ctypes.c_int64(0)
    resid = ctypes.c_double(0.0)
    with torch.cuda.device(dev):
        call("sinkslot_hvp", ptr(X), ptr(Y), d, ptr(v), ptr(a), ptr(a), ptr(r_ptr), ptr(r_idx),
             ptr(r_T), ptr(c_ptr), ptr(c_idx), ptr(c_T), _idx_bytes(r_idx), n, m, float(eps),
             float(tau2), float(solve_tol), int(max_cg_iter), ptr(ws), ws.numel(), ptr(out), None,
             ctypes.byref(iters), ctypes.byref(resid), stream_of(dev))
    return out, int(iters.value), float(resid.value)


@jaxtyped(typechecker=beartype)
def hvp_x_sqeuclid(X: Float[torch.Tensor, "n d"], Y: Float[torch.Tensor, "m d"],
                   a: Float[torch.Tensor, "n"], eps, L, seed, n_iters,
                   v: Float[torch.Tensor, "n d"], tau2=3e-7, solve_tol=1e-11,
                   max_cg_iter=8000, backend="auto"):
    """End-to-end H(X) @ v of grad_X SLOT_eps (reference: hvp.py:116-206): the
    sliced support of (X, Y) with ``a`` as both marginals, ``n_iters``
    alternating iterations, the plan, then
    :func:`hvp_x_sqeuclid_from_potentials`.  ``backend`` as for
    ``sinkslot_solve``."""
    _validate(X, Y, a, a, backend, "alternating")
    r = sinkslot_solve(X, Y, a, a, eps, L, seed, n_iters, backend=backend)
    T_vals = plan_values(r.phi, r.psi, r.rows, r.cols, r.S, X, Y, eps, grad_form=True)
    return hvp_x_sqeuclid_from_potentials(X, Y, a, v, r.rows, r.cols, T_vals, eps, tau2=tau2,
                                          solve_tol=solve_tol, max_cg_iter=max_cg_iter)
