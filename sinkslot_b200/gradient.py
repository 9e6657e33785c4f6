"""Envelope-theorem gradient and barycentric map (host side).

Mirrors ``sinkslot/gradient.py`` of the reference: ``sparse_barycentric_map``
(two call forms) and ``slot_grad``.  The plan values, the per-row sums and the
gradient ``2 a (X - T_eps(X))`` run in libsinkslot_b200.so.
"""

from __future__ import annotations

import ctypes

import torch
from beartype import beartype
from jaxtyping import Float, jaxtyped

from . import _lib
from ._lib import call, ptr, stream_of
from .sinkhorn_solvers import plan_values, sinkslot_solve


def _bary(T_vals, rows, cols, x, y, a=None, want_tx=True, want_ty=True, want_grad=False):
    Tx, Ty, g = torch.ops.sinkslot_b200.barycentric(T_vals, rows, cols, x, y, a, bool(want_tx),
                                                     bool(want_ty), bool(want_grad))
    return (Tx if want_tx else None), (Ty if want_ty else None), (g if want_grad else None)


def _bary_impl(T_vals, rows, cols, x, y, a, want_tx, want_ty, want_grad):
    """The body of the ``sinkslot_b200::barycentric`` operator."""
    dev = x.device
    n, d = x.shape
    m = y.shape[0]
    x, y = x.contiguous(), y.contiguous()
    T_vals = T_vals.contiguous()
    rows = rows.to(torch.int64).contiguous()
    cols = cols.to(torch.int64).contiguous()
    if T_vals.dtype != torch.float32 or x.dtype != torch.float32 or y.dtype != torch.float32:
        raise ValueError("sparse_barycentric_map: sinkslot_b200 is float32-only")
    nb = _lib.out_i64()
    call("sinkslot_barycentric_workspace_bytes", rows.numel(), n, m, d, ctypes.byref(nb))
    ws = torch.empty(max(nb.value, 1), dtype=torch.uint8, device=dev)
    Tx = torch.empty((n, d), dtype=torch.float32, device=dev) if want_tx else None
    Ty = torch.empty((m, d), dtype=torch.float32, device=dev) if want_ty else None
    g = torch.empty((n, d), dtype=torch.float32, device=dev) if want_grad else None
    if a is not None:
        a = a.contiguous()
    with torch.cuda.device(dev):
        call("sinkslot_barycentric", ptr(T_vals), ptr(rows), ptr(cols), rows.numel(), ptr(x),
             ptr(y), n, m, d, ptr(a), ptr(Tx), ptr(Ty), ptr(g), ptr(ws), ws.numel(),
             stream_of(dev))
    return Tx, Ty, g


def sparse_barycentric_map(*args):
    """Barycentric projections (Tx, Ty) of a sparse plan
    (reference: gradient.py:25-61).

    ``sparse_barycentric_map(P, x, y)`` with ``P`` a sparse COO tensor, or
    ``sparse_barycentric_map(T_vals, rows, cols, x, y)``.  Normalised by the
    plan's own achieved marginals (clamped at the float32 tiny).
    """
    if len(args) == 3:
        P, x, y = args
        rows, cols = P.indices()
        T_vals = P.values()
    elif len(args) == 5:
        T_vals, rows, cols, x, y = args
    else:
        raise TypeError(
            f"sparse_barycentric_map expects (P, x, y) or "
            f"(T_vals, rows, cols, x, y), got {len(args)} positional args"
        )
    if not x.is_cuda:
        raise ValueError("sparse_barycentric_map: sinkslot_b200 runs on CUDA tensors only")
    Tx, Ty, _ = _bary(T_vals, rows, cols, x, y)
    return Tx, Ty


def grad_from_plan(T_vals, rows, cols, X, Y, a) -> torch.Tensor:
    """``2 * a[:, None] * (X - Tx)`` fused with the row sums of the barycentric
    map (gradient.py:97-99, samples_loss.py:81-82)."""
    _, _, g = _bary(T_vals, rows, cols, X, Y, a=a, want_tx=False, want_ty=False, want_grad=True)
    return g


@jaxtyped(typechecker=beartype)
def slot_grad(
    X: Float[torch.Tensor, "n d"], Y: Float[torch.Tensor, "m d"],
    a: Float[torch.Tensor, "n"], b: Float[torch.Tensor, "m"],
    eps: float, L: int, seed: int, n_iters: int, backend: str = "auto",
) -> Float[torch.Tensor, "n d"]:
    """grad_X SLOT_eps(X, Y) = 2 diag(a) (X - T_eps(X)) by the envelope theorem
    (reference: gradient.py:64-99)."""
    phi, psi, rows, cols, S, _, _, _ = sinkslot_solve(
        X, Y, a, b, eps, L, seed, n_iters, backend=backend)
    T_vals = plan_values(phi, psi, rows, cols, S, X, Y, eps, grad_form=True)
    return grad_from_plan(T_vals, rows, cols, X, Y, a)
