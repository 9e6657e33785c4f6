"""The reference's torch-op sequence for the support build and the torch-backend
Sinkhorn loop, runnable on whichever device the tensors live on -- TEST
INFRASTRUCTURE.

Only ``tests/`` may use this module, as a checker.  On a CUDA device these are
the same torch operations the reference executes on that device
(cai4cai/SinkSLOT, torch-ext/sinkslot/solver.py:107-150 and 194-232;
sinkhorn_solvers.py:427-588), so their outputs are the reference's CUDA
outputs bit for bit wherever the torch ops are deterministic (sort, scan,
searchsorted, gather).  The duplicate sum uses ``index_add_``, which is
order-nondeterministic on CUDA, so S from here is compared with a tolerance.
The sequence of operations has to be the reference's own to reproduce its
bits; it is restated here, not imported, so the tests run without the
reference tree.
"""

from __future__ import annotations

import torch


def ot1d_cuda_builder(PX: torch.Tensor, PY: torch.Tensor, a: torch.Tensor, b: torch.Tensor,
                      return_intermediates: bool = False):
    """Kept (R, C, mass) of C slices in the (C, len) layout; PX (n, C), PY (m, C)."""
    n, C = PX.shape
    m = PY.shape[0]
    dev = PX.device
    px_t, py_t = PX.T.contiguous(), PY.T.contiguous()
    ix = torch.argsort(px_t, dim=-1)
    iy = torch.argsort(py_t, dim=-1)
    ca = torch.cumsum(a[ix], dim=-1)
    cb = torch.cumsum(b[iy], dim=-1)
    rank_a = torch.arange(n, device=dev)[None, :] + torch.searchsorted(cb, ca, right=True)
    rank_b = torch.arange(m, device=dev)[None, :] + torch.searchsorted(ca, cb, right=False)
    merged = ca.new_empty(C, n + m)
    merged.scatter_(1, rank_a, ca)
    merged.scatter_(1, rank_b, cb)
    before = torch.cat([merged.new_zeros(C, 1), merged[:, :-1]], dim=1)
    mass = merged - before
    mid = 0.5 * (before + merged)
    i = torch.searchsorted(ca, mid).clamp_(max=n - 1)
    j = torch.searchsorted(cb, mid).clamp_(max=m - 1)
    R = torch.gather(ix, 1, i)
    Cc = torch.gather(iy, 1, j)
    sel = (mass > 0).reshape(-1).nonzero(as_tuple=False).squeeze(1)
    out = (R.reshape(-1)[sel], Cc.reshape(-1)[sel], mass.reshape(-1)[sel])
    if return_intermediates:
        return out + (ix, iy, ca, cb)
    return out


def sot_plan_coo(X, Y, a, b, theta: torch.Tensor, chunk=None):
    """rows, cols (int64), S: the reference's coalesce of all slices' entries."""
    n, d = X.shape
    m = Y.shape[0]
    L = theta.shape[0]
    key_dtype = torch.int32 if n * m < 2 ** 31 else torch.int64
    chunk = L if chunk is None else chunk
    keys, vals = [], []
    for s in range(0, L, chunk):
        th = theta[s:s + chunk]
        r, c, v = ot1d_cuda_builder(X @ th.T, Y @ th.T, a, b)
        keys.append((r * m + c).to(key_dtype))
        vals.append(v)
    f, v = torch.cat(keys), torch.cat(vals)
    uniq = torch.unique(f)
    inv = torch.searchsorted(uniq, f, out_int32=True)
    S = v.new_zeros(uniq.numel()).index_add_(0, inv, v)
    return (uniq // m).long(), (uniq % m).long(), S / L


def seg_lse_coo(vals: torch.Tensor, idx: torch.Tensor, size: int) -> torch.Tensor:
    mx = vals.new_full((size,), float("-inf")).scatter_reduce(
        0, idx, vals, reduce="amax", include_self=True)
    acc = vals.new_zeros(size).index_add_(0, idx, (vals - mx[idx]).exp())
    return torch.where(acc > 0, mx + acc.clamp_min(torch.finfo(vals.dtype).tiny).log(),
                       torch.full_like(mx, float("-inf")))


def alternating_fixed(rows, cols, lam, log_a, log_b, n, m, n_iters):
    phi, psi = torch.zeros_like(log_a), torch.zeros_like(log_b)
    for _ in range(n_iters):
        phi = log_a - seg_lse_coo(lam + psi[cols], rows, n)
        psi = log_b - seg_lse_coo(lam + phi[rows], cols, m)
    return phi, psi


def symmetric_fixed(rows, cols, lam, log_a, log_b, n, m, n_iters, alpha=0.5):
    phi, psi = torch.zeros_like(log_a), torch.zeros_like(log_b)
    for _ in range(n_iters):
        pc = log_a - seg_lse_coo(lam + psi[cols], rows, n)
        qc = log_b - seg_lse_coo(lam + phi[rows], cols, m)
        phi = (1.0 - alpha) * phi + alpha * pc
        psi = (1.0 - alpha) * psi + alpha * qc
    return phi, psi
