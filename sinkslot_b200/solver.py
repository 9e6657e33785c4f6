"""Sliced-OT support construction, COO -> CSR and the sparse cost (host side).

Mirrors ``sinkslot/solver.py`` of the reference (cai4cai/SinkSLOT, torch-ext/):
same names, arguments, return values and errors.  Every computation runs in
libsinkslot_b200.so; PyTorch only allocates device memory and supplies the
current stream.

Parity notes (the support is integer work and is bit-exact against the
reference's CUDA builder, ``_ot_1d_coo_batched_cuda``):

* projections are the sequential fp32 FMA chain over ``d`` (cuBLAS's result
  for these K = d; for d > 4 cuBLAS's own product is used);
* the per-slice argsort is stable with -0.0 == +0.0 (CUB radix sort);
* ``cumsum(a[ix])`` follows torch's CUDA innermost-dim scan association order;
* duplicate entries are summed in emission order and scaled by ``1/L`` (torch's
  division of a CUDA tensor by a Python scalar).
"""

from __future__ import annotations

import ctypes

import torch
from beartype import beartype
from jaxtyping import Float, Int, jaxtyped

from . import _lib
from ._lib import call, ptr, stream_of


@jaxtyped(typechecker=beartype)
def get_random_projections(d: int, L: int, seed: int) -> Float[torch.Tensor, "L d"]:
    """L unit directions in R^d (reference: solver.py:31-52).

    The directions are defined by torch's CPU generator: ``manual_seed(seed)``,
    ``randn((L, d), float64)``, each row divided by its norm clamped at 1e-300.
    Those same CPU ops run here, so the directions are bit-identical to the
    reference's.  Returns float64; callers cast to the data dtype.
    """
    gen = torch.Generator(device="cpu").manual_seed(seed)
    thetas = torch.randn((L, d), generator=gen, dtype=torch.float64)
    return thetas / thetas.norm(dim=1, keepdim=True).clamp_min(1e-300)


def _require_cuda_f32(name: str, *ts: torch.Tensor) -> torch.device:
    dev = None
    for t in ts:
        if not t.is_cuda:
            raise ValueError(f"{name}: sinkslot_b200 runs on CUDA tensors only (got {t.device})")
        if t.dtype != torch.float32:
            raise ValueError(f"{name}: the sm_100a kernels are float32-only, got {t.dtype}")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"{name}: all tensors must be on one device")
    return dev


def _ws(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


def project(X: torch.Tensor, theta: torch.Tensor) -> torch.Tensor:
    """Slice-major projections (L, n) of X onto fp32 directions theta (L, d):
    ``(X @ theta.T).T`` of solver.py:221 as the sequential FMA chain."""
    dev = _require_cuda_f32("project", X, theta)
    X = X.contiguous()
    theta = theta.contiguous()
    n, d = X.shape
    L = theta.shape[0]
    out = torch.empty((L, n), dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        call("sinkslot_project", ptr(X), n, d, ptr(theta), L, ptr(out), stream_of(dev))
    return out


def _ot_1d_coo_batched_cuda(PX: torch.Tensor, PY: torch.Tensor, a: torch.Tensor,
                            b: torch.Tensor, return_intermediates: bool = False,
                            scan_rows: int = 0):
    """1-D optimal plans of C slices as flat COO (reference: solver.py:107-150).

    PX (n, C), PY (m, C).  Returns (rows, cols, vals) of the kept entries in the
    reference's emission order (slice-major).  With ``return_intermediates`` also
    returns (ix, iy, ca, cb) in the (C, len) layout.  ``scan_rows`` (0: C)
    selects the cumsum association of a batch of that many slices.
    """
    dev = _require_cuda_f32("_ot_1d_coo_batched_cuda", PX, PY, a, b)
    n, C = PX.shape
    m = PY.shape[0]
    PXt, PYt = PX.T.contiguous(), PY.T.contiguous()
    a, b = a.contiguous(), b.contiguous()
    nb = _lib.out_i64()
    call("sinkslot_ot1d_workspace_bytes", n, m, C, ctypes.byref(nb))
    ws = _ws(nb.value, dev)
    cap = C * (n + m)
    R = torch.empty(cap, dtype=torch.int64, device=dev)
    Cc = torch.empty(cap, dtype=torch.int64, device=dev)
    M = torch.empty(cap, dtype=torch.float32, device=dev)
    inter = None
    if return_intermediates:
        inter = (torch.empty((C, n), dtype=torch.int32, device=dev),
                 torch.empty((C, m), dtype=torch.int32, device=dev),
                 torch.empty((C, n), dtype=torch.float32, device=dev),
                 torch.empty((C, m), dtype=torch.float32, device=dev))
    cnt = _lib.out_i64()
    with torch.cuda.device(dev):
        call("sinkslot_ot1d_batched", ptr(PXt), ptr(PYt), ptr(a), ptr(b), n, m, C, int(scan_rows),
             ptr(ws),
             ws.numel(), ptr(R), ptr(Cc), ptr(M),
             *(ptr(t) for t in (inter if inter else (None,) * 4)), ctypes.byref(cnt),
             stream_of(dev))
    k = cnt.value
    out = (R[:k], Cc[:k], M[:k])
    if return_intermediates:
        return out + inter
    return out


ot_1d_coo_batched = _ot_1d_coo_batched_cuda


# widest d for which the support builder projects with its own kernel
OWN_PROJECTION_MAX_D = 4


@jaxtyped(typechecker=beartype)
def sot_plan_coo(
    X: Float[torch.Tensor, "n d"], Y: Float[torch.Tensor, "m d"],
    a: Float[torch.Tensor, "n"], b: Float[torch.Tensor, "m"],
    L: int, seed: int, chunk: int | None = None, ot1d=None,
) -> tuple[Int[torch.Tensor, "nnz"], Int[torch.Tensor, "nnz"], Float[torch.Tensor, "nnz"]]:
    """Unsmoothed sliced-OT plan as COO (rows, cols, S), nnz <= L(n+m)
    (reference: solver.py:153-232).

    Sorted by ``rows * m + cols``; rows/cols int64, S float32.  ``chunk`` slices
    are built per batch (all L by default).  ``ot1d`` is accepted for signature
    compatibility; only the CUDA builder's semantics exist here.
    """
    if ot1d is not None and ot1d is not _ot_1d_coo_batched_cuda:
        raise ValueError("sot_plan_coo: sinkslot_b200 builds the support with the CUDA "
                         "builder's semantics only (ot1d must be None)")
    _require_cuda_f32("sot_plan_coo", X, Y, a, b)
    if chunk is not None and int(chunk) < 1:
        raise ValueError("chunk must be a positive int")
    return torch.ops.sinkslot_b200.sot_plan_coo(X, Y, a, b, int(L), int(seed),
                                                None if chunk is None else int(chunk))


def _sot_plan_coo_impl(X, Y, a, b, L: int, seed: int, chunk):
    """The body of the ``sinkslot_b200::sot_plan_coo`` operator."""
    dev = X.device
    n, d = X.shape
    m = Y.shape[0]
    thetas = torch.as_tensor(get_random_projections(d, L, seed), dtype=X.dtype, device=dev)
    X, Y, a, b = X.contiguous(), Y.contiguous(), a.contiguous(), b.contiguous()
    ck = 0 if chunk is None else int(chunk)
    if chunk is not None and ck < 1:
        raise ValueError("chunk must be a positive int")
    # The sort keys are the reference's projections `X @ theta.T`, chunk by
    # chunk (solver.py:219-221).  For d <= OWN_PROJECTION_MAX_D the library
    # computes them itself, fused into the key generation, as the sequential
    # fp32 FMA chain over d -- bit-equal to cuBLAS's product at these d for every
    # workload shape (tested on the device) -- so no (n, L) projection matrix is
    # materialised.  Wider d: cuBLAS's rounding there can differ from the
    # chain, so the product is taken from cuBLAS itself.
    PX = PY = None
    if d > OWN_PROJECTION_MAX_D:
        step = L if chunk is None else ck
        if step >= L:
            PX, PY = X @ thetas.T, Y @ thetas.T
        else:
            PX = torch.cat([X @ thetas[s:s + step].T for s in range(0, L, step)], dim=1)
            PY = torch.cat([Y @ thetas[s:s + step].T for s in range(0, L, step)], dim=1)
        PX, PY = PX.contiguous(), PY.contiguous()
    nb = _lib.out_i64()
    call("sinkslot_support_workspace_bytes", n, m, d, L, ck, ctypes.byref(nb))
    ws = _ws(nb.value, dev)
    nnz = _lib.out_i64()
    s = stream_of(dev)
    with torch.cuda.device(dev):
        call("sinkslot_build_support", ptr(X), ptr(Y), ptr(a), ptr(b), n, m, d, ptr(thetas),
             ptr(PX), ptr(PY), L, ck, ptr(ws), ws.numel(), ctypes.byref(nnz), s)
        del PX, PY
        k = nnz.value
        rows = torch.empty(k, dtype=torch.int64, device=dev)
        cols = torch.empty(k, dtype=torch.int64, device=dev)
        S = torch.empty(k, dtype=torch.float32, device=dev)
        call("sinkslot_support_export", ptr(ws), ws.numel(), n, m, d, L, ck, k, ptr(rows),
             ptr(cols), ptr(S), s)
    return rows, cols, S


def max_index(v: torch.Tensor) -> int:
    """``int(v.max())`` for an int64 device vector (0 when empty)."""
    dev = v.device
    ws = torch.empty(8, dtype=torch.uint8, device=dev)
    out = _lib.out_i64()
    v = v.contiguous()
    with torch.cuda.device(dev):
        call("sinkslot_max_index", ptr(v), v.numel(), ptr(ws), ctypes.byref(out), stream_of(dev))
    return int(out.value)


def to_csr(rows: torch.Tensor, cols: torch.Tensor, vals: torch.Tensor, n: int,
           narrow_key: bool = False):
    """COO -> CSR: (indptr int32, idx, vals_permuted, perm) (reference: solver.py:235-276).

    Stable by ``rows``; when ``rows`` is already non-decreasing the permutation is
    the identity, ``perm`` is None and ``vals`` is returned as is.  ``idx`` is
    int16 when its maximum is below 2**15, else int32.  ``narrow_key`` is
    accepted for compatibility (the sort key is always 32-bit here).
    """
    return _to_csr(rows, cols, vals, n, want_perm=True)


def _to_csr(rows: torch.Tensor, cols: torch.Tensor, vals: torch.Tensor, n: int,
            want_perm: bool):
    """``to_csr``; without ``want_perm`` the permutation is not formed (None)
    and the sort carries the indices and values themselves."""
    if not rows.is_cuda:
        raise ValueError("to_csr: sinkslot_b200 runs on CUDA tensors only")
    dev = rows.device
    rows = rows.to(torch.int64).contiguous()
    cols = cols.to(torch.int64).contiguous()
    vals = vals.contiguous()
    if vals.dtype != torch.float32:
        raise ValueError(f"to_csr: vals must be float32, got {vals.dtype}")
    nnz = rows.numel()
    mx = max_index(cols) if nnz else 0
    idx_dtype = torch.int16 if mx < 2 ** 15 else torch.int32
    nb = _lib.out_i64()
    call("sinkslot_csr_workspace_bytes", nnz, n, ctypes.byref(nb))
    ws = _ws(nb.value, dev)
    indptr = torch.empty(n + 1, dtype=torch.int32, device=dev)
    idx = torch.empty(nnz, dtype=idx_dtype, device=dev)
    out_vals = torch.empty_like(vals)
    perm = torch.empty(nnz, dtype=torch.int64, device=dev) if want_perm else None
    was_sorted = ctypes.c_int(0)
    with torch.cuda.device(dev):
        call("sinkslot_coo_to_csr", ptr(rows), ptr(cols), ptr(vals), nnz, n,
             2 if idx_dtype == torch.int16 else 4, ptr(ws), ws.numel(), ptr(indptr), ptr(idx),
             ptr(out_vals), ptr(perm) if want_perm else None, ctypes.byref(was_sorted),
             stream_of(dev))
    if was_sorted.value:
        return indptr, idx, vals, None
    return indptr, idx, out_vals, perm


@jaxtyped(typechecker=beartype)
def sparse_sqeuclidean_cost(
    x: Float[torch.Tensor, "n d"], y: Float[torch.Tensor, "m d"],
    rows: Int[torch.Tensor, "nnz"], cols: Int[torch.Tensor, "nnz"],
    block: int = 1024, use_triton=None,
) -> Float[torch.Tensor, "nnz"]:
    """``||x[rows] - y[cols]||^2`` per support entry (reference: solver.py:302-360).

    Computed by the fused sm_100a kernel with each operation rounded as the
    reference's torch expression ``(x[rows]-y[cols]).square().sum(1)`` rounds it
    on the CPU (the d terms summed in index order).
    float32-only, like the reference's fused path; ``block`` and ``use_triton``
    are accepted for signature compatibility.
    """
    if x.dtype != torch.float32 or y.dtype != torch.float32:
        raise ValueError(
            f"sparse_sqeuclidean_cost's fused path is float32-only (fixed float32 "
            f"accumulator); got x.dtype={x.dtype}, y.dtype={y.dtype}. Cast to float32 first.")
    _require_cuda_f32("sparse_sqeuclidean_cost", x, y)
    return torch.ops.sinkslot_b200.sparse_sqeuclidean_cost(x, y, rows, cols)


def _sqeuclid_cost_impl(x, y, rows, cols):
    """The body of the ``sinkslot_b200::sparse_sqeuclidean_cost`` operator."""
    dev = x.device
    x, y = x.contiguous(), y.contiguous()
    rows = rows.to(torch.int64).contiguous()
    cols = cols.to(torch.int64).contiguous()
    nnz = rows.numel()
    out = torch.empty(nnz, dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        call("sinkslot_cost_lam", ptr(x), ptr(y), x.shape[1], ptr(rows), ptr(cols), None, nnz,
             1.0, None, ptr(out), stream_of(dev))
    return out


def cost_and_lam(x: torch.Tensor, y: torch.Tensor, rows: torch.Tensor, cols: torch.Tensor,
                 S: torch.Tensor, eps: float, want_cost: bool = False):
    """``lam = log(S.clamp_min(tiny)) - cost / eps`` in one fused pass
    (sinkhorn_solvers.py:699-700); returns (lam, cost or None)."""
    dev = _require_cuda_f32("cost_and_lam", x, y, S)
    x, y = x.contiguous(), y.contiguous()
    nnz = rows.numel()
    lam = torch.empty(nnz, dtype=torch.float32, device=dev)
    cost = torch.empty(nnz, dtype=torch.float32, device=dev) if want_cost else None
    with torch.cuda.device(dev):
        call("sinkslot_cost_lam", ptr(x), ptr(y), x.shape[1], ptr(rows), ptr(cols), ptr(S), nnz,
             float(eps), ptr(lam), ptr(cost), stream_of(dev))
    return lam, cost
