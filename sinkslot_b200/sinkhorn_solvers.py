"""Sinkhorn solve loops and the ``sinkslot_solve`` entry point (host side).

Mirrors ``sinkslot/sinkhorn_solvers.py`` of the reference: ``seg_lse_online``,
``launch_cfg``, ``SinkslotSolveResult``, the alternating / symmetric loops over
prebuilt CSR/CSC, ``sinkslot_solve`` and ``sparse_transport_plan``, with the
same arguments, validation messages and stop-mode semantics.  The loops run in
libsinkslot_b200.so: two fused segmented-LSE launches per iteration (the
symmetric blend and the stop-criterion reductions are fused into them) and one
host read-back per stop check.
"""

from __future__ import annotations

import ctypes
from types import SimpleNamespace
from typing import NamedTuple, Optional

import torch
from beartype import beartype
from jaxtyping import Float, jaxtyped

from . import _lib
from ._lib import call, ptr, stream_of
from .solver import _to_csr, cost_and_lam, sot_plan_coo, to_csr

BACKENDS = ("auto", "b200", "triton")


def launch_cfg(nnz: int, n: int) -> tuple[int, int]:
    """(BLOCK, num_warps) the reference's Triton kernel would use for a mean row
    length of nnz/n (reference: sinkhorn_solvers.py:97-118).  Kept for API
    compatibility; the sm_100a kernel sizes its lane groups itself."""
    mean_row = max(1, nnz // max(1, n))
    block = 1 << max(5, min(10, (mean_row - 1).bit_length()))
    return block, 2 if block <= 512 else 4


def _idx_bytes(t: torch.Tensor) -> int:
    if t.dtype == torch.int16:
        return 2
    if t.dtype == torch.int32:
        return 4
    raise ValueError(f"index arrays must be int16 or int32, got {t.dtype}")


def seg_lse_online(indptr, colidx, lam, phi, psi, n, block=None, num_warps=None,
                   base=None, out=None):
    """Segmented LSE over CSR: ``out[i] = base[i] - LSE_k(lam_k + phi_i + psi_{c_k})``
    (``LSE`` itself when ``base`` is None), written into ``out`` when given
    (reference: sinkhorn_solvers.py:121-146).  ``block``/``num_warps`` are
    accepted for compatibility."""
    if out is None:
        return torch.ops.sinkslot_b200.seg_lse(indptr, colidx, lam, phi, psi, int(n), base)
    _seg_lse_impl(indptr, colidx, lam, phi, psi, n, base, out)
    return out


def _seg_lse_impl(indptr, colidx, lam, phi, psi, n, base, out):
    dev = lam.device
    with torch.cuda.device(dev):
        call("sinkslot_seg_lse", ptr(indptr), ptr(colidx), _idx_bytes(colidx), ptr(lam),
             colidx.numel(), ptr(phi), ptr(psi), ptr(base), n, ptr(out), stream_of(dev))


class SinkslotSolveResult(NamedTuple):
    """``sinkslot_solve``'s return value (reference: sinkhorn_solvers.py:154-167)."""
    phi: torch.Tensor
    psi: torch.Tensor
    rows: torch.Tensor
    cols: torch.Tensor
    S: torch.Tensor
    iters_run: Optional[int]
    converged: Optional[bool]
    final_viol: Optional[float]


_STOP_MODES = ("fixed", "marginal", "potential")
_MODE_CODE = {"fixed": 0, "potential": 1, "marginal": 2}


def _resolve_stop_mode(stop):
    """``stop.mode`` (or "fixed" for None), validated (reference: :173-192)."""
    mode = getattr(stop, "mode", "fixed") if stop is not None else "fixed"
    if mode not in _STOP_MODES:
        raise ValueError(
            f"unknown stop.mode {mode!r}; expected one of "
            f"'fixed', 'marginal', 'potential'"
        )
    return mode


# Below this many entries a half-step is a few microseconds of memory traffic:
# the tiled kernels' fixed cost (a 1024-thread CTA per SM, barrier set-up, a
# second launch for handed-back rows) outweighs their gain (measured at N = 10^4,
# L = 64: 22.9 us per iteration tiled, 14.4 us exact).
TILE_MIN_NNZ = 1 << 22

# How a side with a tiled layout runs (libsinkslot_b200 picks per side, by
# sizes): "staged" stages every block of the gathered potential in shared
# memory once per panel (one pass; P * m_other * 4 bytes copied per
# half-step); "two_pass" first writes every entry's exponent lam + potential
# with one CTA per block, then sums each panel's entries without a gather (16
# bytes per entry, all streamed).  "auto" (the default) takes the staged kind
# while its staging costs at most 4x the entry stream, else the two-pass kind:
# large gathered axes (N = 2^24 on one GPU, row slices of a many-GPU partition)
# no longer fall back to the exact kernel's random gathers (about 36 bytes of
# HBM time per entry).
TILES_KINDS = {"auto": 0, "staged": 1, "two_pass": 2}


def set_tiles_kind(kind: str) -> None:
    """Process-wide choice of the tiled half-step's kind ("auto", "staged",
    "two_pass").  Layouts must be built and used under the same setting."""
    if kind not in TILES_KINDS:
        raise ValueError(f"tiles kind must be one of {tuple(TILES_KINDS)}, got {kind!r}")
    call("sinkslot_set_tiles_kind", TILES_KINDS[kind])


def get_tiles_kind() -> str:
    k = ctypes.c_int(0)
    call("sinkslot_get_tiles_kind", ctypes.byref(k))
    return {v: n for n, v in TILES_KINDS.items()}[k.value]


def tiles_kind_of(nseg: int, m_other: int, nnz: int) -> str:
    """The kind ("staged" or "two_pass") a layout of these sizes gets now."""
    k = ctypes.c_int(0)
    call("sinkslot_tiles_kind_of", nseg, m_other, nnz, ctypes.byref(k))
    return {1: "staged", 2: "two_pass"}[k.value]


def tiles_pay_off(nseg: int, m_other: int, nnz: int) -> bool:
    """Whether a side of nseg segments gathering from m_other potentials with
    nnz entries should run a tiled half-step (either kind) rather than the
    exact kernel (see TILE_MIN_NNZ)."""
    return nseg > 0 and m_other > 0 and nnz >= TILE_MIN_NNZ


def build_tiles(indptr, idx, lam, nseg: int, m_other: int) -> torch.Tensor:
    """Column-blocked layout of one CSR side (device bytes) for the half-step
    that stages the gathered potential in shared memory."""
    dev = lam.device
    nnz = idx.numel()
    lb, bb = _lib.out_i64(), _lib.out_i64()
    call("sinkslot_tiles_bytes", nseg, m_other, nnz, ctypes.byref(lb), ctypes.byref(bb))
    layout = torch.empty(max(lb.value, 1), dtype=torch.uint8, device=dev)
    ws = torch.empty(max(bb.value, 1), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        call("sinkslot_build_tiles", ptr(indptr), ptr(idx), _idx_bytes(idx), ptr(lam), nseg,
             m_other, nnz, ptr(layout), layout.numel(), ptr(ws), ws.numel(), stream_of(dev))
    return layout


def _solve_csr(r_ptr, r_idx, r_lam, c_ptr, c_idx, c_lam, log_a, log_b, n, m, n_iters, stop,
               eps, alpha, variant: int, tiles=None):
    mode = _resolve_stop_mode(stop)
    if mode == "potential" and eps is None:
        raise ValueError("eps is required for stop.mode == 'potential'")
    dev = log_a.device
    r_tiles, c_tiles = tiles if tiles is not None else (None, None)
    log_a = log_a.contiguous()
    log_b = log_b.contiguous()
    phi = torch.empty(n, dtype=torch.float32, device=dev)
    psi = torch.empty(m, dtype=torch.float32, device=dev)
    wf = _lib.out_i64()
    call("sinkslot_solve_work_floats", n, m, ctypes.byref(wf))
    work = torch.empty(wf.value, dtype=torch.float32, device=dev)
    it = ctypes.c_int64(0)
    conv = ctypes.c_int(0)
    viol = ctypes.c_double(0.0)
    max_iter = int(getattr(stop, "max_iter", 0)) if stop is not None else 0
    check_every = int(getattr(stop, "check_every", 1)) if stop is not None else 1
    tol = float(getattr(stop, "tol", 0.0)) if stop is not None else 0.0
    with torch.cuda.device(dev):
        call("sinkslot_solve_csr", ptr(r_ptr), ptr(r_idx), _idx_bytes(r_idx), ptr(r_lam),
             ptr(c_ptr), ptr(c_idx), _idx_bytes(c_idx), ptr(c_lam), r_idx.numel(), ptr(log_a),
             ptr(log_b), n, m, variant, _MODE_CODE[mode], int(n_iters), max_iter, check_every, tol,
             float(eps) if eps is not None else 0.0, float(alpha),
             ptr(r_tiles), r_tiles.numel() if r_tiles is not None else 0,
             ptr(c_tiles), c_tiles.numel() if c_tiles is not None else 0, ptr(phi), ptr(psi), ptr(work),
             work.numel(), ctypes.byref(it), ctypes.byref(conv), ctypes.byref(viol),
             stream_of(dev))
    if mode == "fixed":
        return phi, psi, int(n_iters), None, None
    return phi, psi, int(it.value), bool(conv.value), float(viol.value)


def sinkslot_alternating_b200(r_ptr, r_idx, r_lam, c_ptr, c_idx, c_lam, log_a, log_b, n, m,
                              n_iters, stop=None, eps=None, tiles=None):
    """Alternating (Gauss-Seidel) Sinkhorn over prebuilt CSR/CSC
    (reference: ``sinkslot_alternating_triton``, sinkhorn_solvers.py:195-289).

    Returns (phi, psi, iters_run, converged, final_viol).  ``stop`` carries
    mode / max_iter / tol / check_every; "fixed" (or None) runs exactly
    ``n_iters``; "potential" stops once eps * max|dphi|, |dpsi| since the last
    check is below tol (``eps`` required); "marginal" stops once
    max(|a e^{phi_old-phi} - a|, |b e^{psi_old-psi} - b|) <= tol, checked every
    ``check_every`` iterations and at ``max_iter``.  ``tiles``: optional
    (row layout, column layout) from :func:`build_tiles`; with them iterations
    after the first stage the gathered potential in shared memory.
    """
    return _solve_csr(r_ptr, r_idx, r_lam, c_ptr, c_idx, c_lam, log_a, log_b, n, m, n_iters,
                      stop, eps, 0.5, 0, tiles)


def sinkslot_symmetric_b200(r_ptr, r_idx, r_lam, c_ptr, c_idx, c_lam, log_a, log_b, n, m,
                            n_iters, stop=None, eps=None, alpha=0.5, tiles=None):
    """Symmetric (Jacobi, alpha-blended) Sinkhorn over prebuilt CSR/CSC
    (reference: ``sinkslot_symmetric_triton``, sinkhorn_solvers.py:292-419).

    Both half-steps read the same (phi, psi); ``x <- (1-alpha) x + alpha cand``.
    "potential" compares against ``alpha * tol``; "marginal" recomputes both
    candidates from the blended state at each check.
    """
    return _solve_csr(r_ptr, r_idx, r_lam, c_ptr, c_idx, c_lam, log_a, log_b, n, m, n_iters,
                      stop, eps, alpha, 1, tiles)


# Drop-in names for callers of the reference's fused loops (its bench harness and
# apps call them directly with prebuilt CSR/CSC).
sinkslot_alternating_triton = sinkslot_alternating_b200
sinkslot_symmetric_triton = sinkslot_symmetric_b200


def _validate(X, Y, a, b, backend, variant):
    """The reference's argument checks, in its order (sinkhorn_solvers.py:654-690),
    then this backend's own requirement: CUDA float32 tensors."""
    if backend not in BACKENDS:
        raise ValueError(f"backend must be 'auto', 'b200', or 'triton', got {backend!r}"
                         + ("; backend='torch' is the reference's portable fallback, which "
                            "sinkslot_b200 does not provide" if backend == "torch" else ""))
    if variant not in ("alternating", "symmetric"):
        raise ValueError(f"variant must be 'alternating' or 'symmetric', got {variant!r}")
    if X.dtype in (torch.float16, torch.bfloat16) or Y.dtype in (torch.float16, torch.bfloat16):
        raise ValueError(
            f"sinkslot_solve does not support half precision: the log-domain "
            f"iteration overflows (bfloat16 returns inf by n=2048; float16 "
            f"drifts several percent). Got X.dtype={X.dtype}, Y.dtype={Y.dtype}. "
            f"Cast to float32 first."
        )
    if not torch.allclose(a.sum(), b.sum().to(a.dtype), rtol=1e-4, atol=1e-4):
        raise ValueError(
            f"a and b must have equal total mass, got sum(a)={a.sum().item():.6g} "
            f"!= sum(b)={b.sum().item():.6g}"
        )
    if not (X.is_cuda and Y.is_cuda):
        raise ValueError(f"backend={backend!r}: sinkslot_b200 requires X and Y on CUDA "
                         f"(there is no CPU path); got X on {X.device}")
    if X.dtype != torch.float32 or Y.dtype != torch.float32:
        raise ValueError(
            f"sinkslot_b200's fused kernels are float32-only (fixed float32 accumulator); "
            f"got X.dtype={X.dtype}, Y.dtype={Y.dtype}. Cast to float32 first.")


@jaxtyped(typechecker=beartype)
def sinkslot_solve(X: Float[torch.Tensor, "n d"], Y: Float[torch.Tensor, "m d"],
                   a: Float[torch.Tensor, "n"] | None = None,
                   b: Float[torch.Tensor, "m"] | None = None,
                   eps=0.05, L=64, seed=0, n_iters=200,
                   stop_mode="fixed", stop_max_iter=20000, stop_tol=1e-6,
                   stop_check_every=5, chunk=None, backend="auto",
                   variant="alternating", alpha=0.5) -> SinkslotSolveResult:
    """SinkSLOT end to end on one B200: build the sliced support, then solve
    (reference: sinkhorn_solvers.py:591-722).

    Same arguments, defaults, validation errors and return value as the
    reference.  ``backend``: "auto" (default) and "b200" run the sm_100a
    kernels; "triton" is accepted as a synonym for the fused GPU path.  X, Y
    must be float32 CUDA tensors.
    """
    if a is None:
        a = torch.full((X.shape[0],), 1.0 / X.shape[0], device=X.device, dtype=X.dtype)
    if b is None:
        b = torch.full((Y.shape[0],), 1.0 / Y.shape[0], device=Y.device, dtype=Y.dtype)
    _validate(X, Y, a, b, backend, variant)
    stop = None if stop_mode == "fixed" else SimpleNamespace(
        mode=stop_mode, max_iter=stop_max_iter, tol=stop_tol, check_every=stop_check_every)
    _resolve_stop_mode(stop)
    if stop_mode == "potential" and eps is None:
        raise ValueError("eps is required for stop.mode == 'potential'")
    phi, psi, rows, cols, S, info = torch.ops.sinkslot_b200.solve(
        X, Y, a, b, float(eps), int(L), int(seed), int(n_iters), str(stop_mode),
        int(stop_max_iter), float(stop_tol), int(stop_check_every),
        None if chunk is None else int(chunk), str(variant), float(alpha))
    it, conv, viol = info.tolist()
    if stop_mode == "fixed":
        return SinkslotSolveResult(phi, psi, rows, cols, S, int(it), None, None)
    return SinkslotSolveResult(phi, psi, rows, cols, S, int(it), bool(conv), float(viol))


def _solve_impl(X, Y, a, b, eps, L, seed, n_iters, stop_mode, stop_max_iter, stop_tol,
                stop_check_every, chunk, variant, alpha):
    """The body of the ``sinkslot_b200::solve`` operator (arguments validated)."""
    stop = None if stop_mode == "fixed" else SimpleNamespace(
        mode=stop_mode, max_iter=stop_max_iter, tol=stop_tol, check_every=stop_check_every)
    n, m = X.shape[0], Y.shape[0]
    rows, cols, S = sot_plan_coo(X, Y, a, b, L=L, seed=seed, chunk=chunk)
    lam, _ = cost_and_lam(X, Y, rows, cols, S, eps)
    log_a, log_b = a.log(), b.log()
    r_ptr, r_idx, r_lam, _ = _to_csr(rows, cols, lam, n, want_perm=False)
    c_ptr, c_idx, c_lam, _ = _to_csr(cols, rows, lam, m, want_perm=False)
    nnz = rows.numel()
    tiles = (build_tiles(r_ptr, r_idx, r_lam, n, m) if tiles_pay_off(n, m, nnz) else None,
             build_tiles(c_ptr, c_idx, c_lam, m, n) if tiles_pay_off(m, n, nnz) else None)
    if variant == "symmetric":
        phi, psi, it, converged, viol = sinkslot_symmetric_b200(
            r_ptr, r_idx, r_lam, c_ptr, c_idx, c_lam, log_a, log_b, n, m, n_iters, stop, eps,
            alpha, tiles=tiles)
    else:
        phi, psi, it, converged, viol = sinkslot_alternating_b200(
            r_ptr, r_idx, r_lam, c_ptr, c_idx, c_lam, log_a, log_b, n, m, n_iters, stop, eps,
            tiles=tiles)
    return phi, psi, rows, cols, S, it, converged, viol


def plan_values(phi, psi, rows, cols, S, x, y, eps, grad_form: bool = False) -> torch.Tensor:
    """exp(phi[r] + psi[c] + log S - cost/eps) with the cost recomputed in-kernel.
    ``grad_form`` selects slot_grad's association (gradient.py:94-97) over
    sparse_transport_plan's (sinkhorn_solvers.py:757-758)."""
    return torch.ops.sinkslot_b200.plan_values(phi, psi, rows, cols, S, x, y, float(eps),
                                               bool(grad_form))


def _plan_values_impl(phi, psi, rows, cols, S, x, y, eps, grad_form):
    dev = phi.device
    out = torch.empty(rows.numel(), dtype=torch.float32, device=dev)
    x, y = x.contiguous(), y.contiguous()
    with torch.cuda.device(dev):
        call("sinkslot_plan_values", ptr(phi), ptr(psi), ptr(rows), ptr(cols), ptr(S), ptr(x),
             ptr(y), x.shape[1], rows.numel(), float(eps), 1 if grad_form else 0, ptr(out),
             stream_of(dev))
    return out


@jaxtyped(typechecker=beartype)
def sparse_transport_plan(x: Float[torch.Tensor, "n d"], y: Float[torch.Tensor, "m d"],
                          a: Float[torch.Tensor, "n"] | None = None,
                          b: Float[torch.Tensor, "m"] | None = None, *,
                          eps=0.05, L=64, seed=0,
                          n_iters=200, stop_mode="fixed", stop_max_iter=20000,
                          stop_tol=1e-6, stop_check_every=5, backend="auto",
                          variant="alternating", alpha=0.5) -> torch.Tensor:
    """The transport plan as a sparse (n, m) COO tensor
    (reference: sinkhorn_solvers.py:725-764)."""
    n, m = x.shape[0], y.shape[0]
    phi, psi, rows, cols, S, it, converged, viol = sinkslot_solve(
        x, y, a, b, eps, L, seed, n_iters, stop_mode=stop_mode,
        stop_max_iter=stop_max_iter, stop_tol=stop_tol,
        stop_check_every=stop_check_every, backend=backend,
        variant=variant, alpha=alpha)
    vals = plan_values(phi, psi, rows, cols, S, x, y, eps, grad_form=False)
    # rows/cols come sorted by r*m+c without duplicates, i.e. already coalesced
    P = torch.sparse_coo_tensor(torch.stack([rows, cols]), vals, size=(n, m),
                                is_coalesced=True)
    return P
