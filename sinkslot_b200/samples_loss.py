"""GeomLoss-style ``SamplesLoss`` on the sm_100a backend.

Mirrors ``sinkslot/samples_loss.py`` of the reference: forward returns the dual
value ``eps * (<phi, a> + <psi, b>)``; backward is the envelope-theorem
gradient ``2 a (x - T_eps(x))`` from the plan saved by forward (no second solve).
"""

from __future__ import annotations

import torch
from beartype import beartype
from jaxtyping import Float, jaxtyped

from ._lib import call, ptr, stream_of
from .gradient import grad_from_plan
from .sinkhorn_solvers import plan_values, sinkslot_solve


def dual_value(phi, a, psi, b, eps) -> torch.Tensor:
    """eps * (<phi, a> + <psi, b>) as a 0-dim float32 tensor (fp64 accumulation)."""
    dev = phi.device
    acc = torch.empty(1, dtype=torch.float64, device=dev)
    with torch.cuda.device(dev):
        call("sinkslot_dual_value", ptr(phi), ptr(a.contiguous()), phi.numel(), ptr(psi),
             ptr(b.contiguous()), psi.numel(), ptr(acc), stream_of(dev))
    return (acc[0] * eps).to(torch.float32)


class _SLOTCostFn(torch.autograd.Function):
    """Forward: solve + dual value; backward: envelope gradient from the saved
    plan (reference: samples_loss.py:37-85)."""

    @staticmethod
    def forward(ctx, X, Y, a, b, eps, L, seed, n_iters, backend, variant, alpha,
                stop_mode, stop_max_iter, stop_tol, stop_check_every):
        phi, psi, rows, cols, S, it, converged, viol = sinkslot_solve(
            X, Y, a, b, eps, L, seed, n_iters, stop_mode=stop_mode,
            stop_max_iter=stop_max_iter, stop_tol=stop_tol,
            stop_check_every=stop_check_every, backend=backend,
            variant=variant, alpha=alpha)
        T_vals = plan_values(phi, psi, rows, cols, S, X, Y, eps, grad_form=True)
        loss = dual_value(phi, a, psi, b, eps)
        ctx.save_for_backward(X, Y, a, T_vals, rows, cols)
        return loss

    @staticmethod
    def backward(ctx, grad_output):
        X, Y, a, T_vals, rows, cols = ctx.saved_tensors
        grad_x = grad_from_plan(T_vals, rows, cols, X, Y, a)
        return (grad_output * grad_x,
                None, None, None, None, None, None, None, None, None, None,
                None, None, None, None)


class SamplesLoss(torch.nn.Module):
    """SLOT_eps(x, y) as a callable loss module (reference: samples_loss.py:88-167).

    Same constructor keywords and ``forward(x, y, a=None, b=None,
    potentials=False)`` contract; ``potentials=True`` returns (phi, psi).
    """

    def __init__(self, *, eps: float = 0.05, L: int = 64,
                 seed: int = 0, n_iters: int = 200, backend: str = "auto",
                 variant: str = "alternating", alpha: float = 0.5,
                 stop_mode: str = "fixed", stop_max_iter: int = 20000,
                 stop_tol: float = 1e-6, stop_check_every: int = 5):
        super().__init__()
        self.eps = eps
        self.L = L
        self.seed = seed
        self.n_iters = n_iters
        self.backend = backend
        self.variant = variant
        self.alpha = alpha
        self.stop_mode = stop_mode
        self.stop_max_iter = stop_max_iter
        self.stop_tol = stop_tol
        self.stop_check_every = stop_check_every

    @jaxtyped(typechecker=beartype)
    def forward(self, x: Float[torch.Tensor, "n d"], y: Float[torch.Tensor, "m d"],
                a: Float[torch.Tensor, "n"] | None = None,
                b: Float[torch.Tensor, "m"] | None = None,
                potentials: bool = False):
        n, m = x.shape[0], y.shape[0]
        if a is None:
            a = torch.full((n,), 1.0 / n, device=x.device, dtype=x.dtype)
        if b is None:
            b = torch.full((m,), 1.0 / m, device=y.device, dtype=y.dtype)
        if potentials:
            phi, psi, *_ = sinkslot_solve(
                x, y, a, b, self.eps, self.L, self.seed, self.n_iters,
                stop_mode=self.stop_mode, stop_max_iter=self.stop_max_iter,
                stop_tol=self.stop_tol, stop_check_every=self.stop_check_every,
                backend=self.backend, variant=self.variant, alpha=self.alpha)
            return phi, psi
        return _SLOTCostFn.apply(x, y, a, b, self.eps, self.L, self.seed,
                                 self.n_iters, self.backend, self.variant, self.alpha,
                                 self.stop_mode, self.stop_max_iter, self.stop_tol,
                                 self.stop_check_every)
