"""The library's entry points as PyTorch operators (``torch.ops.sinkslot_b200.*``).

Every public function of the package reaches libsinkslot_b200.so through one of
these operators, so the calls are visible to PyTorch's dispatcher, profiler and
``torch.compile`` (each operator has a fake implementation that gives its output
shapes without running anything; the support's size is data-dependent and is a
dynamic size there).  The operator bodies are the host wrappers of the C ABI;
none has a CPU kernel: the library runs on CUDA tensors only.
"""

from __future__ import annotations

from typing import Optional

import torch
from torch import Tensor
from torch.library import custom_op

NS = "sinkslot_b200"


@custom_op(f"{NS}::sot_plan_coo", mutates_args=())
def sot_plan_coo(X: Tensor, Y: Tensor, a: Tensor, b: Tensor, L: int, seed: int,
                 chunk: Optional[int]) -> tuple[Tensor, Tensor, Tensor]:
    from .solver import _sot_plan_coo_impl
    return _sot_plan_coo_impl(X, Y, a, b, L, seed, chunk)


@sot_plan_coo.register_fake
def _(X, Y, a, b, L, seed, chunk):
    k = torch.library.get_ctx().new_dynamic_size()
    return (X.new_empty(k, dtype=torch.int64), X.new_empty(k, dtype=torch.int64),
            X.new_empty(k, dtype=torch.float32))


@custom_op(f"{NS}::sparse_sqeuclidean_cost", mutates_args=())
def sparse_sqeuclidean_cost(x: Tensor, y: Tensor, rows: Tensor, cols: Tensor) -> Tensor:
    from .solver import _sqeuclid_cost_impl
    return _sqeuclid_cost_impl(x, y, rows, cols)


@sparse_sqeuclidean_cost.register_fake
def _(x, y, rows, cols):
    return x.new_empty(rows.shape[0], dtype=torch.float32)


@custom_op(f"{NS}::seg_lse", mutates_args=())
def seg_lse(indptr: Tensor, colidx: Tensor, lam: Tensor, phi: Tensor, psi: Tensor, n: int,
            base: Optional[Tensor]) -> Tensor:
    from .sinkhorn_solvers import _seg_lse_impl
    out = torch.empty(n, dtype=lam.dtype, device=lam.device)
    _seg_lse_impl(indptr, colidx, lam, phi, psi, n, base, out)
    return out


@seg_lse.register_fake
def _(indptr, colidx, lam, phi, psi, n, base):
    return lam.new_empty(n)


@custom_op(f"{NS}::solve", mutates_args=())
def solve(X: Tensor, Y: Tensor, a: Tensor, b: Tensor, eps: float, L: int, seed: int,
          n_iters: int, stop_mode: str, stop_max_iter: int, stop_tol: float,
          stop_check_every: int, chunk: Optional[int], variant: str,
          alpha: float) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor, Tensor]:
    """The whole sinkslot_solve; the last output is a CPU float64 tensor
    [iters_run, converged (-1: fixed mode), final_viol (NaN: fixed mode)]."""
    from .sinkhorn_solvers import _solve_impl
    phi, psi, rows, cols, S, it, conv, viol = _solve_impl(
        X, Y, a, b, eps, L, seed, n_iters, stop_mode, stop_max_iter, stop_tol,
        stop_check_every, chunk, variant, alpha)
    info = torch.tensor([float(it), -1.0 if conv is None else float(conv),
                         float("nan") if viol is None else float(viol)], dtype=torch.float64)
    return phi, psi, rows, cols, S, info


@solve.register_fake
def _(X, Y, a, b, eps, L, seed, n_iters, stop_mode, stop_max_iter, stop_tol, stop_check_every,
      chunk, variant, alpha):
    k = torch.library.get_ctx().new_dynamic_size()
    return (X.new_empty(X.shape[0]), X.new_empty(Y.shape[0]),
            X.new_empty(k, dtype=torch.int64), X.new_empty(k, dtype=torch.int64),
            X.new_empty(k), torch.empty(3, dtype=torch.float64, device="cpu"))


@custom_op(f"{NS}::plan_values", mutates_args=())
def plan_values(phi: Tensor, psi: Tensor, rows: Tensor, cols: Tensor, S: Tensor, x: Tensor,
                y: Tensor, eps: float, grad_form: bool) -> Tensor:
    from .sinkhorn_solvers import _plan_values_impl
    return _plan_values_impl(phi, psi, rows, cols, S, x, y, eps, grad_form)


@plan_values.register_fake
def _(phi, psi, rows, cols, S, x, y, eps, grad_form):
    return S.new_empty(rows.shape[0])


@custom_op(f"{NS}::barycentric", mutates_args=())
def barycentric(T_vals: Tensor, rows: Tensor, cols: Tensor, x: Tensor, y: Tensor,
                a: Optional[Tensor], want_tx: bool, want_ty: bool,
                want_grad: bool) -> tuple[Tensor, Tensor, Tensor]:
    """(Tx, Ty, grad); the ones not asked for are empty."""
    from .gradient import _bary_impl
    Tx, Ty, g = _bary_impl(T_vals, rows, cols, x, y, a, want_tx, want_ty, want_grad)
    # (operator outputs may not alias one another: a fresh empty tensor each)
    return (Tx if Tx is not None else x.new_empty(0), Ty if Ty is not None else x.new_empty(0),
            g if g is not None else x.new_empty(0))


@barycentric.register_fake
def _(T_vals, rows, cols, x, y, a, want_tx, want_ty, want_grad):
    return (x.new_empty(x.shape) if want_tx else x.new_empty(0),
            y.new_empty(y.shape) if want_ty else x.new_empty(0),
            x.new_empty(x.shape) if want_grad else x.new_empty(0))


@custom_op(f"{NS}::hvp_from_potentials", mutates_args=())
def hvp_from_potentials(X: Tensor, Y: Tensor, a: Tensor, v: Tensor, rows: Tensor, cols: Tensor,
                        T_vals: Tensor, eps: float, tau2: float, solve_tol: float,
                        max_cg_iter: int) -> tuple[Tensor, Tensor]:
    """(H v, CPU float64 [iterations, relative residual])."""
    from .hvp import _hvp_impl
    out, it, res = _hvp_impl(X, Y, a, v, rows, cols, T_vals, eps, tau2, solve_tol, max_cg_iter)
    return out, torch.tensor([float(it), float(res)], dtype=torch.float64)


@hvp_from_potentials.register_fake
def _(X, Y, a, v, rows, cols, T_vals, eps, tau2, solve_tol, max_cg_iter):
    return X.new_empty(X.shape), torch.empty(2, dtype=torch.float64, device="cpu")
