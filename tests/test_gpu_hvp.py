"""Hessian-vector product on the device (reference: sinkslot/hvp.py, tests in
sinkslot/testing/test_hvp.py).

* against the oracle's float64 restatement with the linear system solved
  exactly (the point MINRES converges to), on the same plan;
* against a frozen-support central finite difference of the envelope gradient
  (the reference's own check: relative error below 8%, at two step sizes);
* linear in v;
* a and b: one marginal for both clouds, as the reference, so n != m is an
  error.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cuda():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import sinkslot_b200
    sinkslot_b200.load_library()
    return torch.device("cuda:0")


def _problem(cuda, n=300, d=3, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(n, d, generator=g).to(cuda)
    y = (torch.randn(n, d, generator=g) + 1.0).to(cuda)
    a = torch.full((n,), 1.0 / n, device=cuda)
    return x, y, a


def _frozen_grad(X, Y, a, rows, cols, S, eps, n_iters):
    """slot_grad's formula on a fixed support (rows, cols, S), through this
    backend's own solve (test_hvp.py:42-63)."""
    from sinkslot_b200.gradient import grad_from_plan
    from sinkslot_b200.sinkhorn_solvers import plan_values, sinkslot_alternating_b200
    from sinkslot_b200.solver import _to_csr, cost_and_lam
    n, m = X.shape[0], Y.shape[0]
    lam, _ = cost_and_lam(X, Y, rows, cols, S, eps)
    r = _to_csr(rows, cols, lam, n, want_perm=False)
    c = _to_csr(cols, rows, lam, m, want_perm=False)
    la = a.log()
    phi, psi, *_ = sinkslot_alternating_b200(r[0], r[1], r[2], c[0], c[1], c[2], la, la, n, m,
                                             n_iters)
    T = plan_values(phi, psi, rows, cols, S, X, Y, eps, grad_form=True)
    return grad_from_plan(T, rows, cols, X, Y, a)


def test_hvp_matches_the_exact_linear_solve(cuda, oracle):
    from sinkslot_b200 import sinkslot_solve
    from sinkslot_b200.hvp import hvp_x_sqeuclid_from_potentials
    from sinkslot_b200.sinkhorn_solvers import plan_values
    X, Y, a = _problem(cuda, n=400, seed=3)
    eps, L = 0.05, 32
    r = sinkslot_solve(X, Y, a, a, eps, L, 0, 3000)
    T = plan_values(r.phi, r.psi, r.rows, r.cols, r.S, X, Y, eps, grad_form=True)
    g = torch.Generator(device="cpu").manual_seed(4)
    v = torch.randn(X.shape, generator=g).to(cuda)
    h, info = hvp_x_sqeuclid_from_potentials(X, Y, a, v, r.rows, r.cols, T, eps,
                                             return_info=True)
    want = oracle.hvp_x_sqeuclid_from_potentials(
        X.cpu().numpy(), Y.cpu().numpy(), a.cpu().numpy(), v.cpu().numpy(), r.rows.cpu().numpy(),
        r.cols.cpu().numpy(), T.cpu().numpy(), eps)
    err = np.linalg.norm(h.cpu().numpy() - want) / np.linalg.norm(want)
    assert err < 2e-3, f"relative error {err:.2e} ({info})"
    assert info.iters >= 1 and np.isfinite(info.rel_residual)


def _frozen_grad64(X, Y, a, rows, cols, S, eps, n_iters):
    """The same envelope gradient in float64 (the reference's torch-backend loop
    restated, test infrastructure): a finite difference of it is free of the
    float32 rounding noise that dominates at small steps."""
    from oracle.torch_ref import alternating_fixed
    X, Y, a, S = X.double(), Y.double(), a.double(), S.double()
    n, m = X.shape[0], Y.shape[0]
    cost = (X[rows] - Y[cols]).square().sum(1)
    lam = S.clamp_min(torch.finfo(torch.float32).tiny).log() - cost / eps
    la = a.log()
    phi, psi = alternating_fixed(rows, cols, lam, la, la, n, m, n_iters)
    T = (phi[rows] + psi[cols] + lam).exp()
    Tx = torch.zeros_like(X).index_add_(0, rows, T[:, None] * Y[cols])
    r = torch.zeros(n, dtype=torch.float64, device=X.device).index_add_(0, rows, T)
    return 2.0 * a[:, None] * (X - Tx / r.clamp_min(torch.finfo(torch.float32).tiny)[:, None])


def test_hvp_matches_frozen_support_finite_difference(cuda):
    """test_hvp.py:66-101: n = 300, eps = 0.05, L = 40, 5000 iterations; the
    relative error against the frozen-support central difference below 8% --
    with this backend's float32 solve at h = 1e-3 (as the reference's test), and
    with the float64 iteration at h = 1e-3 and 3e-4 (at 3e-4 a float32
    difference quotient is dominated by rounding)."""
    from sinkslot_b200 import hvp_x_sqeuclid, sot_plan_coo
    X, Y, a = _problem(cuda)
    eps, L, seed, n_iters = 0.05, 40, 0, 5000
    g = torch.Generator(device="cpu").manual_seed(1)
    v = torch.randn(X.shape, generator=g).to(cuda)
    v = v / v.norm()
    hvp = hvp_x_sqeuclid(X, Y, a, eps, L, seed, n_iters, v)
    rows, cols, S = sot_plan_coo(X, Y, a, a, L=L, seed=seed)
    h = 1e-3
    fd = (_frozen_grad(X + h * v, Y, a, rows, cols, S, eps, n_iters)
          - _frozen_grad(X - h * v, Y, a, rows, cols, S, eps, n_iters)) / (2 * h)
    rel = float((hvp - fd).norm() / fd.norm())
    assert rel < 0.08, f"h={h:g}: hvp disagrees with the frozen-support FD: {rel:.3e}"
    for h in (1e-3, 3e-4):
        fd = (_frozen_grad64(X + h * v, Y, a, rows, cols, S, eps, n_iters)
              - _frozen_grad64(X - h * v, Y, a, rows, cols, S, eps, n_iters)) / (2 * h)
        rel = float((hvp.double() - fd).norm() / fd.norm())
        assert rel < 0.08, f"h={h:g}: hvp disagrees with the float64 frozen FD: {rel:.3e}"


def test_hvp_is_linear_in_v(cuda):
    """test_hvp.py:103-119."""
    from sinkslot_b200 import hvp_x_sqeuclid
    X, Y, a = _problem(cuda, n=150, seed=4)
    g = torch.Generator(device="cpu").manual_seed(5)
    v = torch.randn(X.shape, generator=g).to(cuda)
    h1 = hvp_x_sqeuclid(X, Y, a, 0.05, 30, 0, 5000, v)
    h2 = hvp_x_sqeuclid(X, Y, a, 0.05, 30, 0, 5000, 2.0 * v)
    assert float((h2 - 2.0 * h1).norm() / h1.norm()) < 1e-2
    # deterministic: the same call twice gives the same bits
    assert torch.equal(h1, hvp_x_sqeuclid(X, Y, a, 0.05, 30, 0, 5000, v))


def test_hvp_needs_one_marginal_for_both_clouds(cuda):
    from sinkslot_b200.hvp import hvp_x_sqeuclid_from_potentials
    X, Y, a = _problem(cuda, n=50)
    with pytest.raises(ValueError, match="same"):
        hvp_x_sqeuclid_from_potentials(X, Y[:40], a, X, torch.zeros(1, dtype=torch.int64,
                                                                    device=cuda),
                                       torch.zeros(1, dtype=torch.int64, device=cuda),
                                       torch.ones(1, device=cuda), 0.05)
