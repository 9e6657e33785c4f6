"""The MINRES recurrence the device solver restates, on CPU (float64): it
converges to the exact solution of symmetric systems -- indefinite ones and the
Hessian-vector product's regularised system (reference: sinkslot/hvp.py:84-108,
whose solve goes through torchsparsegradutils' MINRES)."""

from __future__ import annotations

import numpy as np
import pytest


def test_minres_solves_symmetric_indefinite_systems():
    from oracle.oracle import minres
    rng = np.random.default_rng(0)
    for n in (5, 40, 200):
        Q, _ = np.linalg.qr(rng.standard_normal((n, n)))
        ev = rng.uniform(0.5, 3.0, n) * rng.choice([-1.0, 1.0], n)
        A = (Q * ev) @ Q.T
        b = rng.standard_normal(n)
        x, it, res = minres(lambda z: A @ z, b, tol=1e-12, max_iter=10 * n)
        np.testing.assert_allclose(x, np.linalg.solve(A, b), rtol=1e-8, atol=1e-9)
        assert res <= 1e-10 and it <= 10 * n


@pytest.mark.parametrize("seed", [0, 1])
def test_minres_on_the_hvp_system_matches_the_dense_solve(seed):
    from oracle import oracle as O
    rng = np.random.default_rng(seed)
    n, d, L, eps = 60, 3, 16, 0.1
    x = rng.standard_normal((n, d)).astype(np.float32)
    y = (rng.standard_normal((n, d)) + 0.5).astype(np.float32)
    a = np.full(n, 1.0 / n, np.float32)
    res = O.sinkslot_solve(x, y, a, a, eps, L, 0, 2000, builder="cuda")
    cost = O.sqeuclid_cost(x, y, res.rows, res.cols)
    T = O.plan_values(res.phi, res.psi, res.rows, res.cols, res.S, cost, eps, grad_form=True)
    v = rng.standard_normal((n, d)).astype(np.float32)
    dense = O.hvp_x_sqeuclid_from_potentials(x, y, a, v, res.rows, res.cols, T, eps)
    kry = O.hvp_x_sqeuclid_from_potentials(x, y, a, v, res.rows, res.cols, T, eps,
                                           solver="minres")
    np.testing.assert_allclose(kry, dense, rtol=1e-6, atol=1e-9 * np.abs(dense).max())
