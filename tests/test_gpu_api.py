"""The reference's public API on the GPU backend: result contract, dtype
contract, plan export, barycentric map, slot_grad and SamplesLoss -- checked
against the oracle (same support) and against the behavioural pins of the
reference's own test suite (marginals, sym == alt plan, envelope gradient)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import assert_close_np, load_golden

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cuda():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import sinkslot_b200
    sinkslot_b200.load_library()
    return torch.device("cuda:0")


def _inputs(case, cuda):
    meta, g = load_golden(case)
    return meta, g, [torch.from_numpy(g[k]).to(cuda) for k in ("x", "y", "a", "b")]


def test_result_contract(cuda):
    from sinkslot_b200 import sinkslot_solve, SinkslotSolveResult
    meta, g, t = _inputs("small_nonuniform", cuda)
    r = sinkslot_solve(*t, 0.05, 40, seed=0, n_iters=10)
    assert isinstance(r, SinkslotSolveResult)
    phi, psi, rows, cols, S, it, conv, viol = r
    assert r.phi is phi and r[0] is phi and r.rows is rows and r.S is S
    assert r.iters_run == it == 10 and r.converged is None and r.final_viol is None
    assert rows.dtype == torch.int64 and cols.dtype == torch.int64 and S.dtype == torch.float32
    assert phi.shape == (300,) and psi.shape == (250,)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_half_precision_refused(cuda, dtype):
    from sinkslot_b200 import sinkslot_solve, SamplesLoss
    x = torch.randn(48, 3, device=cuda).to(dtype)
    y = torch.randn(40, 3, device=cuda).to(dtype)
    with pytest.raises(ValueError, match="half precision"):
        sinkslot_solve(x, y, eps=0.1, L=16, seed=0, n_iters=10)
    with pytest.raises(ValueError, match="half precision"):
        SamplesLoss(eps=0.1, L=16, seed=0, n_iters=10)(x, y)


def test_float64_is_an_explicit_error(cuda):
    from sinkslot_b200 import sinkslot_solve
    x = torch.randn(48, 3, device=cuda, dtype=torch.float64)
    y = torch.randn(40, 3, device=cuda, dtype=torch.float64)
    with pytest.raises(ValueError, match="float32"):
        sinkslot_solve(x, y, eps=0.1, L=16, seed=0, n_iters=10)


def test_marginal_stop_gives_plan_marginals(cuda):
    """test_torch_fallback.py:161-178 on this backend: converged marginal-mode
    solve reproduces a and b to 1e-5."""
    from sinkslot_b200 import sinkslot_solve, sparse_sqeuclidean_cost
    meta, g, (x, y, a, b) = _inputs("small_nonuniform", cuda)
    r = sinkslot_solve(x, y, a, b, 0.05, 40, seed=0, n_iters=20000, stop_mode="marginal",
                       stop_max_iter=20000)
    assert r.converged and r.final_viol <= 1e-6
    cost = sparse_sqeuclidean_cost(x, y, r.rows, r.cols)
    lam = r.S.clamp_min(torch.finfo(torch.float32).tiny).log() - cost / 0.05
    P = (r.phi[r.rows] + r.psi[r.cols] + lam).exp()
    row = torch.zeros(300, device=cuda).index_add_(0, r.rows, P)
    col = torch.zeros(250, device=cuda).index_add_(0, r.cols, P)
    torch.testing.assert_close(row, a, rtol=0, atol=1e-5)
    torch.testing.assert_close(col, b, rtol=0, atol=1e-5)


def test_symmetric_and_alternating_reach_the_same_plan(cuda):
    from sinkslot_b200 import sinkslot_solve
    from sinkslot_b200.sinkhorn_solvers import plan_values
    meta, g, (x, y, a, b) = _inputs("small_nonuniform", cuda)
    kw = dict(stop_mode="marginal", stop_max_iter=20000, stop_tol=1e-8)
    ra = sinkslot_solve(x, y, a, b, 0.05, 40, 0, 20000, variant="alternating", **kw)
    rs = sinkslot_solve(x, y, a, b, 0.05, 40, 0, 20000, variant="symmetric", **kw)
    assert torch.equal(ra.rows, rs.rows) and torch.equal(ra.cols, rs.cols)
    Ta = plan_values(ra.phi, ra.psi, ra.rows, ra.cols, ra.S, x, y, 0.05)
    Ts = plan_values(rs.phi, rs.psi, rs.rows, rs.cols, rs.S, x, y, 0.05)
    assert float((Ta - Ts).norm() / Ta.norm()) < 1e-3


@pytest.mark.parametrize("case", ["small_nonuniform", "bench_shape", "zero_weights"])
def test_plan_export_and_barycentric_match_oracle(cuda, oracle, case):
    from sinkslot_b200 import sparse_transport_plan, sparse_barycentric_map
    meta, g, (x, y, a, b) = _inputs(case, cuda)
    eps, L, it = meta["eps"], meta["L"], meta["n_iters"]
    P = sparse_transport_plan(x, y, a, b, eps=eps, L=L, seed=0, n_iters=it)
    assert P.is_sparse and P.shape == (x.shape[0], y.shape[0]) and P.is_coalesced()
    o = oracle.sinkslot_solve(g["x"], g["y"], g["a"], g["b"], eps, L, 0, it, builder="cuda")
    rows, cols = P.indices()
    np.testing.assert_array_equal(rows.cpu().numpy(), o.rows)
    np.testing.assert_array_equal(cols.cpu().numpy(), o.cols)
    cost = oracle.sqeuclid_cost(g["x"], g["y"], o.rows, o.cols)
    ov = oracle.plan_values(o.phi, o.psi, o.rows, o.cols, o.S, cost, eps)
    sc = float(np.abs(ov[np.isfinite(ov)]).max()) if np.isfinite(ov).any() else 1.0
    assert_close_np(P.values().cpu().numpy(), ov, rtol=2e-3, atol=1e-6 * sc, name="plan")
    Tx, Ty = sparse_barycentric_map(P, x, y)
    Tx2, Ty2 = sparse_barycentric_map(P.values(), rows, cols, x, y)
    assert torch.equal(Tx, Tx2) and torch.equal(Ty, Ty2)
    oTx, oTy = oracle.barycentric_map(P.values().cpu().numpy(), o.rows, o.cols, g["x"], g["y"])
    assert_close_np(Tx.cpu().numpy(), oTx, rtol=1e-5, atol=1e-6, name="Tx")
    assert_close_np(Ty.cpu().numpy(), oTy, rtol=1e-5, atol=1e-6, name="Ty")
    with pytest.raises(TypeError, match="expects"):
        sparse_barycentric_map(P, x)


@pytest.mark.parametrize("case", ["small_nonuniform", "cfg1", "unequal_ties"])
def test_slot_grad_and_samples_loss_match_oracle(cuda, oracle, case):
    from sinkslot_b200 import SamplesLoss, slot_grad
    meta, g, (x, y, a, b) = _inputs(case, cuda)
    eps, L, it = meta["eps"], meta["L"], meta["n_iters"]
    grad = slot_grad(x, y, a, b, eps, L, 0, it)
    og = oracle.slot_grad(g["x"], g["y"], g["a"], g["b"], eps, L, 0, it, builder="cuda")
    sc = float(np.abs(og).max())
    assert_close_np(grad.cpu().numpy(), og, rtol=1e-4, atol=1e-5 * sc, name="grad")
    xr = x.clone().requires_grad_(True)
    loss = SamplesLoss(eps=eps, L=L, n_iters=it)(xr, y, a, b)
    (gx,) = torch.autograd.grad(loss, [xr])
    torch.testing.assert_close(gx, grad, rtol=0, atol=0)
    o = oracle.sinkslot_solve(g["x"], g["y"], g["a"], g["b"], eps, L, 0, it, builder="cuda")
    ol = oracle.samples_loss_value(o.phi, o.psi, g["a"], g["b"], eps)
    assert float(loss) == pytest.approx(ol, rel=1e-4, abs=1e-6)
    phi, psi = SamplesLoss(eps=eps, L=L, n_iters=it)(x, y, a, b, potentials=True)
    assert phi.shape == (x.shape[0],) and psi.shape == (y.shape[0],)


def test_envelope_gradient_matches_frozen_support_finite_difference(cuda):
    """test_torch_fallback.py:587-631 in fp32: the gradient against a central
    difference of <T, C(x)> with the plan frozen."""
    from sinkslot_b200 import slot_grad, sinkslot_solve
    from sinkslot_b200.sinkhorn_solvers import plan_values
    g = torch.Generator().manual_seed(1)
    n, m, eps, L = 50, 35, 0.05, 60
    x = torch.randn(n, 3, generator=g).to(cuda)
    y = (torch.randn(m, 3, generator=g) + 1.0).to(cuda)
    a = torch.rand(n, generator=g).to(cuda); a = a / a.sum()
    b = torch.rand(m, generator=g).to(cuda); b = b / b.sum()
    r = sinkslot_solve(x, y, a, b, eps, L, seed=0, n_iters=3000)
    T = plan_values(r.phi, r.psi, r.rows, r.cols, r.S, x, y, eps, grad_form=True).double()
    v = torch.randn(n, 3, generator=g).double().to(cuda); v = v / v.norm()

    def frozen(xp):
        return (T * (xp[r.rows] - y.double()[r.cols]).square().sum(1)).sum()

    h = 1e-4
    fd = float((frozen(x.double() + h * v) - frozen(x.double() - h * v)) / (2 * h))
    gs = slot_grad(x, y, a, b, eps, L, seed=0, n_iters=3000)
    assert abs(fd - float((gs.double() * v).sum())) / abs(fd) < 1e-4


def test_batched_solves_equal_single_solves(cuda):
    """Independent problems spread over every visible GPU (one host thread per
    device, no communication): each result equals the single-GPU solve of the
    same problem bit for bit (the solve is deterministic)."""
    from sinkslot_b200 import sinkslot_solve, sinkslot_solve_batched
    g = torch.Generator().manual_seed(3)
    probs = []
    for k, (n, m) in enumerate([(700, 500), (400, 400), (900, 650), (300, 800), (550, 550)]):
        x = torch.randn(n, 3, generator=g)
        y = torch.randn(m, 3, generator=g) + 1.0
        if k % 2:
            a = torch.rand(n, generator=g) + 0.1
            b = torch.rand(m, generator=g) + 0.1
            probs.append((x, y, a / a.sum(), b / b.sum()))
        else:
            probs.append((x, y))
    kw = dict(eps=0.05, L=24, seed=0, n_iters=120, variant="alternating")
    out = sinkslot_solve_batched(probs, **kw)
    ndev = torch.cuda.device_count()
    for i, (p, r) in enumerate(zip(probs, out)):
        assert r.phi.device == torch.device("cuda", i % ndev)
        t = [v.to(cuda) for v in p]
        want = sinkslot_solve(*(t if len(t) == 4 else t + [None, None]), **kw)
        assert torch.equal(r.rows.to(cuda), want.rows) and torch.equal(r.cols.to(cuda), want.cols)
        assert torch.equal(r.phi.to(cuda), want.phi) and torch.equal(r.psi.to(cuda), want.psi)
    # stop modes pass through, and a bad problem shape is a TypeError
    out = sinkslot_solve_batched(probs[:2], eps=0.05, L=24, stop_mode="marginal",
                                 stop_max_iter=5000, stop_tol=1e-6)
    assert all(r.converged for r in out)
    with pytest.raises(TypeError):
        sinkslot_solve_batched([(probs[0][0],)], eps=0.05)


@pytest.mark.parametrize("case", ["small_nonuniform", "bench_shape", "cfg1", "unequal_ties",
                                  "zero_weights"])
def test_cost_bit_exact_vs_reference_cpu_run(cuda, oracle, case):
    """sparse_sqeuclidean_cost (and the fused cost of cost_and_lam) on the device
    against the reference's own CPU run of `(x[rows]-y[cols]).square().sum(1)`
    (solver.py:346), stored as a sha256 in the golden fixture, on the support
    of that run: bit for bit."""
    import hashlib
    from sinkslot_b200 import sparse_sqeuclidean_cost
    from sinkslot_b200.solver import cost_and_lam
    meta, g, (x, y, a, b) = _inputs(case, cuda)
    rows, cols, S = oracle.sot_plan_coo(g["x"], g["y"], g["a"], g["b"], meta["L"], 0,
                                        builder="cpu")
    r, c = torch.from_numpy(rows).to(cuda), torch.from_numpy(cols).to(cuda)
    cost = sparse_sqeuclidean_cost(x, y, r, c).cpu().numpy()
    assert hashlib.sha256(np.ascontiguousarray(cost).tobytes()).hexdigest() == meta["sha_cost"]
    np.testing.assert_array_equal(cost, oracle.sqeuclid_cost(g["x"], g["y"], rows, cols))
    _, fused = cost_and_lam(x, y, r, c, torch.from_numpy(S).to(cuda), meta["eps"],
                            want_cost=True)
    np.testing.assert_array_equal(fused.cpu().numpy(), cost)
