"""The CPU oracle against the reference's own outputs (tests/golden/*.npz).

Pins the oracle before it is trusted as the checker of the sm_100a kernels:
support (rows, cols, S) bit-exact, costs bit-exact, potentials / gradient /
plan within rtol 1e-4, atol 1e-5 after a fixed number of iterations, and the
stop-mode results of the reference's loops.
"""

from __future__ import annotations

import hashlib

import numpy as np
import pytest

from conftest import GOLDEN_CASES, assert_close_np, load_golden


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.mark.parametrize("case", GOLDEN_CASES)
@pytest.mark.parametrize("builder,tag", [("cuda_on_cpu", "cudabuilder"), ("cpu", "naive")])
def test_oracle_support_matches_reference(oracle, case, builder, tag):
    meta, g = load_golden(case)
    rows, cols, S = oracle.sot_plan_coo(g["x"], g["y"], g["a"], g["b"], meta["L"], 0,
                                        builder=builder)
    assert rows.size == meta[f"nnz_{tag}"]
    assert sha(rows) == meta[f"sha_rows_{tag}"]
    assert sha(cols) == meta[f"sha_cols_{tag}"]
    assert sha(S) == meta[f"sha_S_{tag}"]
    if f"rows_{tag}" in g:
        np.testing.assert_array_equal(rows, g[f"rows_{tag}"])
        np.testing.assert_array_equal(S, g[f"S_{tag}"])


@pytest.mark.parametrize("case", GOLDEN_CASES)
def test_oracle_directions_match_reference(oracle, case):
    meta, g = load_golden(case)
    th = oracle.get_random_projections(meta["d"], meta["L"], 0)
    np.testing.assert_array_equal(th, g["theta"])


@pytest.mark.parametrize("case", GOLDEN_CASES)
def test_oracle_cost_matches_reference(oracle, case):
    meta, g = load_golden(case)
    rows, cols, S = oracle.sot_plan_coo(g["x"], g["y"], g["a"], g["b"], meta["L"], 0,
                                        builder="cpu")
    cost = oracle.sqeuclid_cost(g["x"], g["y"], rows, cols)
    assert sha(cost) == meta["sha_cost"]


@pytest.mark.parametrize("case", GOLDEN_CASES)
@pytest.mark.parametrize("variant", ["alternating", "symmetric"])
def test_oracle_fixed_solve_matches_reference(oracle, case, variant):
    meta, g = load_golden(case)
    res = oracle.sinkslot_solve(g["x"], g["y"], g["a"], g["b"], meta["eps"], meta["L"], 0,
                                meta["n_iters"], variant=variant, builder="cpu")
    key = "alt" if variant == "alternating" else "sym"
    assert res.iters_run == meta["n_iters"] and res.converged is None
    assert_close_np(res.phi, g[f"phi_{key}"], name="phi")
    assert_close_np(res.psi, g[f"psi_{key}"], name="psi")


@pytest.mark.parametrize("case", GOLDEN_CASES)
def test_oracle_grad_and_loss_match_reference(oracle, case):
    meta, g = load_golden(case)
    grad = oracle.slot_grad(g["x"], g["y"], g["a"], g["b"], meta["eps"], meta["L"], 0,
                            meta["n_iters"], builder="cpu")
    scale = np.abs(g["grad"]).max()
    assert_close_np(grad, g["grad"], rtol=1e-4, atol=1e-5 * scale, name="grad")
    res = oracle.sinkslot_solve(g["x"], g["y"], g["a"], g["b"], meta["eps"], meta["L"], 0,
                                meta["n_iters"], builder="cpu")
    loss = oracle.samples_loss_value(res.phi, res.psi, g["a"], g["b"], meta["eps"])
    if np.isnan(meta["loss"]):  # zero weights: phi * a = inf * 0 in the reference too
        assert np.isnan(loss)
    else:
        assert loss == pytest.approx(meta["loss"], rel=1e-5, abs=1e-6)


@pytest.mark.parametrize("case", ["small_nonuniform", "bench_shape", "zero_weights"])
def test_oracle_plan_and_barycentric_match_reference(oracle, case):
    meta, g = load_golden(case)
    res = oracle.sinkslot_solve(g["x"], g["y"], g["a"], g["b"], meta["eps"], meta["L"], 0,
                                meta["n_iters"], builder="cpu")
    cost = oracle.sqeuclid_cost(g["x"], g["y"], res.rows, res.cols)
    P = oracle.plan_values(res.phi, res.psi, res.rows, res.cols, res.S, cost, meta["eps"])
    sc = np.abs(g["plan_vals"]).max()
    assert_close_np(P, g["plan_vals"], rtol=1e-4, atol=1e-6 * sc, name="plan")
    Tx, Ty = oracle.barycentric_map(g["plan_vals"], res.rows, res.cols, g["x"], g["y"])
    assert_close_np(Tx, g["Tx"], rtol=1e-5, atol=1e-6, name="Tx")
    assert_close_np(Ty, g["Ty"], rtol=1e-5, atol=1e-6, name="Ty")


@pytest.mark.parametrize("variant", ["alternating", "symmetric"])
@pytest.mark.parametrize("mode,tol", [("marginal", 1e-6), ("potential", 1e-4)])
def test_oracle_stop_modes_match_reference(oracle, variant, mode, tol):
    """Early-stopping runs: the iteration count agrees to within one check
    interval (exp/log differ by an ulp between libm and torch's vector
    library, which can move the crossing by one check), convergence agrees,
    and the plans agree (potentials are compared after removing the common
    (+c, -c) shift, which the iteration does not damp)."""
    meta, g = load_golden("small_nonuniform")
    res = oracle.sinkslot_solve(g["x"], g["y"], g["a"], g["b"], meta["eps"], meta["L"], 0, 20000,
                                stop_mode=mode, stop_max_iter=20000, stop_tol=tol,
                                variant=variant, builder="cpu")
    key = f"{variant}_{mode}"
    assert res.converged == meta[f"conv_{key}"]
    assert abs(res.iters_run - meta[f"iters_{key}"]) <= 5
    phi, psi = g[f"phi_{key}"], g[f"psi_{key}"]
    c = (res.phi.astype(np.float64) - phi).mean()
    np.testing.assert_allclose(res.phi - c, phi, rtol=0, atol=5e-3)
    np.testing.assert_allclose(res.psi + c, psi, rtol=0, atol=5e-3)
