"""Host-side API behaviour that needs no GPU: the reference's validation
errors (same exception types and messages, same order), the absence of any
CPU fallback, and the reference-compatible helpers."""

from __future__ import annotations

import pytest
import torch


def _pair(dtype=torch.float32, n=48, m=40, d=3):
    g = torch.Generator(device="cpu").manual_seed(0)
    x = torch.randn(n, d, generator=g).to(dtype)
    y = (torch.randn(m, d, generator=g) + 1.0).to(dtype)
    return x, y


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_half_precision_refused(dtype):
    from sinkslot_b200 import sinkslot_solve, SamplesLoss
    x, y = _pair(dtype)
    with pytest.raises(ValueError, match="half precision"):
        sinkslot_solve(x, y, eps=0.1, L=16, seed=0, n_iters=10)
    with pytest.raises(ValueError, match="half precision"):
        SamplesLoss(eps=0.1, L=16, seed=0, n_iters=10)(x, y)


def test_bad_backend_and_variant():
    from sinkslot_b200 import sinkslot_solve
    x, y = _pair()
    with pytest.raises(ValueError, match="backend must be"):
        sinkslot_solve(x, y, backend="bogus")
    with pytest.raises(ValueError, match="portable fallback"):
        sinkslot_solve(x, y, backend="torch")
    with pytest.raises(ValueError, match="variant must be"):
        sinkslot_solve(x, y, variant="bogus")


def test_unequal_mass_refused():
    from sinkslot_b200 import sinkslot_solve
    x, y = _pair()
    a = torch.full((48,), 1 / 48)
    b = torch.full((40,), 2 / 40)
    with pytest.raises(ValueError, match="equal total mass"):
        sinkslot_solve(x, y, a, b, 0.1, 16, seed=0, n_iters=10)


def test_cpu_tensors_fail_loudly_no_fallback():
    from sinkslot_b200 import sinkslot_solve, SamplesLoss, sot_plan_coo
    x, y = _pair()
    with pytest.raises(ValueError, match="CUDA"):
        sinkslot_solve(x, y, eps=0.1, L=16, seed=0, n_iters=10)
    with pytest.raises(ValueError, match="CUDA"):
        SamplesLoss(eps=0.1, L=16, n_iters=10)(x, y)
    a = torch.full((48,), 1 / 48)
    b = torch.full((40,), 1 / 40)
    with pytest.raises(ValueError, match="CUDA"):
        sot_plan_coo(x, y, a, b, 16, 0)


def test_unknown_stop_mode_refused():
    from sinkslot_b200.sinkhorn_solvers import _resolve_stop_mode
    from types import SimpleNamespace
    with pytest.raises(ValueError, match="unknown stop.mode"):
        _resolve_stop_mode(SimpleNamespace(mode="bogus"))
    assert _resolve_stop_mode(None) == "fixed"


def test_barycentric_call_forms():
    from sinkslot_b200 import sparse_barycentric_map
    with pytest.raises(TypeError, match="expects"):
        sparse_barycentric_map(1, 2)


def test_launch_cfg_matches_reference_rule():
    from sinkslot_b200 import launch_cfg
    # sinkhorn_solvers.py:97-118: pow2(mean row) in [32, 1024]; 2 warps up to 512
    assert launch_cfg(64 * 1000, 1000) == (64, 2)
    assert launch_cfg(10, 1000) == (32, 2)
    assert launch_cfg(700 * 10, 10) == (1024, 4)
    assert launch_cfg(512 * 3, 3) == (512, 2)


def test_random_projections_match_definition():
    from sinkslot_b200 import get_random_projections
    th = get_random_projections(3, 64, 0)
    assert th.dtype == torch.float64 and th.shape == (64, 3)
    torch.testing.assert_close(th.norm(dim=1), torch.ones(64, dtype=torch.float64))
    g = torch.Generator(device="cpu").manual_seed(0)
    raw = torch.randn((64, 3), generator=g, dtype=torch.float64)
    assert torch.equal(th, raw / raw.norm(dim=1, keepdim=True).clamp_min(1e-300))


def test_exports_match_reference_names():
    import sinkslot_b200
    for name in ["get_random_projections", "sot_plan_coo", "to_csr", "sparse_sqeuclidean_cost",
                 "seg_lse_online", "launch_cfg", "sinkslot_solve", "sparse_transport_plan",
                 "SinkslotSolveResult", "slot_grad", "sparse_barycentric_map", "SamplesLoss"]:
        assert hasattr(sinkslot_b200, name)
    from sinkslot_b200.sinkhorn_solvers import (sinkslot_alternating_triton,
                                                sinkslot_symmetric_triton)
    assert callable(sinkslot_alternating_triton) and callable(sinkslot_symmetric_triton)


def test_batch_assignment_round_robin():
    from sinkslot_b200.batched import batch_assignment
    assert batch_assignment(7, 3) == [[0, 3, 6], [1, 4], [2, 5]]
    assert batch_assignment(2, 4) == [[0], [1], [], []]
    assert batch_assignment(0, 2) == [[], []]
    shares = batch_assignment(101, 8)
    assert sorted(i for s in shares for i in s) == list(range(101))
    with pytest.raises(ValueError):
        batch_assignment(3, 0)


def test_reference_dispatch_patch_applies(tmp_path):
    """The maintainer's dispatch edit applies to the installed reference and the
    patched package still runs its own CPU path (no CUDA here)."""
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    ref = os.path.join(root, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "sinkslot")):
        pytest.skip("the reference package is not installed in baseline/_ref")
    code = f"""
import sys, torch
sys.path.insert(0, {root!r}); sys.path.insert(0, {os.path.join(root, "tests")!r})
from reference_dispatch_patch import patched_copy
sys.path.insert(0, patched_copy({ref!r}, {str(tmp_path)!r}))
import sinkslot
from sinkslot import sinkhorn_solvers as s
assert hasattr(s, "_HAS_B200")
torch.manual_seed(0)
r = sinkslot.sinkslot_solve(torch.randn(50, 2), torch.randn(40, 2), eps=0.1, L=8, n_iters=5)
assert r.phi.device.type == "cpu"
print("ok")
"""
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0 and "ok" in out.stdout, out.stdout + out.stderr
