"""The library's entry points are PyTorch operators (torch.ops.sinkslot_b200.*):
their schemas exist, and their fake implementations give output shapes without
a GPU (what torch.compile and the dispatcher's meta passes use)."""

from __future__ import annotations

import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode
from torch.fx.experimental.symbolic_shapes import ShapeEnv

OPS = ["sot_plan_coo", "solve", "sparse_sqeuclidean_cost", "seg_lse", "plan_values",
       "barycentric", "hvp_from_potentials"]


@pytest.mark.parametrize("name", OPS)
def test_operator_is_registered(name):
    import sinkslot_b200  # noqa: F401
    op = getattr(torch.ops.sinkslot_b200, name)
    assert op.default._schema.name == f"sinkslot_b200::{name}"


def test_fake_shapes():
    import sinkslot_b200  # noqa: F401
    ops = torch.ops.sinkslot_b200
    with FakeTensorMode(shape_env=ShapeEnv()):
        X = torch.empty(100, 3, device="cuda")
        Y = torch.empty(80, 3, device="cuda")
        a = torch.empty(100, device="cuda")
        b = torch.empty(80, device="cuda")
        rows, cols, S = ops.sot_plan_coo(X, Y, a, b, 16, 0, None)
        assert rows.dtype == torch.int64 and S.dtype == torch.float32
        assert rows.shape == cols.shape == S.shape
        phi, psi, r2, c2, S2, info = ops.solve(X, Y, a, b, 0.05, 16, 0, 10, "fixed", 100, 1e-6, 5,
                                               None, "alternating", 0.5)
        assert phi.shape == (100,) and psi.shape == (80,) and info.shape == (3,)
        r = torch.empty(500, dtype=torch.int64, device="cuda")
        c = torch.empty(500, dtype=torch.int64, device="cuda")
        cost = ops.sparse_sqeuclidean_cost(X, Y, r, c)
        assert cost.shape == (500,)
        T = ops.plan_values(phi, psi, r, c, torch.empty(500, device="cuda"), X, Y, 0.05, True)
        assert T.shape == (500,)
        Tx, Ty, g = ops.barycentric(T, r, c, X, Y, a, True, False, True)
        assert Tx.shape == (100, 3) and Ty.shape == (0,) and g.shape == (100, 3)
        out = ops.seg_lse(torch.empty(101, dtype=torch.int32, device="cuda"),
                          torch.empty(500, dtype=torch.int32, device="cuda"),
                          torch.empty(500, device="cuda"), torch.empty(100, device="cuda"),
                          torch.empty(80, device="cuda"), 100, None)
        assert out.shape == (100,)
        h, hinfo = ops.hvp_from_potentials(X, X, a, X, r, c, T, 0.05, 3e-7, 1e-11, 100)
        assert h.shape == (100, 3) and hinfo.shape == (2,)
