"""Shared test configuration.

Markers: ``gpu`` -- needs a CUDA device (a B200 for the sm_100a library).
Everything unmarked runs on a CPU-only machine.
"""

from __future__ import annotations

import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def load_golden(name: str):
    z = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    meta = json.loads(str(z["meta"]))
    return meta, {k: z[k] for k in z.files if k != "meta"}


GOLDEN_CASES = ["small_nonuniform", "bench_shape", "cfg1", "unequal_ties", "zero_weights"]


def assert_close_np(got, want, rtol=1e-4, atol=1e-5, name=""):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    assert got.shape == want.shape, f"{name}: shape {got.shape} != {want.shape}"
    fin = np.isfinite(want)
    assert np.array_equal(np.isfinite(got), fin), f"{name}: non-finite pattern differs"
    assert np.array_equal(np.isnan(got), np.isnan(want)), f"{name}: NaN pattern differs"
    inf = np.isinf(want)
    assert np.array_equal(got[inf], want[inf]), f"{name}: infinities differ"
    d = np.abs(got[fin] - want[fin])
    bad = d > atol + rtol * np.abs(want[fin])
    assert not bad.any(), (f"{name}: {bad.sum()}/{bad.size} outside rtol={rtol} atol={atol}; "
                           f"max|d|={d.max():.3e}")


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O
    O.build()
    return O
