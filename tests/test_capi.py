"""The C ABI (include/*.h) against the built library, without a GPU: every
declared entry point is exported, the Python binding covers it, and host-only
calls (workspace sizing, argument checks) behave."""

from __future__ import annotations

import ctypes
import glob
import os
import re

import pytest

from conftest import ROOT

HEADERS = sorted(glob.glob(os.path.join(ROOT, "include", "*.h")))


def declared_functions():
    names = []
    for h in HEADERS:
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        names += re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(sinkslot_\w+)\s*\(", src, flags=re.M)
    return sorted(set(names))


@pytest.fixture(scope="module")
def lib():
    from sinkslot_b200 import build
    build.build()
    from sinkslot_b200 import _lib
    return _lib.lib()


def test_header_declares_entry_points():
    names = declared_functions()
    assert len(names) >= 15
    assert "sinkslot_solve_csr" in names and "sinkslot_build_support" in names


def test_library_exports_every_declared_symbol(lib):
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, f"not exported: {missing}"


def test_python_binding_covers_every_compute_entry_point():
    from sinkslot_b200 import _lib
    extra = {"sinkslot_last_error", "sinkslot_abi_version"}
    for n in declared_functions():
        assert n in _lib._SIGNATURES or n in extra, f"{n} has no ctypes signature"


def test_abi_version_and_error_channel(lib):
    assert lib.sinkslot_abi_version() >= 100
    out = ctypes.c_int64(0)
    st = lib.sinkslot_support_workspace_bytes(0, 10, 3, 8, 0, ctypes.byref(out))
    assert st == 1
    assert b"bad args" in lib.sinkslot_last_error()
    st = lib.sinkslot_support_workspace_bytes(1000, 800, 3, 8, 0, ctypes.byref(out))
    assert st == 0 and out.value > 8 * (1000 + 800) * 12
    assert lib.sinkslot_last_error() == b""


def test_workspace_sizes_scale(lib):
    a, b = ctypes.c_int64(0), ctypes.c_int64(0)
    assert lib.sinkslot_support_workspace_bytes(1 << 16, 1 << 16, 3, 64, 0, ctypes.byref(a)) == 0
    assert lib.sinkslot_support_workspace_bytes(1 << 16, 1 << 16, 3, 64, 8, ctypes.byref(b)) == 0
    assert b.value < a.value  # chunking bounds the per-batch sort buffers
    f = ctypes.c_int64(0)
    assert lib.sinkslot_solve_work_floats(100, 50, ctypes.byref(f)) == 0
    assert f.value >= 2 * 150
    assert lib.sinkslot_csr_workspace_bytes(1000, 10, ctypes.byref(f)) == 0 and f.value > 4000
    assert lib.sinkslot_barycentric_workspace_bytes(100, 10, 20, 3, ctypes.byref(f)) == 0


def test_null_arguments_rejected_without_touching_a_device(lib):
    nnz = ctypes.c_int64(0)
    st = lib.sinkslot_build_support(None, None, None, None, 10, 10, 3, None, None, None, 4, 0,
                                    None, 0, ctypes.byref(nnz), None)
    assert st == 1 and b"null" in lib.sinkslot_last_error()


def _align256(x):
    return (x + 255) // 256 * 256


def test_tiles_kind_policy_and_geometry(lib):
    """The tiled kind per side: staged while staging the gathered potential
    (P panels x m_other x 4 bytes) costs at most 4x the entry stream (nnz x 8
    bytes), else two-pass; the setting is process-wide and validated; a
    two-pass layout is the staged one plus four per-slot arrays, its panels up
    to 16383 rows (host logic only, no device work; 148 SMs assumed here)."""
    kind = ctypes.c_int(-1)
    geom = (ctypes.c_int * 5)()
    assert lib.sinkslot_get_tiles_kind(ctypes.byref(kind)) == 0 and kind.value == 0
    try:
        for log2n, want in [(20, 1), (21, 1), (22, 2), (24, 2)]:
            n = 1 << log2n
            nnz = 64 * n
            assert lib.sinkslot_tiles_geometry(n, n, nnz, geom) == 0
            P = geom[0]
            assert lib.sinkslot_tiles_kind_of(n, n, nnz, ctypes.byref(kind)) == 0
            assert kind.value == want, (log2n, kind.value)
            # the rule itself, on the staged geometry
            assert lib.sinkslot_set_tiles_kind(1) == 0
            assert lib.sinkslot_tiles_geometry(n, n, nnz, geom) == 0
            staged_P = geom[0]
            assert (staged_P * n * 4 <= 4 * nnz * 8) == (want == 1)
            assert lib.sinkslot_set_tiles_kind(0) == 0
            del P
        # a forced kind, its geometry and the layout bytes
        n, m, nnz = 1 << 20, 1 << 20, 64 << 20
        sizes = {}
        for k in (1, 2):
            assert lib.sinkslot_set_tiles_kind(k) == 0
            lb, bb = ctypes.c_int64(0), ctypes.c_int64(0)
            assert lib.sinkslot_tiles_bytes(n, m, nnz, ctypes.byref(lb), ctypes.byref(bb)) == 0
            assert lib.sinkslot_tiles_geometry(n, m, nnz, geom) == 0
            P, R, B, logW, smem = list(geom)
            assert P * R >= n and R + 1 <= (16384 if k == 2 else 8320) and smem <= 227 * 1024
            cap = nnz + 63 * P * B
            staged = _align256(64) + _align256(8 * (P * B + 1)) + _align256(8 * cap)
            extra = 2 * _align256(2 * cap) + 2 * _align256(4 * cap) if k == 2 else 0
            assert lb.value == staged + extra
            sizes[k] = (P, R, B, logW)
        # the two-pass kind keeps the blocks and takes longer panels
        assert sizes[2][2:] == sizes[1][2:] and sizes[2][1] >= sizes[1][1]
        assert lib.sinkslot_set_tiles_kind(3) == 1 and b"kind" in lib.sinkslot_last_error()
    finally:
        lib.sinkslot_set_tiles_kind(0)
