"""Support construction on the GPU: bit-exact against the oracle and against the
reference's own torch-op sequence executed on the same CUDA device.

Covers projection (vs the CPU FMA chain and vs cuBLAS), the per-slice argsort
(vs torch.argsort on CUDA, including exact ties), the cumsum association order
(vs torch.cumsum on CUDA), the merged 1-D couplings, the coalesced support and
COO -> CSR.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import GOLDEN_CASES, load_golden

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cuda():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    torch.backends.cuda.matmul.allow_tf32 = False
    import sinkslot_b200
    sinkslot_b200.load_library()
    return torch.device("cuda:0")


def _points(n, d, seed, shift=0.0, dup=1):
    g = torch.Generator().manual_seed(seed)
    base = torch.randn((n + dup - 1) // dup, d, generator=g) + shift
    x = base.repeat(dup, 1)[:n]
    return x[torch.randperm(n, generator=g)].contiguous()


def _weights(n, seed, kind):
    g = torch.Generator().manual_seed(seed)
    if kind == "uniform":
        return torch.full((n,), 1.0 / n)
    w = -torch.log(torch.rand(n, generator=g).clamp_min(1e-12))  # Dirichlet(1)
    return (w / w.sum()).float()


@pytest.mark.parametrize("n,d,L,same_as_cublas", [(1000, 3, 64, True), (4097, 2, 8, True),
                                                  (65536, 4, 16, True), (3, 5, 3, False)])
def test_projection_bits(cuda, oracle, n, d, L, same_as_cublas):
    """The C ABI's own projection (theta given, no precomputed projections) is
    the sequential FMA chain: bit-equal to the oracle always, and to cuBLAS's
    `X @ theta.T` for the d <= 4 shapes of the workloads.  cuBLAS rounds some
    other shapes differently (d = 5, n = 3 here), which is why the Python layer
    hands the support builder cuBLAS's projections, as the reference computes
    them."""
    from sinkslot_b200.solver import get_random_projections, project
    X = _points(n, d, 1)
    th = get_random_projections(d, L, 7).float()
    got = project(X.to(cuda), th.to(cuda)).cpu().numpy()
    np.testing.assert_array_equal(got, oracle.project(X.numpy(), th.numpy()))
    cublas = (X.to(cuda) @ th.to(cuda).T).T.contiguous().cpu().numpy()
    if same_as_cublas:
        np.testing.assert_array_equal(got, cublas)


@pytest.mark.parametrize("n,d,L,chunk", [
    (10000, 2, 64, None),        # the CPU-runnable configuration's shape
    (1 << 18, 2, 100, None),     # gradient flow
    (1 << 20, 3, 64, None),      # the headline
    (1 << 20, 3, 64, 8),         # chunked GEMMs
    (1 << 21, 3, 128, None),     # colour-transfer source cloud
    (1 << 24, 3, 64, 8),         # scale-out
    (100003, 4, 48, 5),
])
def test_own_projection_equals_cublas_at_workload_shapes(cuda, n, d, L, chunk):
    """For d <= 4 the support builder projects with its own FMA-chain kernel
    instead of materialising cuBLAS's `X @ theta.T`: bit-equal to cuBLAS's
    product at every workload shape, chunk by chunk as the reference issues it
    (solver.py:219-221)."""
    from sinkslot_b200.solver import get_random_projections, project
    X = _points(n, d, 2).to(cuda)
    th = get_random_projections(d, L, 0).float().to(cuda)
    got = project(X, th)
    step = L if chunk is None else chunk
    for s in range(0, L, step):
        want = (X @ th[s:s + step].T).T
        assert torch.equal(got[s:s + step], want), f"slices {s}..{s + step} differ from cuBLAS"
    del got


def test_support_uses_the_reference_gemm_bits(cuda):
    """d = 5 with few points, where cuBLAS's rounding differs from the FMA
    chain: the support still equals the reference op sequence on this device."""
    from oracle.torch_ref import sot_plan_coo as ref_plan
    from sinkslot_b200 import sot_plan_coo
    from sinkslot_b200.solver import get_random_projections
    for n, m in ((3, 4), (40, 33)):
        X, Y = _points(n, 5, 21).to(cuda), _points(m, 5, 22, shift=0.3).to(cuda)
        a, b = _weights(n, 23, "dirichlet").to(cuda), _weights(m, 24, "dirichlet").to(cuda)
        rows, cols, S = sot_plan_coo(X, Y, a, b, L=3, seed=1)
        r2, c2, S2 = ref_plan(X, Y, a, b, get_random_projections(5, 3, 1).float().to(cuda))
        assert torch.equal(rows, r2) and torch.equal(cols, c2)
        torch.testing.assert_close(S, S2, rtol=1e-6, atol=1e-12)


@pytest.mark.parametrize("n,m,C,kind,dup", [
    (3000, 2000, 7, "dirichlet", 1),     # torch's in-block sort path (<= 4096)
    (50000, 40000, 5, "dirichlet", 1),   # torch's segmented radix sort path
    (20000, 20000, 64, "uniform", 1),
    (30000, 25000, 9, "dirichlet", 3),   # every point present 3 times: exact ties
    (100, 4100, 2, "dirichlet", 2),
])
def test_ot1d_matches_torch_cuda_ops(cuda, oracle, n, m, C, kind, dup):
    from oracle.torch_ref import ot1d_cuda_builder
    from sinkslot_b200.solver import _ot_1d_coo_batched_cuda, get_random_projections
    X = _points(n, 3, 2, dup=dup)
    Y = _points(m, 3, 3, shift=1.0, dup=dup)
    th = get_random_projections(3, C, 0).float().to(cuda)
    PX, PY = X.to(cuda) @ th.T, Y.to(cuda) @ th.T
    a = _weights(n, 4, kind).to(cuda)
    b = _weights(m, 5, kind).to(cuda)
    R, Cc, M, ix, iy, ca, cb = _ot_1d_coo_batched_cuda(PX, PY, a, b, return_intermediates=True)
    tR, tC, tM, tix, tiy, tca, tcb = ot1d_cuda_builder(PX, PY, a, b, return_intermediates=True)
    assert torch.equal(ix.long(), tix) and torch.equal(iy.long(), tiy), "argsort differs"
    assert torch.equal(ca, tca) and torch.equal(cb, tcb), "cumsum bits differ"
    assert torch.equal(R, tR) and torch.equal(Cc, tC) and torch.equal(M, tM)
    oR, oC, oM = oracle.ot1d(PX.T.contiguous().cpu().numpy(), PY.T.contiguous().cpu().numpy(),
                             a.cpu().numpy(), b.cpu().numpy(), builder="cuda")
    np.testing.assert_array_equal(R.cpu().numpy(), oR)
    np.testing.assert_array_equal(Cc.cpu().numpy(), oC)
    np.testing.assert_array_equal(M.cpu().numpy(), oM)


@pytest.mark.parametrize("case", GOLDEN_CASES)
def test_support_matches_oracle_on_golden_inputs(cuda, oracle, case):
    from sinkslot_b200 import sot_plan_coo
    meta, g = load_golden(case)
    t = [torch.from_numpy(g[k]).to(cuda) for k in ("x", "y", "a", "b")]
    rows, cols, S = sot_plan_coo(*t, L=meta["L"], seed=0)
    orow, ocol, oS = oracle.sot_plan_coo(g["x"], g["y"], g["a"], g["b"], meta["L"], 0,
                                         builder="cuda")
    np.testing.assert_array_equal(rows.cpu().numpy(), orow)
    np.testing.assert_array_equal(cols.cpu().numpy(), ocol)
    np.testing.assert_array_equal(S.cpu().numpy(), oS)


@pytest.mark.parametrize("chunk", [None, 5])
def test_support_matches_torch_cuda_ops_nonuniform(cuda, chunk):
    """n != m, Dirichlet weights, chunked and one-shot: rows/cols bit-exact with
    the reference's op sequence on this device; S to fp32 rounding (the
    reference sums duplicates with order-free atomics)."""
    from oracle.torch_ref import sot_plan_coo as ref_plan
    from sinkslot_b200 import sot_plan_coo
    from sinkslot_b200.solver import get_random_projections
    n, m, L = 1 << 15, 1 << 14, 24
    X, Y = _points(n, 3, 11).to(cuda), _points(m, 3, 12, shift=0.5).to(cuda)
    a, b = _weights(n, 13, "dirichlet").to(cuda), _weights(m, 14, "dirichlet").to(cuda)
    rows, cols, S = sot_plan_coo(X, Y, a, b, L=L, seed=3, chunk=chunk)
    th = get_random_projections(3, L, 3).float().to(cuda)
    r2, c2, S2 = ref_plan(X, Y, a, b, th, chunk=chunk)
    assert torch.equal(rows, r2) and torch.equal(cols, c2)
    torch.testing.assert_close(S, S2, rtol=1e-6, atol=1e-12)


def test_support_full_size_uniform_matches_torch_cuda_ops(cuda):
    """N = M = 2^20, d = 3, L = 64, x ~ N(0, I), y ~ N(0, I) + 1.5 (seed 1): the
    single-GPU headline problem.  Uniform power-of-two weights make every mass
    and sum exact, so S must match bit for bit as well."""
    from oracle.torch_ref import sot_plan_coo as ref_plan
    from sinkslot_b200 import sot_plan_coo
    from sinkslot_b200.solver import get_random_projections
    torch.manual_seed(1)
    n = 1 << 20
    X = torch.randn(n, 3).to(cuda)
    Y = (torch.randn(n, 3) + 1.5).to(cuda)
    a = torch.full((n,), 1.0 / n, device=cuda)
    rows, cols, S = sot_plan_coo(X, Y, a, a, L=64, seed=0)
    th = get_random_projections(3, 64, 0).float().to(cuda)
    r2, c2, S2 = ref_plan(X, Y, a, a, th)
    assert rows.numel() == r2.numel()
    assert torch.equal(rows, r2) and torch.equal(cols, c2)
    assert torch.equal(S, S2)
    # size-independent properties: sorted unique keys, row sums of S = a
    key = rows * n + cols
    assert bool((key[1:] > key[:-1]).all())
    rs = torch.zeros(n, device=cuda, dtype=torch.float64).index_add_(0, rows, S.double())
    torch.testing.assert_close(rs, a.double(), rtol=0, atol=1e-12)


@pytest.mark.parametrize("sorted_rows", [True, False])
@pytest.mark.parametrize("nseg,nnz,maxidx", [(1000, 20000, 30000), (70000, 500000, 1 << 20),
                                             (5, 0, 10)])
def test_to_csr_matches_oracle(cuda, oracle, sorted_rows, nseg, nnz, maxidx):
    from sinkslot_b200 import to_csr
    g = torch.Generator().manual_seed(nseg + nnz)
    rows = torch.randint(0, nseg, (nnz,), generator=g)
    if sorted_rows:
        rows, _ = torch.sort(rows)
    cols = torch.randint(0, maxidx, (nnz,), generator=g)
    vals = torch.randn(nnz, generator=g)
    ptr, idx, v, perm = to_csr(rows.to(cuda), cols.to(cuda), vals.to(cuda), nseg)
    optr, oidx, ov, operm = oracle.to_csr(rows.numpy(), cols.numpy(), vals.numpy(), nseg)
    np.testing.assert_array_equal(ptr.cpu().numpy(), optr)
    assert idx.dtype == {np.int16: torch.int16, np.int32: torch.int32}[oidx.dtype.type]
    np.testing.assert_array_equal(idx.cpu().numpy(), oidx)
    np.testing.assert_array_equal(v.cpu().numpy(), ov)
    assert (perm is None) == (operm is None)
    if perm is not None:
        np.testing.assert_array_equal(perm.cpu().numpy(), operm)


@pytest.mark.parametrize("sorted_rows", [True, False])
@pytest.mark.parametrize("nseg,nnz,maxidx", [(1000, 20000, 30000), (70000, 500000, 1 << 20),
                                             (5, 0, 10), (3, 1, 7)])
def test_csr_without_permutation_matches_oracle(cuda, oracle, sorted_rows, nseg, nnz, maxidx):
    """The solve's CSR/CSC path (no permutation formed; the sort carries index
    and value) gives the same arrays as to_csr."""
    from sinkslot_b200.solver import _to_csr
    g = torch.Generator().manual_seed(7 * nseg + nnz)
    rows = torch.randint(0, nseg, (nnz,), generator=g)
    if sorted_rows:
        rows, _ = torch.sort(rows)
    cols = torch.randint(0, maxidx, (nnz,), generator=g)
    vals = torch.randn(nnz, generator=g)
    vals[::97] = -float("inf")
    ptr, idx, v, perm = _to_csr(rows.to(cuda), cols.to(cuda), vals.to(cuda), nseg, want_perm=False)
    assert perm is None
    optr, oidx, ov, _ = oracle.to_csr(rows.numpy(), cols.numpy(), vals.numpy(), nseg)
    np.testing.assert_array_equal(ptr.cpu().numpy(), optr)
    assert idx.dtype == {np.int16: torch.int16, np.int32: torch.int32}[oidx.dtype.type]
    np.testing.assert_array_equal(idx.cpu().numpy(), oidx)
    np.testing.assert_array_equal(v.cpu().numpy().view(np.uint32), ov.view(np.uint32))
