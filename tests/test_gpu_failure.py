"""Failure detection of the partitioned solve on one GPU, without a GPU fault.

Rank 0 of a two-rank partition runs against a peer that never publishes: its
potential buffers and flag words are plain local allocations that nothing
writes.  The bounded epoch wait must give up (about four seconds of clock),
the call must fail with a status naming the missing peer, and the CUDA context
must stay usable for the next solve.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_peer_that_never_publishes_fails_the_call_and_leaves_the_context_usable():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import sinkslot_b200
    from sinkslot_b200 import _lib, sinkslot_solve
    from sinkslot_b200._lib import SinkslotError, ptr, stream_of
    from sinkslot_b200.sharded import shard_bounds, slice_csr
    from sinkslot_b200.solver import cost_and_lam, sot_plan_coo, to_csr
    sinkslot_b200.load_library()
    dev = torch.device("cuda:0")
    g = torch.Generator().manual_seed(4)
    n = m = 2000
    x = torch.randn(n, 3, generator=g).to(dev)
    y = (torch.randn(m, 3, generator=g) + 1.0).to(dev)
    a = torch.full((n,), 1.0 / n, device=dev)
    rows, cols, S = sot_plan_coo(x, y, a, a, L=16, seed=0)
    lam, _ = cost_and_lam(x, y, rows, cols, S, 0.05)
    r_ptr, r_idx, r_lam, _ = to_csr(rows, cols, lam, n)
    c_ptr, c_idx, c_lam, _ = to_csr(cols, rows, lam, m)
    world, rank = 2, 0
    r0, nr = shard_bounds(n, world, rank)
    c0, nc = shard_bounds(m, world, rank)
    lr = slice_csr(r_ptr, r_idx, r_lam, r0, nr)
    lc = slice_csr(c_ptr, c_idx, c_lam, c0, nc)
    # both "ranks'" buffers are local; the absent peer's are never written by it
    phi = [torch.zeros(n, device=dev) for _ in range(world)]
    psi = [torch.zeros(m, device=dev) for _ in range(world)]
    flags = [torch.zeros(world, dtype=torch.int32, device=dev) for _ in range(world)]
    phi_p = (ctypes.c_void_p * (2 * world))(phi[0].data_ptr(), None, phi[1].data_ptr(), None)
    psi_p = (ctypes.c_void_p * (2 * world))(psi[0].data_ptr(), None, psi[1].data_ptr(), None)
    flag_p = (ctypes.c_void_p * world)(flags[0].data_ptr(), flags[1].data_ptr())
    wf = _lib.out_i64()
    _lib.call("sinkslot_shard_work_floats", nr, nc, ctypes.byref(wf))
    work = torch.empty(wf.value, device=dev)
    cur, epoch = ctypes.c_int(0), ctypes.c_uint32(0)
    ch0, ch1 = ctypes.c_double(0.0), ctypes.c_double(0.0)
    log_a = a.log()
    with pytest.raises(SinkslotError, match="did not publish"):
        _lib.call("sinkslot_solve_shard", ptr(lr[0]), ptr(lr[1]), lr[1].element_size(), ptr(lr[2]),
                  lr[3], r0, nr, None, 0, ptr(lc[0]), ptr(lc[1]), lc[1].element_size(),
                  ptr(lc[2]), lc[3], c0, nc, None, 0, ptr(log_a), ptr(log_a), n, m, 0, 0.5,
                  rank, world, phi_p, psi_p, flag_p, 0, 2, 0, ctypes.byref(cur),
                  ctypes.byref(epoch), ptr(work), work.numel(), ctypes.byref(ch0),
                  ctypes.byref(ch1), stream_of(dev))
    # rank 0 did publish its own epochs into the absent peer's flag words
    assert int(flags[1][rank]) >= 1
    # the context is intact: a normal solve runs and is finite
    torch.cuda.synchronize()
    res = sinkslot_solve(x, y, a, a, 0.05, 16, 0, 20)
    assert torch.isfinite(res.phi).all() and torch.isfinite(res.psi).all()
