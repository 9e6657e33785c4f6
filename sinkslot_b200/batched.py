"""Batches of independent SinkSLOT problems spread over the GPUs of a node.

Independent problems need no communication: each one is solved whole on one
GPU by ``sinkslot_solve``, and the GPUs work on their shares at the same time.

* One process driving several GPUs: problem i goes to ``devices[i % D]``; one
  host thread per device issues that device's solves on its own current stream
  (the library's calls release the GIL), and each result stays on the device
  that computed it.
* One process per GPU (``torch.distributed`` initialised): rank r solves the
  problems i with i % world == r on its current device and returns None in the
  other slots -- nothing is exchanged between the ranks.
"""

from __future__ import annotations

from concurrent.futures import ThreadPoolExecutor
from typing import Optional, Sequence

import torch

from .sinkhorn_solvers import SinkslotSolveResult, sinkslot_solve


def batch_assignment(n_problems: int, n_slots: int) -> list[list[int]]:
    """Problem indices per slot (device or rank): slot s takes s, s + D, s + 2D ..."""
    if n_slots < 1:
        raise ValueError("need at least one device")
    return [list(range(s, n_problems, n_slots)) for s in range(n_slots)]


def _unpack(p):
    if not isinstance(p, (tuple, list)) or len(p) not in (2, 4):
        raise TypeError("each problem is (X, Y) or (X, Y, a, b)")
    X, Y = p[0], p[1]
    a, b = (p[2], p[3]) if len(p) == 4 else (None, None)
    return X, Y, a, b


def _solve_on(device: torch.device, problem, kwargs) -> SinkslotSolveResult:
    X, Y, a, b = _unpack(problem)
    with torch.cuda.device(device):
        X = X.to(device, non_blocking=True)
        Y = Y.to(device, non_blocking=True)
        a = a.to(device, non_blocking=True) if a is not None else None
        b = b.to(device, non_blocking=True) if b is not None else None
        return sinkslot_solve(X, Y, a, b, **kwargs)


def sinkslot_solve_batched(problems: Sequence, *, devices: Optional[Sequence] = None,
                           **solve_kwargs) -> list[Optional[SinkslotSolveResult]]:
    """``sinkslot_solve`` for each of ``problems`` ((X, Y) or (X, Y, a, b)),
    spread over GPUs with no communication; ``solve_kwargs`` are
    ``sinkslot_solve``'s keyword arguments (eps, L, seed, n_iters, stop_mode,
    variant, ...).

    Without torch.distributed: ``devices`` (default: every visible GPU) each
    take every D-th problem; result i lives on the device that solved it.
    Under torch.distributed: this rank solves its share (i % world == rank) on
    its current device and the other entries are None.
    """
    if not torch.cuda.is_available():
        raise RuntimeError("sinkslot_solve_batched needs CUDA devices (there is no CPU path)")
    problems = list(problems)
    out: list[Optional[SinkslotSolveResult]] = [None] * len(problems)
    dist = torch.distributed
    if dist.is_available() and dist.is_initialized() and devices is None:
        mine = batch_assignment(len(problems), dist.get_world_size())[dist.get_rank()]
        dev = torch.device("cuda", torch.cuda.current_device())
        for i in mine:
            out[i] = _solve_on(dev, problems[i], solve_kwargs)
        return out
    if devices is None:
        devices = [torch.device("cuda", k) for k in range(torch.cuda.device_count())]
    devices = [torch.device(d) for d in devices]
    if any(d.type != "cuda" for d in devices):
        raise ValueError("devices must be CUDA devices")
    shares = batch_assignment(len(problems), len(devices))

    def run(slot: int):
        dev = devices[slot]
        for i in shares[slot]:
            out[i] = _solve_on(dev, problems[i], solve_kwargs)

    busy = [s for s in range(len(devices)) if shares[s]]
    if len(busy) <= 1:
        for s in busy:
            run(s)
        return out
    with ThreadPoolExecutor(max_workers=len(busy)) as ex:
        for f in [ex.submit(run, s) for s in busy]:
            f.result()  # re-raises a device's error
    return out
