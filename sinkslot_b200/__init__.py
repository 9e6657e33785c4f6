"""sinkslot_b200: SinkSLOT's sparse Sinkhorn hot path as hand-written sm_100a CUDA.

Drop-in for the reference package's public API (cai4cai/SinkSLOT,
``torch-ext/sinkslot/__init__.py``): the same names, signatures and semantics,
backed by ``libsinkslot_b200.so`` (C ABI: ``include/sinkslot_b200.h``).
Inputs must be float32 CUDA tensors; there is no CPU or library fallback.
"""

from . import ops as _ops  # noqa: F401  (registers torch.ops.sinkslot_b200.*)
from .solver import (
    get_random_projections,
    sot_plan_coo,
    to_csr,
    sparse_sqeuclidean_cost,
)
from .sinkhorn_solvers import (
    seg_lse_online,
    launch_cfg,
    sinkslot_solve,
    sparse_transport_plan,
    SinkslotSolveResult,
)
from .gradient import (
    slot_grad,
    sparse_barycentric_map,
)
from .hvp import hvp_x_sqeuclid, hvp_x_sqeuclid_from_potentials
from .samples_loss import SamplesLoss
from .batched import sinkslot_solve_batched
from ._lib import LIB_PATH, SinkslotError, lib as load_library

__all__ = [
    "get_random_projections",
    "sot_plan_coo",
    "to_csr",
    "sparse_sqeuclidean_cost",
    "seg_lse_online",
    "launch_cfg",
    "sinkslot_solve",
    "sparse_transport_plan",
    "SinkslotSolveResult",
    "slot_grad",
    "sparse_barycentric_map",
    "hvp_x_sqeuclid",
    "hvp_x_sqeuclid_from_potentials",
    "SamplesLoss",
    "sinkslot_solve_batched",
    "SinkslotError",
    "LIB_PATH",
    "load_library",
]
