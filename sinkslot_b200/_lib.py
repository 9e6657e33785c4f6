"""ctypes binding of libsinkslot_b200.so (the C ABI in include/sinkslot_b200.h).

PyTorch provides device memory, the current stream and the device guard; every
computation runs in the library's sm_100a kernels.  A missing or unloadable
library is an error: there is no fallback path.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libsinkslot_b200.so")

_lock = threading.Lock()
_lib = None

c_i64 = ctypes.c_int64
c_int = ctypes.c_int
c_dbl = ctypes.c_double
c_vp = ctypes.c_void_p
P_i64 = ctypes.POINTER(ctypes.c_int64)
P_int = ctypes.POINTER(ctypes.c_int)
P_dbl = ctypes.POINTER(ctypes.c_double)

# name -> argtypes (every entry point returns int status)
_SIGNATURES = {
    "sinkslot_project": [c_vp, c_i64, c_int, c_vp, c_int, c_vp, c_vp],
    "sinkslot_ot1d_workspace_bytes": [c_i64, c_i64, c_int, P_i64],
    "sinkslot_ot1d_batched": [c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_int, c_int, c_vp, c_i64, c_vp,
                              c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, P_i64, c_vp],
    "sinkslot_support_workspace_bytes": [c_i64, c_i64, c_int, c_int, c_int, P_i64],
    "sinkslot_build_support": [c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_int, c_vp, c_vp, c_vp,
                               c_int, c_int, c_vp, c_i64, P_i64, c_vp],
    "sinkslot_support_export": [c_vp, c_i64, c_i64, c_i64, c_int, c_int, c_int, c_i64, c_vp, c_vp,
                                c_vp, c_vp],
    "sinkslot_partition_workspace_bytes": [c_i64, P_i64],
    "sinkslot_partition_coo": [c_vp, c_vp, c_vp, c_i64, P_i64, c_int, c_vp, c_i64, c_vp, c_vp,
                               c_vp, P_i64, c_vp],
    "sinkslot_coalesce_workspace_bytes": [c_i64, P_i64],
    "sinkslot_coalesce_coo": [c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_int, c_vp, c_i64, c_vp,
                              c_vp, c_vp, P_i64, c_vp],
    "sinkslot_csr_workspace_bytes": [c_i64, c_i64, P_i64],
    "sinkslot_coo_to_csr": [c_vp, c_vp, c_vp, c_i64, c_i64, c_int, c_vp, c_i64, c_vp, c_vp, c_vp,
                            c_vp, P_int, c_vp],
    "sinkslot_max_index": [c_vp, c_i64, c_vp, P_i64, c_vp],
    "sinkslot_cost_lam": [c_vp, c_vp, c_int, c_vp, c_vp, c_vp, c_i64, c_dbl, c_vp, c_vp, c_vp],
    "sinkslot_seg_lse": [c_vp, c_vp, c_int, c_vp, c_i64, c_vp, c_vp, c_vp, c_i64, c_vp, c_vp],
    "sinkslot_solve_work_floats": [c_i64, c_i64, P_i64],
    "sinkslot_solve_csr": [c_vp, c_vp, c_int, c_vp, c_vp, c_vp, c_int, c_vp, c_i64, c_vp, c_vp,
                           c_i64, c_i64, c_int, c_int, c_i64, c_i64, c_i64, c_dbl, c_dbl, c_dbl,
                           c_vp, c_i64, c_vp, c_i64,
                           c_vp, c_vp, c_vp, c_i64, P_i64, P_int, P_dbl, c_vp],
    "sinkslot_solve_csr_static": [c_vp, c_vp, c_int, c_vp, c_vp, c_vp, c_int, c_vp, c_i64, c_vp,
                                  c_vp, c_i64, c_i64, c_int, c_int, c_i64, c_i64, c_i64, c_dbl,
                                  c_dbl, c_dbl, c_vp, c_i64, c_vp, c_i64,
                                  c_vp, c_vp, P_i64, P_int, P_dbl, c_vp],
    "sinkslot_ipc_export": [c_vp, c_vp, P_i64],
    "sinkslot_ipc_import": [c_vp, c_i64, ctypes.POINTER(c_vp)],
    "sinkslot_ipc_close": [c_vp, c_i64],
    "sinkslot_shard_work_floats": [c_i64, c_i64, P_i64],
    "sinkslot_solve_shard": [c_vp, c_vp, c_int, c_vp, c_i64, c_i64, c_i64, c_vp, c_i64,
                             c_vp, c_vp, c_int, c_vp, c_i64, c_i64, c_i64, c_vp, c_i64,
                             c_vp, c_vp, c_i64, c_i64, c_int, c_dbl, c_int, c_int,
                             c_vp, c_vp, c_vp, c_i64, c_i64, c_int, P_int,
                             ctypes.POINTER(ctypes.c_uint32), c_vp, c_i64, P_dbl, P_dbl, c_vp],
    "sinkslot_tiles_bytes": [c_i64, c_i64, c_i64, P_i64, P_i64],
    "sinkslot_tiles_geometry": [c_i64, c_i64, c_i64, P_int],
    "sinkslot_set_tiles_kind": [c_int],
    "sinkslot_get_tiles_kind": [P_int],
    "sinkslot_tiles_kind_of": [c_i64, c_i64, c_i64, P_int],
    "sinkslot_build_tiles": [c_vp, c_vp, c_int, c_vp, c_i64, c_i64, c_i64, c_vp, c_i64, c_vp,
                             c_i64, c_vp],
    "sinkslot_plan_values": [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_i64, c_dbl, c_int,
                             c_vp, c_vp],
    "sinkslot_barycentric_workspace_bytes": [c_i64, c_i64, c_i64, c_int, P_i64],
    "sinkslot_barycentric": [c_vp, c_vp, c_vp, c_i64, c_vp, c_vp, c_i64, c_i64, c_int, c_vp, c_vp,
                             c_vp, c_vp, c_vp, c_i64, c_vp],
    "sinkslot_dual_value": [c_vp, c_vp, c_i64, c_vp, c_vp, c_i64, c_vp, c_vp],
    "sinkslot_hvp_workspace_bytes": [c_i64, c_i64, P_i64],
    "sinkslot_hvp": [c_vp, c_vp, c_int, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_int,
                     c_i64, c_i64, c_dbl, c_dbl, c_dbl, c_i64, c_vp, c_i64, c_vp, c_vp, P_i64,
                     P_dbl, c_vp],
}


class SinkslotError(RuntimeError):
    """A call into libsinkslot_b200.so failed (CUDA error or bad argument)."""


def lib():
    """The loaded library; raises if it is missing (no fallback exists)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: the sm_100a extension must be built "
                f"(python -m sinkslot_b200.build); sinkslot_b200 has no CPU or library fallback")
        L = ctypes.CDLL(LIB_PATH)
        for name, argtypes in _SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = argtypes
            fn.restype = c_int
        L.sinkslot_last_error.argtypes = []
        L.sinkslot_last_error.restype = ctypes.c_char_p
        L.sinkslot_abi_version.argtypes = []
        L.sinkslot_abi_version.restype = c_int
        _lib = L
    return _lib


def call(name: str, *args) -> None:
    """Invoke an entry point; map a nonzero status to an exception."""
    L = lib()
    st = getattr(L, name)(*args)
    if st != 0:
        msg = L.sinkslot_last_error().decode(errors="replace")
        if st == 1:
            raise ValueError(f"{name}: {msg}")
        raise SinkslotError(f"{name} failed (status {st}): {msg}")


def ptr(t) -> int | None:
    """Device pointer of a tensor (None for None / empty tensors)."""
    if t is None:
        return None
    if t.numel() == 0:
        return None
    return t.data_ptr()


def stream_of(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def out_i64() -> ctypes.c_int64:
    return ctypes.c_int64(0)
