"""The reference-side edit that makes ``backend="auto"`` select sinkslot_b200 on
CUDA float32 tensors -- the dispatch a maintainer adds to the reference's
``sinkslot/sinkhorn_solvers.py`` (the patch shown in the integration notes),
applied here to a copy of an installed reference package for the tests.

Three edits, each anchored on a line of the reference's dispatcher:
1. after ``import torch``: try to import sinkslot_b200 and load its library;
2. the accepted backend names (``sinkslot_solve``'s first check) gain "b200";
3. before the backend resolution (``if backend == "triton":`` inside
   ``sinkslot_solve``): "b200", or "auto" with the library present and X a CUDA
   float32 tensor, returns ``sinkslot_b200.sinkslot_solve(...)``'s fields as
   the reference's own ``SinkslotSolveResult`` (its return annotation is
   checked at run time).
"""

from __future__ import annotations

import os
import shutil

IMPORT_BLOCK = '''
try:
    import sinkslot_b200 as _b200
    _b200.load_library()          # raises if libsinkslot_b200.so is missing
    _HAS_B200 = True
except Exception:
    _HAS_B200 = False
'''

DISPATCH_BLOCK = '''    if backend == "b200" or (backend == "auto" and _HAS_B200 and X.is_cuda
                             and X.dtype == torch.float32):
        return SinkslotSolveResult(*_b200.sinkslot_solve(
            X, Y, a, b, eps, L, seed, n_iters, stop_mode=stop_mode,
            stop_max_iter=stop_max_iter, stop_tol=stop_tol,
            stop_check_every=stop_check_every, chunk=chunk, variant=variant,
            alpha=alpha))
'''


def patch_source(src: str) -> str:
    lines = src.splitlines(keepends=True)
    out, in_solve, imported, names, dispatched = [], False, False, False, False
    for ln in lines:
        if ln.startswith("def sinkslot_solve("):
            in_solve = True
        elif ln.startswith("def ") and in_solve:
            in_solve = False
        if in_solve and not names and ln.strip().startswith("if backend not in ("):
            ln = ln.replace('("auto", "triton", "torch")', '("auto", "triton", "torch", "b200")')
            names = True
        if in_solve and not dispatched and ln.startswith('    if backend == "triton":'):
            out.append(DISPATCH_BLOCK)
            dispatched = True
        out.append(ln)
        if not imported and ln.strip() == "import torch":
            out.append(IMPORT_BLOCK)
            imported = True
    if not (imported and names and dispatched):
        raise RuntimeError("the reference's dispatcher did not match the expected anchors")
    return "".join(out)


def patched_copy(ref_root: str, dest: str) -> str:
    """Copies the ``sinkslot`` package under ref_root to dest, patches its
    dispatcher, and returns the directory to put on sys.path."""
    target = os.path.join(dest, "sinkslot")
    shutil.copytree(os.path.join(ref_root, "sinkslot"), target)
    path = os.path.join(target, "sinkhorn_solvers.py")
    with open(path) as f:
        src = f.read()
    with open(path, "w") as f:
        f.write(patch_source(src))
    return dest
