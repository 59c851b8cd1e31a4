"""Launch-grid inference (easy_as ``eas/runtime/grid.py:11-130``).

* 1D kernels: the thread count is ``_nthreads`` or the scalar argument ``N``;
  SPMD kernels launch ``ceil(N / BLOCK)`` programs, thread kernels launch
  exactly ``N`` threads (the last block may be partial).
* Kernels using ``program_id``/``thread_id`` on axis 1 (2D) or 2 (3D):
  ``(ceil(W / BLOCK), H, D)`` from ``_shape`` (last 2/3 dims) or from scalar
  arguments named ``H``, ``W`` and ``D``.
"""

from __future__ import annotations

from collections.abc import Mapping
from typing import Any

from ..ir import IRModule


def infer_nthreads(runtime_args: Mapping[str, Any], *, nthreads: int | None = None) -> int:
    if nthreads is None:
        if "N" not in runtime_args:
            raise ValueError("MVP runtime requires either `_nthreads=...` or a scalar argument named 'N' "
                             "for grid sizing")
        nthreads = int(runtime_args["N"])
    n = int(nthreads)
    if n < 0:
        raise ValueError("nthreads must be >= 0")
    return n


def _cdiv(a: int, b: int) -> int:
    return -(-a // b)


def infer_1d_grid(runtime_args: Mapping[str, Any], threadgroup_size: int, *, nthreads: int | None = None) -> int:
    n = infer_nthreads(runtime_args, nthreads=nthreads)
    if threadgroup_size <= 0:
        raise ValueError("threadgroup_size must be > 0")
    return _cdiv(n, threadgroup_size)


def grid_rank(ir: IRModule) -> int:
    """1 + the highest axis any program_id/thread_id uses (0 when none do)."""
    axes = [int(i.args[0]) for i in ir.insts if i.op in ("program_id", "thread_id")]
    return max(axes, default=-1) + 1


def infer_grid(ir: IRModule, runtime_args: Mapping[str, Any], threadgroup_size: int, *,
               shape: tuple[int, ...] | None = None, rank: int | None = None) -> tuple[int, int, int] | None:
    """``rank`` may pass a precomputed ``grid_rank(ir)`` (the runtime caches it per kernel)."""
    if rank is None:
        rank = grid_rank(ir)
    if rank <= 1:
        return None
    if rank > 3:
        raise ValueError("MVP runtime only supports 1D/2D/3D grids")
    if threadgroup_size <= 0:
        raise ValueError("threadgroup_size must be > 0")
    if shape is not None:
        if len(shape) < rank:
            raise ValueError(f"_shape must have >= {rank} dims for this kernel")
        dims = [int(x) for x in shape]
        if any(x < 0 for x in dims):
            raise ValueError("_shape dims must be >= 0")
        d, h, w = (1, dims[-2], dims[-1]) if rank == 2 else (dims[-3], dims[-2], dims[-1])
    else:
        need = ("H", "W") if rank == 2 else ("D", "H", "W")
        if any(k not in runtime_args for k in need):
            if rank == 2:
                raise ValueError("2D grid inference requires either `_shape=(H, W)` or scalar runtime args "
                                 "named 'H' and 'W' (or pass `_grid=...` explicitly)")
            raise ValueError("3D grid inference requires either `_shape=(D, H, W)` or scalar runtime args "
                             "named 'D', 'H', and 'W' (or pass `_grid=...` explicitly)")
        h, w = int(runtime_args["H"]), int(runtime_args["W"])
        d = int(runtime_args["D"]) if rank == 3 else 1
    if min(d, h, w) < 0:
        raise ValueError("shape dims must be >= 0")
    return (_cdiv(w, threadgroup_size) if w else 0, h, d)
