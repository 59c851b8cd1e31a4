"""Kernels that access memory outside their buffers, for the bounds-checked lowering
(EAS_BOUNDS_CHECK=1).  Each case names the buffer and the kind of the access the oracle reports
first; a checked kernel skips every such access and reports one of them.

``OOB_CASES``: (case id, kernel, args builder, meta, grid or None, buffer name or None for a
threadgroup allocation, "load" | "store")."""

from __future__ import annotations

import numpy as np

import eas
from eas import mk


@eas.kernel
def tail_load(a, b, c, N, BLOCK: eas.constexpr):
    """The load of ``a`` is unmasked: the last program reads past N."""
    offs = mk.program_id(0) * BLOCK + mk.arange(0, BLOCK)
    m = offs < N
    mk.store(c, offs, mk.load(a, offs, True) + mk.load(b, offs, m), m)


@eas.kernel
def tail_store(a, c, N, BLOCK: eas.constexpr):
    """The store to ``c`` is unmasked."""
    offs = mk.program_id(0) * BLOCK + mk.arange(0, BLOCK)
    mk.store(c, offs, mk.load(a, offs, offs < N), True)


@eas.kernel
def shifted_store(a, c, N, BLOCK: eas.constexpr):
    """Masked by ``offs < N`` but stored one element to the right: element N is written."""
    offs = mk.program_id(0) * BLOCK + mk.arange(0, BLOCK)
    m = offs < N
    mk.store(c, offs + 1, mk.load(a, offs, m), m)


@eas.kernel
def tg_overrun(x, y, N, BLOCK: eas.constexpr):
    """Each thread stages its element one slot to the right of a BLOCK-element threadgroup array."""
    t = mk.tid(0, BLOCK)
    s = mk.alloc_tg(BLOCK)
    g = mk.program_id(0) * BLOCK + t
    mk.store(s, t + 1, mk.load(x, g, g < N), True)
    mk.barrier()
    mk.store(y, g, mk.load(s, t, True), g < N)


@eas.kernel
def gemv_overrun(A, x, y, M, K, BLOCK: eas.constexpr):
    """y[r] = dot(row r of A, x) over K + 1 terms for the rows r < M: x[K] is read (A holds one
    spare element, so its reads stay inside)."""
    r = mk.program_id(0) * BLOCK + mk.tid(0, BLOCK)
    y_r = mk.dot(A, r * K, 1, x, 0, 1, mk.where(r < M, K + 1, 0))
    mk.store(y, r, y_r, r < M)


def _f32(n: int, seed: int) -> np.ndarray:
    return np.random.default_rng(seed).standard_normal(n).astype(np.float32)


OOB_CASES = [
    ("tail_load", tail_load, lambda: (_f32(1000, 1), _f32(1000, 2), np.zeros(1000, np.float32), 1000),
     {"BLOCK": 256}, None, "a", "load"),
    ("tail_store", tail_store, lambda: (_f32(1000, 3), np.zeros(1000, np.float32), 1000),
     {"BLOCK": 256}, None, "c", "store"),
    ("shifted_store", shifted_store, lambda: (_f32(1000, 4), np.zeros(1000, np.float32), 1000),
     {"BLOCK": 256}, None, "c", "store"),
    ("tg_overrun", tg_overrun, lambda: (_f32(64, 5), np.zeros(64, np.float32), 64),
     {"BLOCK": 32}, None, None, "store"),
    ("gemv_overrun", gemv_overrun, lambda: (_f32(8 * 16 + 1, 6), _f32(16, 7), np.zeros(8, np.float32), 8, 16),
     {"BLOCK": 32}, (1, 1, 1), "x", "load"),
]
