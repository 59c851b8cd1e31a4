"""SPMD kernels with loops over constexpr ranges (this repository's own DSL code), for the
re-rolling tests: a column sum (carried lane vector) and a row-by-row copy (a store per step)."""

import eas
from eas import mk


@eas.kernel
def colsum(x, y, N, W: eas.constexpr, BLOCK: eas.constexpr):
    offs = mk.program_id(0) * BLOCK + mk.arange(0, BLOCK)
    m = offs < N
    acc = mk.load(x, offs, m)
    for j in range(1, W):
        acc = acc + mk.load(x, offs + j * N, m)
    mk.store(y, offs, acc, m)


@eas.kernel
def rows_scale(x, y, N, W: eas.constexpr, BLOCK: eas.constexpr):
    offs = mk.program_id(0) * BLOCK + mk.arange(0, BLOCK)
    m = offs < N
    for j in range(W):
        mk.store(y, offs + j * N, mk.load(x, offs + j * N, m) * 2.0 + 1.0, m)
