"""Near-miss variants of the fp16 ``mk.dot`` GEMM kernel (examples/matmul_dot_f16.py), for soundness
tests of the dot-GEMM pattern that routes it to the tcgen05 kernel.  ``MUT`` selects one change;
``DOT_MUTANTS`` lists (MUT, what changes, must the pattern decline).  A declined mutant runs the
generated kernel; an accepted one must compute what the mutant computes."""

from __future__ import annotations

import eas
from eas import mk

DOT_MUTANTS = [
    (0, "unchanged", False),
    (1, "A rows start one element later (A[m][k+1])", False),
    (2, "B rows at pitch N + 8", False),
    (3, "A read at k stride 2", True),
    (4, "dot over K // 2 terms", False),
    (5, "last row masked out of the store", False),
    (6, "C stored one element to the right", False),
    (7, "B columns at stride 2", True),
    (8, "A batches at stride M*K + 8", False),
    (9, "1.0 added to the dot before the store", True),
    (10, "dot scaled by 2 before the store", True),
    (11, "column index taken modulo 64", True),
]


@eas.kernel
def dot_mut(a, b, c, M, N, K, MUT: eas.constexpr, BLOCK_N: eas.constexpr = 256):
    col = mk.program_id(0) * BLOCK_N + mk.tid(0, BLOCK_N)
    if MUT == 11:
        col = col % 64
    row = mk.program_id(1)
    bat = mk.program_id(2)
    inside = (row < M) & (col < N)
    if MUT == 5:
        inside = (row + 1 < M) & (col < N)
    a_base = bat * (M * K + 8) + row * K if MUT == 8 else bat * (M * K) + row * K
    if MUT == 1:
        a_base = a_base + 1
    a_stride = 2 if MUT == 3 else 1
    ldb = N + 8 if MUT == 2 else N
    b_base = bat * (K * ldb) + (col * 2 if MUT == 7 else col)
    n_terms = mk.where(inside, K // 2 if MUT == 4 else K, 0)
    acc = mk.dot(a, a_base, a_stride, b, b_base, ldb, n_terms)
    if MUT == 9:
        acc = acc + 1.0
    if MUT == 10:
        acc = acc * 2.0
    c_off = bat * (M * N) + row * N + col + (1 if MUT == 6 else 0)
    mk.store(c, c_off, acc, inside)


def grid(batch, M, N, block_n=256):
    return (-(-N // block_n), M, batch)


def sizes(mut, batch, M, N, K):
    ldb = N + 8 if mut == 2 else N
    a = batch * (M * K + 8) + 2 * K + 8
    b = batch * K * ldb + 2 * N + 8
    return {"a": a, "b": b, "c": batch * M * N + 1}
