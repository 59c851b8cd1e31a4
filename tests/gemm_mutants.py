"""Near-miss variants of a tiled fp32 matmul, for soundness tests of the tiled-GEMM proof.

``tile_mm_mut`` is the tiled kernel of ``tiled_variants.tile_mm`` with one change selected by
the constexpr ``MUT``.  Some mutants are still GEMMs in another layout (the proof may accept
them, and then the native kernel must compute exactly what they compute); the others are not
GEMMs (the proof must decline, and the generated kernel runs).  Either way the result must be
the oracle's, bit for bit.  ``MUTANTS`` lists (MUT, what changes, must the proof decline).
"""

from __future__ import annotations

import eas
from eas import mk

MUTANTS = [
    (0, "unchanged", False),
    (1, "A rows read one row further down (A[m+1])", False),
    (2, "B columns read with stride 2 (B[k][2n])", True),
    (3, "A's k slots rotated by one within each staged row", True),
    (4, "partial sums multiplied into the accumulator instead of added", True),
    (5, "dot over TK-1 of each tile's TK slots (skips one k per tile)", False),
    (6, "K loop starts at the second tile", False),
    (7, "A masked one row early (last row reads zeros)", False),
    (8, "C stored one column to the right", False),
    (9, "B read transposed from its own layout (B[n][k] of an N x K buffer)", False),
    (10, "accumulator starts from a loaded value instead of zero", True),
    (11, "two dots per tile into the same output (each k counted twice)", False),
]


@eas.kernel
def tile_mm_mut(a, b, c, M, N, K: eas.constexpr, MUT: eas.constexpr):
    TM, TN, TK, NT = 32, 32, 16, 128
    t = mk.tid(0, NT)
    row0 = mk.program_id(1) * TM
    col0 = mk.program_id(0) * TN
    lda_s = TK + 1
    ldb_s = TN + 1
    sa = mk.alloc_tg(TM * lda_s)
    sb = mk.alloc_tg(TK * ldb_s)
    per = TM * TN // NT            # 8 outputs per thread, along a row
    r = t // (TN // per)
    cq = (t % (TN // per)) * per
    acc = [0.0] * per
    if MUT == 10:
        acc = [mk.load(c, (row0 + r) * N + col0 + cq + j, (row0 + r < M) & (col0 + cq + j < N)) for j in range(per)]
    k_start = TK if MUT == 6 else 0
    for k0 in range(k_start, K, TK):
        for i in range(0, TM * TK, NT):
            e = t + i
            ar, ak = e // TK, e % TK
            arow = row0 + ar + 1 if MUT == 1 else row0 + ar
            rows_ok = arow + 1 < M if MUT == 7 else arow < M
            ok = rows_ok & (k0 + ak < K)
            slot = ar * lda_s + (ak + 1) % TK if MUT == 3 else ar * lda_s + ak
            mk.store(sa, slot, mk.load(a, arow * K + k0 + ak, ok))
        for i in range(0, TK * TN, NT):
            e = t + i
            bk, bc = e // TN, e % TN
            ok = (k0 + bk < K) & (col0 + bc < N)
            if MUT == 2:
                off = (k0 + bk) * (2 * N) + 2 * (col0 + bc)
            elif MUT == 9:
                off = (col0 + bc) * K + k0 + bk
            else:
                off = (k0 + bk) * N + col0 + bc
            mk.store(sb, bk * ldb_s + bc, mk.load(b, off, ok))
        mk.barrier()
        for j in range(per):
            d = mk.dot(sa, r * lda_s, 1, sb, cq + j, ldb_s, TK - 1 if MUT == 5 else TK)
            if MUT == 4:
                acc[j] = acc[j] * d
            elif MUT == 11:
                acc[j] = acc[j] + d + mk.dot(sa, r * lda_s, 1, sb, cq + j, ldb_s, TK)
            else:
                acc[j] = acc[j] + d
        mk.barrier()
    for j in range(per):
        col = col0 + cq + j + 1 if MUT == 8 else col0 + cq + j
        mk.store(c, (row0 + r) * N + col, acc[j], (row0 + r < M) & (col < N))


def grid(M: int, N: int) -> tuple[int, int, int]:
    return (-(-N // 32), -(-M // 32), 1)


def sizes(mut: int, M: int, N: int, K: int) -> dict[str, int]:
    """Elements each buffer needs so that every masked access of the mutant stays inside."""
    a = (M + 1) * K
    b = K * 2 * N if mut == 2 else max(K * N, N * K)
    return {"a": a, "b": b, "c": M * N + 1}
